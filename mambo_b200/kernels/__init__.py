"""Operator API of the IQ3_S x MXFP8 linear path (mirror of mambo.kernels)."""
