"""Weight preparation and autotuning utilities (mirror of mambo.utils)."""
