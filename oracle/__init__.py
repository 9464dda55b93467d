"""CPU oracle for the IQ3_S x MXFP8 linear path -- TEST INFRASTRUCTURE ONLY.

Nothing in ``mambo_b200`` imports this package. Only ``tests/``, the
``smoke()`` check in ``__graft_entry__.py`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may use it, and only as the checker
or as the timed CPU baseline -- never as the thing measured or shipped.

Parity pin: the numpy restatement in :mod:`oracle.iq3s_oracle` is checked in
``tests/test_oracle.py`` against golden vectors under ``tests/golden`` that
were produced by the reference's own oracles (gguf-py 0.19.0 ``dequantize``
for IQ3_S and the reference's ``tests/python/utils/fp8_reference.py`` for
MXFP8), see ``tests/golden/make_golden.py``.
"""
