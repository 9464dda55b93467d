"""CPU: the oracle's Q4_K and IQ4_XS decoders (oracle/gguf_quants_oracle.py)
pinned bit for bit against gguf-py 0.19.0's dequantization, the format's own
package (the reference's decode oracle for GGUF types,
tests/python/utils/compute_reference_gguf.py:80-100). These two types are the
next ones for the decode + block-scaled MMA skeleton (the reference's type
table, src/python/mambo/utils/gguf_manifest.py:30-42).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gguf_quants_oracle as G
from mambo_b200.utils.gguf_weight import read_model_weight

CASES = [("Q4_K", G.dequantize_q4_k, G.Q4_K_BLOCK_BYTES), ("IQ4_XS", G.dequantize_iq4_xs, G.IQ4_XS_BLOCK_BYTES)]


def _reference(raw: np.ndarray, type_name: str) -> np.ndarray:
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    return dequantize(raw, GGMLQuantizationType[type_name]).reshape(-1).astype(np.float32)


def _blocks(rng, n_blocks: int, block_bytes: int, f16_fields: int) -> np.ndarray:
    """Random blocks whose leading fp16 fields are finite scales in [1e-4, 1e-1), either sign."""
    raw = rng.integers(0, 256, size=(n_blocks, block_bytes), dtype=np.uint8)
    for f in range(f16_fields):
        v = (rng.uniform(1e-4, 1e-1, n_blocks) * rng.choice([-1, 1], n_blocks)).astype("<f2")
        raw[:, 2 * f:2 * f + 2] = v.view(np.uint8).reshape(n_blocks, 2)
    return raw


@pytest.mark.parametrize("type_name,decode,block_bytes", CASES)
def test_decode_equals_gguf_py(type_name, decode, block_bytes):
    rng = np.random.default_rng(0x4B)
    raw = _blocks(rng, 4096, block_bytes, 2 if type_name == "Q4_K" else 1)
    assert np.array_equal(decode(raw), _reference(raw, type_name))


@pytest.mark.parametrize("type_name,decode,block_bytes", CASES)
def test_decode_equals_gguf_py_on_every_bit_pattern(type_name, decode, block_bytes):
    """Fully random bytes: scales include zeros, subnormals, infinities and NaNs."""
    raw = np.random.default_rng(0x4C).integers(0, 256, size=(8192, block_bytes), dtype=np.uint8)
    with np.errstate(invalid="ignore", over="ignore"):  # inf * 0 on both sides
        ours, ref = decode(raw), _reference(raw, type_name)
    assert np.array_equal(ours, ref, equal_nan=True)


def test_q4_k_tensor_read_from_a_gguf_file(tmp_path, write_gguf):
    raw = _blocks(np.random.default_rng(5), 48 * 2, G.Q4_K_BLOCK_BYTES, 2).reshape(48, -1)
    path = write_gguf(tmp_path / "q4k.gguf", {"blk.0.ffn_up.weight": (raw, "Q4_K")})
    packed, n, k = read_model_weight(path, "blk.0.ffn_up.weight", expected_type="q4_k")
    assert (n, k) == (48, 512) and packed.shape == (48, 2, G.Q4_K_BLOCK_BYTES)
    assert np.array_equal(G.dequantize_q4_k(packed), _reference(raw, "Q4_K"))


def test_partial_blocks_are_rejected():
    with pytest.raises(ValueError):
        G.dequantize_q4_k(np.zeros(G.Q4_K_BLOCK_BYTES + 1, dtype=np.uint8))
    with pytest.raises(ValueError):
        G.dequantize_iq4_xs(np.zeros(G.IQ4_XS_BLOCK_BYTES - 1, dtype=np.uint8))


def test_q4_k_group_decomposition_equals_the_direct_product():
    """The planned Q4_K kernel arithmetic (exact E4M3 codes, per-group scale and the
    min term through the activation's group sums) gives the dequantized product."""
    from oracle import iq3s_oracle as O

    rng = np.random.default_rng(0x4D)
    raw = _blocks(rng, 64 * 4, G.Q4_K_BLOCK_BYTES, 2).reshape(64, 4, G.Q4_K_BLOCK_BYTES)
    x = rng.standard_normal((6, 1024)).astype(np.float32)
    xq, xs = O.quantize_mxfp8(x)
    xe = O.decode_mxfp8(xq, xs)  # the MXFP8 activations the kernel multiplies
    direct = G.q4_k_linear_f64(xe, raw)
    split = G.q4_k_linear_group_decomposed(xe, raw)
    assert O.relative_frobenius(split, direct) < 1e-12
    # gguf-py's float32 weights round each value: the same product within float32 rounding.
    w32 = G.dequantize_q4_k(raw).reshape(64, -1).astype(np.float64)
    assert O.relative_frobenius(xe.astype(np.float64) @ w32.T, direct) < 1e-7


def test_iq4_xs_fp16_operands_are_exact_and_the_decomposition_holds():
    from oracle import iq3s_oracle as O

    values = G.iq4_nl_values().astype(np.float64)
    assert np.array_equal(values.astype(np.float16).astype(np.float64), values)
    rng = np.random.default_rng(0x4E)
    raw = _blocks(rng, 32 * 4, G.IQ4_XS_BLOCK_BYTES, 1).reshape(32, 4, G.IQ4_XS_BLOCK_BYTES)
    x = rng.standard_normal((5, 1024))
    direct = x @ G.dequantize_iq4_xs(raw).reshape(32, -1).astype(np.float64).T
    assert O.relative_frobenius(G.iq4_xs_linear_group_decomposed(x, raw), direct) < 1e-12
