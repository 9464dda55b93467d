"""NumPy restatement of two more GGUF block formats' decode (CPU oracle):
Q4_K and IQ4_XS, the next quant types for the same decode-into-operand +
block-scaled-MMA skeleton as IQ3_S.

TEST INFRASTRUCTURE ONLY: imported by ``tests/``; never by ``mambo_b200``.

The reference lists these types in its GGUF tensor-type table
(src/python/mambo/utils/gguf_manifest.py:30-42) but has no kernel for them.
Their decoders live in ggml (``dequantize_row_q4_K``, ``dequantize_row_iq4_xs``
in the pinned llama.cpp submodule, absent here) and in gguf-py 0.19.0
(``gguf.quants.Q4_K`` / ``IQ4_XS``, installed). What follows restates the
published block layouts; ``tests/test_gguf_quants_oracle.py`` pins both
decoders bit for bit against gguf-py's dequantization.

* Q4_K, 144 bytes per 256 values: fp16 d | fp16 dmin | 12 bytes holding eight
  6-bit scales and eight 6-bit mins | 128 bytes of 4-bit codes. Sub-block j
  (32 values) has scale s_j and min m_j:
  j < 4:  s_j = b[j] & 63,                       m_j = b[j+4] & 63;
  j >= 4: s_j = (b[j+4] & 15) | (b[j-4] >> 6) << 4, m_j = (b[j+4] >> 4) | (b[j] >> 6) << 4.
  Code bytes 32c..32c+31 hold sub-block 2c in their low nibbles and 2c+1 in
  their high nibbles. Value = d*s_j*q - dmin*m_j.
* IQ4_XS, 136 bytes per 256 values: fp16 d | uint16 scales_h | 4 bytes
  scales_l | 128 bytes of 4-bit indices. Sub-block j has the 6-bit scale
  l_j = (scales_l[j/2] >> 4*(j%2)) & 15 | ((scales_h >> 2j) & 3) << 4; its 16
  code bytes (16j..16j+15) hold values 0-15 in the low nibbles and 16-31 in
  the high ones. Value = d*(l_j - 32)*kvalues[index], with kvalues the
  16-entry non-linear table of IQ4_NL, taken from gguf-py (the format's own
  package) as the IQ3_S grid is.
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np

Q4_K_BLOCK_BYTES = 144
IQ4_XS_BLOCK_BYTES = 136
BLOCK_VALUES = 256


def _blocks(raw: np.ndarray, block_bytes: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    if raw.size % block_bytes:
        raise ValueError(f"byte count {raw.size} is not a whole number of {block_bytes}-byte blocks")
    return raw.reshape(-1, block_bytes)


def _f16(blocks: np.ndarray, offset: int) -> np.ndarray:
    """The little-endian float16 at ``offset`` of every block, as float32 [n, 1]."""
    return blocks[:, offset:offset + 2].copy().view("<f2").astype(np.float32)


def _nibbles(codes: np.ndarray, chunk: int) -> np.ndarray:
    """Bytes [n, c*chunk] -> 4-bit values [n, c*2*chunk]: per chunk, the low nibbles then the high ones."""
    n = codes.shape[0]
    c = codes.reshape(n, -1, chunk)
    return np.concatenate([c & 15, c >> 4], axis=2).reshape(n, -1)


def q4_k_scales_mins(b: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """The 12 packed scale bytes of each block [n, 12] -> 6-bit scales and mins, each [n, 8]."""
    b = b.astype(np.uint8)
    lo = b[:, 0:4], b[:, 4:8], b[:, 8:12]
    s = np.empty((b.shape[0], 8), dtype=np.uint8)
    m = np.empty_like(s)
    s[:, :4] = lo[0] & 63
    m[:, :4] = lo[1] & 63
    s[:, 4:] = (lo[2] & 15) | ((lo[0] >> 6) << 4)
    m[:, 4:] = (lo[2] >> 4) | ((lo[1] >> 6) << 4)
    return s, m


def dequantize_q4_k(raw: np.ndarray, dtype=np.float32) -> np.ndarray:
    """Q4_K blocks (any shape whose bytes are whole 144-byte blocks) -> ``dtype`` [blocks * 256].

    float32 rounds each weight as gguf-py and ggml do; float64 is exact (fp16
    scales times 6-bit and 4-bit integers).
    """
    blk = _blocks(raw, Q4_K_BLOCK_BYTES)
    d, dmin = _f16(blk, 0).astype(dtype), _f16(blk, 2).astype(dtype)
    s, m = q4_k_scales_mins(blk[:, 4:16])
    q = _nibbles(blk[:, 16:144], 32).reshape(-1, 8, 32).astype(dtype)
    scale = (d * s.astype(dtype))[:, :, None]
    offset = (dmin * m.astype(dtype))[:, :, None]
    return (scale * q - offset).reshape(-1)


@lru_cache(maxsize=1)
def iq4_nl_values() -> np.ndarray:
    """The 16 non-linear values of the IQ4_NL / IQ4_XS codebook (int8), from gguf-py 0.19.0."""
    from gguf.quants import IQ4_NL

    return np.asarray(IQ4_NL.kvalues, dtype=np.int8)


def iq4_xs_scales(blk: np.ndarray) -> np.ndarray:
    """6-bit sub-block scales of each IQ4_XS block [n, 136] -> [n, 8] (0..63)."""
    h = blk[:, 2:4].copy().view("<u2").astype(np.uint32)  # [n, 1]
    low = blk[:, 4:8].astype(np.uint32)
    j = np.arange(8)
    l_lo = (low[:, j // 2] >> (4 * (j % 2))) & 15
    l_hi = (h >> (2 * j)) & 3
    return (l_lo | (l_hi << 4)).astype(np.int32)


def dequantize_iq4_xs(raw: np.ndarray) -> np.ndarray:
    """IQ4_XS blocks (whole 136-byte blocks) -> float32 [blocks * 256]."""
    blk = _blocks(raw, IQ4_XS_BLOCK_BYTES)
    d = _f16(blk, 0)
    dl = d * (iq4_xs_scales(blk) - 32).astype(np.float32)  # [n, 8]
    idx = _nibbles(blk[:, 8:136], 16).reshape(-1, 8, 32)
    v = iq4_nl_values()[idx].astype(np.float32)
    return (dl[:, :, None] * v).reshape(-1)


def make_synthetic_q4_k(n_rows: int, k: int, seed: int, d_low: float = 1e-4, d_high: float = 1e-2) -> np.ndarray:
    """uint8 [N, K/256, 144]: uniform random scale, min and code bytes with finite fp16 d and dmin of
    either sign, |d|, |dmin| in [d_low, d_high) (test input, not a property of the format)."""
    if k % BLOCK_VALUES:
        raise ValueError("Q4_K K must be divisible by 256")
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(n_rows, k // BLOCK_VALUES, Q4_K_BLOCK_BYTES), dtype=np.uint8)
    for f in range(2):
        v = rng.uniform(d_low, d_high, size=raw.shape[:2]) * rng.choice([-1.0, 1.0], size=raw.shape[:2])
        raw[..., 2 * f:2 * f + 2] = v.astype("<f2").view(np.uint8).reshape(*raw.shape[:2], 2)
    return raw


def q4_k_linear_f64(x: np.ndarray, raw: np.ndarray) -> np.ndarray:
    """Direct reference: float64 ``x [M, K] @ W.T`` with the exact (float64) weights of raw [N, K/256, 144]."""
    n = raw.shape[0]
    w = dequantize_q4_k(raw, np.float64).reshape(n, -1)
    return np.asarray(x, dtype=np.float64) @ w.T


def q4_k_linear_group_decomposed(x: np.ndarray, raw: np.ndarray) -> np.ndarray:
    """The same product as the FP8 GEMV skeleton would form it, in float64.

    Per 32-value group g of row r: P = sum x * code (the codes 0..15 are exact
    E4M3 operands, so this is the tensor core's group partial), then
    out += d*s_g * P - dmin*m_g * sum x (the epilogue, with the activation's
    group sums from the quantizing warps).
    """
    x = np.asarray(x, dtype=np.float64)
    m_tokens, k = x.shape
    blk = _blocks(raw, Q4_K_BLOCK_BYTES)  # [N * K/256, 144]
    n = raw.shape[0]
    d, dmin = _f16(blk, 0).astype(np.float64), _f16(blk, 2).astype(np.float64)
    s, mn = q4_k_scales_mins(blk[:, 4:16])
    codes = _nibbles(blk[:, 16:144], 32).reshape(n, k // 32, 32).astype(np.float64)
    scale = (d * s).reshape(n, k // 32)            # d * s_g per (row, group)
    offset = (dmin * mn).reshape(n, k // 32)       # dmin * m_g per (row, group)
    xg = x.reshape(m_tokens, k // 32, 32)
    partial = np.einsum("tgj,rgj->trg", xg, codes)  # tensor-core group partials
    xsum = xg.sum(axis=2)                            # [M, K/32] activation group sums
    return np.einsum("trg,rg->tr", partial, scale) - xsum @ offset.T


def iq4_xs_linear_group_decomposed(x: np.ndarray, raw: np.ndarray) -> np.ndarray:
    """IQ4_XS product as an FP16-operand kernel would form it, in float64.

    The operand is the table value itself (an integer of magnitude <= 127, exact
    in FP16, not always in E4M3); per 32-value group g of row r: P = sum x * value,
    then out += d*(l_g - 32) * P in the epilogue.
    """
    x = np.asarray(x, dtype=np.float64)
    m_tokens, k = x.shape
    n = raw.shape[0]
    blk = _blocks(raw, IQ4_XS_BLOCK_BYTES)
    operand = iq4_nl_values().astype(np.float16)[_nibbles(blk[:, 8:136], 16)]  # FP16 operands
    operand = operand.reshape(n, k // 32, 32).astype(np.float64)
    scale = (_f16(blk, 0).astype(np.float64) * (iq4_xs_scales(blk) - 32)).reshape(n, k // 32)
    partial = np.einsum("tgj,rgj->trg", x.reshape(m_tokens, k // 32, 32), operand)
    return np.einsum("trg,rg->tr", partial, scale)
