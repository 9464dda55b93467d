"""NumPy restatement of the reference's IQ3_S x MXFP8 linear path (CPU oracle).

TEST INFRASTRUCTURE ONLY: imported by ``tests/``, ``__graft_entry__.smoke()``
and the CPU-baseline legs of ``bench.py``; never by ``mambo_b200``.

What is restated, and from where (paths relative to the Menooker/Mambo tree):

* IQ3_S codebook: ``iq3_s_table`` (src/python/mambo/kernels/iq3_s_fp8.py:63-74)
  parses ``iq3s_grid`` from the pinned llama.cpp ``ggml-common.h``. That
  submodule is absent, so the 512x4 magnitude grid is taken from the installed
  gguf-py 0.19.0 (``gguf.quants.IQ3_S.grid``), the same package the reference
  uses as its bit-exact decode oracle (tests/python/utils/compute_reference_gguf.py:80-100,245).
* E4M3 re-encoding of the codebook: ``iq3_s_fp8_table`` (iq3_s_fp8.py:77-94).
* IQ3_S block decode (ggml ``dequantize_row_iq3_s``, gguf-py
  ``IQ3_S.dequantize_blocks``): 110-byte block = fp16 d | 64 qs | 8 qh |
  32 sign bytes | 4 scale bytes; weight k of a block is
  ``d * (1 + 2*nibble(k//32)) * grid[qs[k//4] | qh_bit << 8][k%4] * sign(k)``.
* Standalone decoder outputs (signed E4M3 bytes + per-32 f32 scales):
  ``decode_iq3_s_blocks`` (iq3_s_fp8.py:202-222, helpers 105-199).
* SoA field split: ``prepare_iq3_s_fields`` (src/python/mambo/utils/iq3_s_weight.py:25-54).
* MXFP8 activation quantization: ``quantize_fp8_group`` (src/python/mambo/kernels/quantize_fp8.py:23-39)
  with round-to-nearest-even, and the reference test oracle
  ``encode_mxfp8_reference`` (tests/python/utils/fp8_reference.py:64-86), whose
  nearest-value search resolves exact ties toward the smaller magnitude.
* Linear: float64 matmul of the decoded operands
  (tests/python/test_iq3_s_fp8.py:192-198, compute_reference_gguf.py:111-121).
"""

from __future__ import annotations

from functools import lru_cache

import numpy as np

IQ3_S_BLOCK_BYTES = 110
IQ3_S_BLOCK_VALUES = 256
IQ3_S_SCALE_VALUES = 32
FP8_GROUP_K = 32
E4M3_MAX = 448.0

# Byte offsets of the fields inside one 110-byte IQ3_S block.
FIELD_LAYOUT = (("d", 0, 2), ("qs", 2, 64), ("qh", 66, 8), ("signs", 74, 32), ("scales", 106, 4))


# ----------------------------------------------------------------------------
# Codebook
# ----------------------------------------------------------------------------
@lru_cache(maxsize=1)
def iq3s_grid_u32() -> np.ndarray:
    """uint32[512]: byte j of entry i is the j-th magnitude (1,3,...,15) of code i.

    Same packing as ``iq3s_grid`` in ggml-common.h (little-endian bytes).
    """
    from gguf.quants import IQ3_S  # gguf-py 0.19.0

    IQ3_S.init_grid()
    grid = np.asarray(IQ3_S.grid, dtype=np.float32).reshape(512, 4)
    mags = grid.astype(np.uint32)
    if not np.array_equal(mags.astype(np.float32), grid):
        raise ValueError("IQ3_S grid holds non-integer magnitudes")
    return (mags[:, 0] | (mags[:, 1] << 8) | (mags[:, 2] << 16) | (mags[:, 3] << 24)).astype(np.uint32)


_MAGNITUDE_TO_E4M3 = {1: 0x38, 3: 0x44, 5: 0x4A, 7: 0x4E, 9: 0x51, 11: 0x53, 13: 0x55, 15: 0x57}


@lru_cache(maxsize=1)
def iq3s_fp8_table() -> np.ndarray:
    """uint32[512]: the codebook with every magnitude byte re-encoded as E4M3 bits."""
    raw = iq3s_grid_u32()
    lut = np.zeros(256, dtype=np.uint32)
    ok = np.zeros(256, dtype=bool)
    for mag, bits in _MAGNITUDE_TO_E4M3.items():
        lut[mag] = bits
        ok[mag] = True
    out = np.zeros_like(raw)
    for shift in (0, 8, 16, 24):
        byte = (raw >> shift) & 0xFF
        if not ok[byte].all():
            raise ValueError("IQ3_S codebook holds a magnitude without an E4M3 encoding")
        out |= lut[byte] << shift
    return out


# ----------------------------------------------------------------------------
# E4M3 / E8M0 codecs
# ----------------------------------------------------------------------------
def _e4m3_value_table() -> np.ndarray:
    codes = np.arange(256, dtype=np.int64)
    exp = (codes >> 3) & 0xF
    man = codes & 0x7
    mag = np.where(exp == 0, man * 2.0 ** -9, (1.0 + man / 8.0) * np.exp2(exp - 7.0))
    mag = np.where((exp == 15) & (man == 7), np.nan, mag)
    return np.where(codes & 0x80, -mag, mag).astype(np.float64)


_E4M3_VALUES = _e4m3_value_table()


def decode_e4m3(bits: np.ndarray) -> np.ndarray:
    """E4M3FN bit patterns -> float32 values (0x7F/0xFF decode to NaN)."""
    return _E4M3_VALUES[np.asarray(bits, dtype=np.uint8)].astype(np.float32)


def decode_e8m0(codes: np.ndarray) -> np.ndarray:
    """UE8M0 scale codes -> float32 powers of two (0xFF is NaN)."""
    c = np.asarray(codes, dtype=np.uint8).astype(np.int32)
    v = np.exp2(c.astype(np.float64) - 127.0)
    return np.where(c == 0xFF, np.nan, v).astype(np.float32)


def decode_mxfp8(q: np.ndarray, s: np.ndarray) -> np.ndarray:
    """[M,K] E4M3 bytes and [M,K/32] UE8M0 bytes -> float32 [M,K] values."""
    vals = decode_e4m3(q)
    scales = decode_e8m0(s)
    if vals.ndim != 2 or scales.shape != (vals.shape[0], vals.shape[1] // FP8_GROUP_K):
        raise ValueError("MXFP8 data and scale shapes do not match")
    return vals * np.repeat(scales, FP8_GROUP_K, axis=1)


def encode_e4m3(y: np.ndarray, rounding: str = "rne") -> np.ndarray:
    """Finite float64 values with |y| <= 448 -> E4M3FN bytes.

    ``rounding="rne"``: round to nearest, ties to even (hardware ``cvt.rn`` and
    the cuTile ``astype`` used by the reference kernel). ``rounding="ties_down"``:
    nearest value, exact ties to the smaller magnitude (the ``np.argmin`` search
    of the reference test oracle). Values above 448 saturate to 448.
    """
    y = np.asarray(y, dtype=np.float64)
    a = np.abs(y)
    mant, ex = np.frexp(a)  # a = mant * 2**ex, mant in [0.5, 1)
    e = np.where(a < 2.0 ** -6, -6, ex - 1)  # unbiased exponent; zero/subnormals use -6
    r = np.ldexp(a, 3 - e)  # a / 2**(e-3): exact
    if rounding == "rne":
        q = np.rint(r)
    elif rounding == "ties_down":
        q = np.ceil(r - 0.5)
    else:
        raise ValueError(f"unknown rounding {rounding!r}")
    # q in [0, 16]; q == 16 carries into the next binade. For e == -6 the
    # subnormal codes 0..7 and the first normal code 8 are exactly q.
    code = np.where(e == -6, q, ((e + 7) << 3) + q - 8).astype(np.int64)
    code = np.minimum(code, 0x7E)
    sign = np.signbit(y).astype(np.int64) << 7
    return (code | sign).astype(np.uint8)


def mxfp8_exponent(amax: np.ndarray) -> np.ndarray:
    """Exact ``clamp(ceil(log2(amax/448)), -127, 127)``; amax == 0 gives 0."""
    amax = np.asarray(amax, dtype=np.float64)
    mant, ex = np.frexp(amax)  # 448 = 0.875 * 2**9
    e = np.where(mant <= 0.875, ex - 9, ex - 8)
    e = np.clip(e, -127, 127)
    return np.where(amax == 0.0, 0, e).astype(np.int64)


def quantize_mxfp8(x: np.ndarray, rounding: str = "rne") -> tuple[np.ndarray, np.ndarray]:
    """[M,K] floats (K % 32 == 0) -> ([M,K] E4M3 bytes, [M,K/32] UE8M0 bytes)."""
    x = np.asarray(x)
    if x.ndim != 2 or x.shape[1] % FP8_GROUP_K:
        raise ValueError("activation must have shape [M,K] with K divisible by 32")
    m, k = x.shape
    xg = x.astype(np.float64).reshape(m, k // FP8_GROUP_K, FP8_GROUP_K)
    amax = np.abs(xg).max(axis=2)
    e = mxfp8_exponent(amax)
    y = np.ldexp(xg, -e[..., None])
    q = encode_e4m3(y, rounding).reshape(m, k)
    return q, (e + 127).astype(np.uint8)


# ----------------------------------------------------------------------------
# IQ3_S decode
# ----------------------------------------------------------------------------
def _split_blocks(raw: np.ndarray):
    raw = np.ascontiguousarray(np.asarray(raw, dtype=np.uint8))
    if raw.shape[-1] != IQ3_S_BLOCK_BYTES:
        raise ValueError("IQ3_S blocks must have 110 bytes")
    d = raw[..., 0:2].copy().view(np.float16)[..., 0].astype(np.float32)
    qs = raw[..., 2:66].astype(np.uint32)
    qh = raw[..., 66:74].astype(np.uint32)
    signs = raw[..., 74:106].astype(np.uint32)
    scales = raw[..., 106:110].astype(np.uint32)
    return d, qs, qh, signs, scales


def iq3s_group_scales(raw: np.ndarray) -> np.ndarray:
    """[..., 110] blocks -> float32 [..., 8] group scales d * (1 + 2*nibble)."""
    d, _, _, _, scales = _split_blocks(raw)
    nib = np.stack([(scales[..., g // 2] >> (4 * (g % 2))) & 0xF for g in range(8)], axis=-1)
    return d[..., None] * (1.0 + 2.0 * nib.astype(np.float32))


def iq3s_signed_codes(raw: np.ndarray) -> np.ndarray:
    """[..., 110] blocks -> uint8 [..., 256] signed E4M3 bytes of the grid magnitudes."""
    _, qs, qh, signs, _ = _split_blocks(raw)
    c = np.arange(64)
    hbit = (qh[..., c // 8] >> (c % 8)) & 1
    idx = qs | (hbit << 8)  # [..., 64]
    words = iq3s_fp8_table()[idx]  # [..., 64] four E4M3 bytes per code
    k = np.arange(256)
    mag = (words[..., k // 4] >> (8 * (k % 4))) & 0xFF
    sbit = (signs[..., k // 8] >> (k % 8)) & 1
    return (mag | (sbit << 7)).astype(np.uint8)


def dequantize_iq3s(raw: np.ndarray) -> np.ndarray:
    """[N,B,110] (or [...,110]) blocks -> float32 [N, B*256] (or [..., 256]) weights."""
    raw = np.asarray(raw, dtype=np.uint8)
    vals = decode_e4m3(iq3s_signed_codes(raw))  # exact +-{1..15}
    scales = iq3s_group_scales(raw)
    w = vals * np.repeat(scales, IQ3_S_SCALE_VALUES, axis=-1)
    if raw.ndim == 3:
        return w.reshape(raw.shape[0], -1)
    return w


def decode_iq3s_fp8(raw: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """[N,B,110] -> (uint8 [N,K] signed E4M3 bytes, float32 [N,K/32] scales).

    The outputs of the reference's ``launch_dequant_iq3_s`` (iq3_s_fp8.py:341-351).
    """
    raw = np.asarray(raw, dtype=np.uint8)
    n = raw.shape[0]
    return iq3s_signed_codes(raw).reshape(n, -1), iq3s_group_scales(raw).reshape(n, -1)


def prepare_fields(raw: np.ndarray) -> dict[str, np.ndarray]:
    """[N,B,110] -> byte-preserving SoA fields with the reference dtypes/shapes."""
    raw = np.asarray(raw, dtype=np.uint8)
    n, b, _ = raw.shape

    def field(off, size, dtype):
        return np.ascontiguousarray(raw[..., off:off + size].transpose(1, 0, 2)).view(dtype)

    return {
        "d": field(0, 2, np.float16).reshape(b, n),
        "qs": field(2, 64, np.uint32),
        "qh": field(66, 8, np.uint16),
        "signs": field(74, 32, np.int32),
        "scales": field(106, 4, np.uint32).reshape(b, n),
    }


# ----------------------------------------------------------------------------
# Linear
# ----------------------------------------------------------------------------
def iq3s_linear_f64(xq: np.ndarray, xs: np.ndarray, raw: np.ndarray) -> np.ndarray:
    """float64 [M,N] = decode_mxfp8(xq, xs) @ dequantize_iq3s(raw).T."""
    x = decode_mxfp8(xq, xs).astype(np.float64)
    w = dequantize_iq3s(raw).astype(np.float64)
    return x @ w.T


def relative_frobenius(a: np.ndarray, ref: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = float(np.sqrt(np.sum(ref * ref)))
    return float(np.sqrt(np.sum((a - ref) ** 2)) / (den if den > 0 else 1.0))


# ----------------------------------------------------------------------------
# Seeded synthetic inputs
# ----------------------------------------------------------------------------
def make_synthetic_iq3s(n_rows: int, k: int, seed: int, d_low: float = 1e-3, d_high: float = 1e-2) -> np.ndarray:
    """uint8 [N, K/256, 110]: uniform random bytes with a positive fp16 d.

    Same construction as the reference's ``make_synthetic_iq3_s``
    (tests/python/test_iq3_s_fp8.py:41-51); the d range defaults to the
    benchmark's U[1e-3, 1e-2] (the reference's test uses U[0.002, 0.04]).
    """
    if k % IQ3_S_BLOCK_VALUES:
        raise ValueError("IQ3_S K must be divisible by 256")
    blocks = k // IQ3_S_BLOCK_VALUES
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(n_rows, blocks, IQ3_S_BLOCK_BYTES), dtype=np.uint8)
    d = rng.uniform(d_low, d_high, size=(n_rows, blocks)).astype("<f2")
    raw[..., :2] = d.view(np.uint8).reshape(n_rows, blocks, 2)
    return raw


def make_all_codes_iq3s() -> np.ndarray:
    """uint8 [8, 16, 110]: every codebook entry with all 16 sign nibbles, d = 1.

    The known-answer case of tests/python/test_iq3_s_fp8.py:105-117.
    """
    n_rows, blocks = 8, 16
    raw = np.zeros((n_rows, blocks, IQ3_S_BLOCK_BYTES), dtype=np.uint8)
    raw[..., :2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    code = (np.arange(8192, dtype=np.uint16) % 512).reshape(n_rows, blocks, 64)
    sign = (np.arange(8192, dtype=np.uint16) // 512).reshape(n_rows, blocks, 64)
    raw[..., 2:66] = code.astype(np.uint8)
    raw[..., 66:74] = np.packbits((code >> 8).astype(np.uint8), axis=-1, bitorder="little")
    raw[..., 74:106] = (sign[..., 0::2] | (sign[..., 1::2] << 4)).astype(np.uint8)
    return raw


def mxfp8_edge_rows(x: np.ndarray) -> np.ndarray:
    """Overwrite rows 0..4 with the reference's MXFP8 edge cases (test_iq3_s_fp8.py:154-161)."""
    x = np.array(x, dtype=np.float32, copy=True)
    x[0, :] = 0.0
    x[1, 0] = 32.0
    x[2, 32 + 7] = -64.0
    x[3, :32] *= 1.0e-4
    x[3, 32:64] = np.float32(2.0 ** -130)
    x[4, 64:96] = np.linspace(-12.0, 12.0, FP8_GROUP_K, dtype=np.float32)
    return x
