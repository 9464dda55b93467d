"""Generate the golden vectors under tests/golden from the reference's own oracles.

Run where a checkout of the reference tree is readable and gguf-py is
installed, with MAMBO_REFERENCE_ROOT naming the checkout's root directory:

    MAMBO_REFERENCE_ROOT=<path to Menooker/Mambo> python tests/golden/make_golden.py

Sources of truth (paths relative to the Menooker/Mambo tree):
* IQ3_S decode: gguf-py 0.19.0 ``gguf.quants.dequantize`` -- the decoder the
  reference's tests use (tests/python/test_iq3_s_fp8.py:84-131,
  tests/python/utils/compute_reference_gguf.py:80-100), and which
  compute_reference_gguf.py:245 asserts equal to ggml's C decode.
* MXFP8: ``encode_mxfp8_reference`` / ``decode_mxfp8`` from
  tests/python/utils/fp8_reference.py, imported from the reference tree; plus
  an ml_dtypes ``float8_e4m3fn`` cast (round-to-nearest-even) for the RNE rule.
* Linear: float64 matmul of the decoded operands (test_iq3_s_fp8.py:192-198).

Inputs follow the reference tests' shapes and seeds; activations use NumPy's
default_rng with the reference's seeds (the reference drew them with CuPy,
which is not available here).
"""

from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _reference_root() -> Path:
    root = os.environ.get("MAMBO_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set MAMBO_REFERENCE_ROOT to the root of a Menooker/Mambo checkout")
    return Path(root)


def _load_fp8_reference():
    path = _reference_root() / "tests" / "python" / "utils" / "fp8_reference.py"
    spec = importlib.util.spec_from_file_location("mambo_ref_fp8_reference", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def synthetic_iq3s(n_rows: int, k: int, seed: int, lo: float, hi: float) -> np.ndarray:
    """Same construction as the reference's make_synthetic_iq3_s (test_iq3_s_fp8.py:41-51)."""
    blocks = k // 256
    rng = np.random.default_rng(seed)
    raw = rng.integers(0, 256, size=(n_rows, blocks, 110), dtype=np.uint8)
    d = rng.uniform(lo, hi, size=(n_rows, blocks)).astype("<f2")
    raw[..., :2] = d.view(np.uint8).reshape(n_rows, blocks, 2)
    return raw


def all_codes_iq3s() -> np.ndarray:
    """Every codebook entry with all 16 sign nibbles, d = 1 (test_iq3_s_fp8.py:105-117)."""
    n_rows, blocks = 8, 16
    raw = np.zeros((n_rows, blocks, 110), dtype=np.uint8)
    raw[..., :2] = np.array([1.0], dtype=np.float16).view(np.uint8)
    code = (np.arange(8192, dtype=np.uint16) % 512).reshape(n_rows, blocks, 64)
    sign = (np.arange(8192, dtype=np.uint16) // 512).reshape(n_rows, blocks, 64)
    raw[..., 2:66] = code.astype(np.uint8)
    raw[..., 66:74] = np.packbits((code >> 8).astype(np.uint8), axis=-1, bitorder="little")
    raw[..., 74:106] = (sign[..., 0::2] | (sign[..., 1::2] << 4)).astype(np.uint8)
    return raw


def edge_rows(x: np.ndarray) -> np.ndarray:
    """The reference's MXFP8 edge rows (test_iq3_s_fp8.py:156-161)."""
    x = x.copy()
    x[0, :] = 0.0
    x[1, 0] = 32.0
    x[2, 32 + 7] = -64.0
    x[3, :32] *= 1.0e-4
    x[3, 32:64] = np.float32(2.0 ** -130)
    x[4, 64:96] = np.linspace(-12.0, 12.0, 32, dtype=np.float32)
    return x


def mxfp8_rne(x: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """RNE E4M3 bytes of x / 2^e using ml_dtypes (independent of the oracle's encoder)."""
    import ml_dtypes

    m, k = x.shape
    e = scales.astype(np.int64) - 127
    y = np.ldexp(x.astype(np.float64).reshape(m, k // 32, 32), -e[..., None]).astype(np.float32)
    return y.astype(ml_dtypes.float8_e4m3fn).view(np.uint8).reshape(m, k)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main() -> None:
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    fp8 = _load_fp8_reference()

    def deq(raw):
        return dequantize(np.ascontiguousarray(raw.reshape(raw.shape[0], -1)), GGMLQuantizationType.IQ3_S)

    # --- IQ3_S decode --------------------------------------------------------
    synth = synthetic_iq3s(5, 768, 0x1A3, 0.002, 0.04)
    codes = all_codes_iq3s()
    soa = synthetic_iq3s(7, 768, 0x50A, 0.002, 0.04)
    np.savez_compressed(
        HERE / "golden_iq3s_decode.npz",
        synth_raw=synth, synth_deq=deq(synth),
        allcodes_raw=codes, allcodes_deq=deq(codes),
        soa_raw=soa,
    )

    # --- MXFP8 ---------------------------------------------------------------
    mx = {}
    for m in (5, 33, 128):
        rng = np.random.default_rng(20261015)
        x = edge_rows(rng.standard_normal((m, 160), dtype=np.float32))
        q, s = fp8.encode_mxfp8_reference(x)
        mx[f"x_{m}"] = x
        mx[f"q_{m}"] = q
        mx[f"s_{m}"] = s
        mx[f"q_rne_{m}"] = mxfp8_rne(x, s)
    # bf16-valued activations: the two tie rules differ here.
    rng = np.random.default_rng(20261017)
    xb = rng.standard_normal((16, 512), dtype=np.float32)
    xb_bits = (xb.view(np.uint32) >> 16).astype(np.uint16)  # truncate to bf16 values
    xb_f32 = (xb_bits.astype(np.uint32) << 16).view(np.float32)
    qb, sb = fp8.encode_mxfp8_reference(xb_f32)
    mx.update(xbf16_bits=xb_bits, q_bf16_ties_down=qb, s_bf16=sb, q_bf16_rne=mxfp8_rne(xb_f32, sb))
    np.savez_compressed(HERE / "golden_mxfp8.npz", **mx)

    # --- Linear --------------------------------------------------------------
    lin_raw = synthetic_iq3s(7, 768, 0x3F8, 0.002, 0.04)
    w = deq(lin_raw).astype(np.float64)
    lin = {"raw": lin_raw}
    for m in (3, 4, 5, 8, 9, 33, 128, 129):
        rng = np.random.default_rng(20261016)
        x = rng.standard_normal((m, 768), dtype=np.float32)
        q, s = fp8.encode_mxfp8_reference(x)
        xe = fp8.decode_mxfp8(q, s).astype(np.float64)
        lin[f"x_sha_{m}"] = np.frombuffer(sha(x).encode(), dtype=np.uint8)
        lin[f"q_{m}"] = q
        lin[f"s_{m}"] = s
        lin[f"out_{m}"] = (xe @ w.T).astype(np.float32)
    np.savez_compressed(HERE / "golden_linear.npz", **lin)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    sys.exit(main())
