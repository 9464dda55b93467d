"""ctypes bindings of the C oracle (oracle/iq3s_ref.c) -- TEST INFRASTRUCTURE ONLY.

Built by ``make -C oracle`` (``__graft_entry__.build()`` runs it) into
``oracle/_build/liboracle_iq3s.so``.
"""

from __future__ import annotations

import ctypes
import os
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

from .iq3s_oracle import IQ3_S_BLOCK_BYTES, IQ3_S_BLOCK_VALUES, iq3s_grid_u32

_LIB_PATH = Path(__file__).resolve().parent / "_build" / "liboracle_iq3s.so"
_lib = None


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.is_file():
            raise FileNotFoundError(f"C oracle not built: run `make -C {_LIB_PATH.parent.parent}`")
        lib = ctypes.CDLL(str(_LIB_PATH))
        p = ctypes.c_void_p
        i64 = ctypes.c_int64
        lib.oracle_iq3s_dequant.argtypes = [p, i64, p, p]
        lib.oracle_iq3s_dequant.restype = None
        lib.oracle_mxfp8_quantize.argtypes = [p, i64, i64, ctypes.c_int, p, p]
        lib.oracle_mxfp8_quantize.restype = None
        lib.oracle_iq3s_linear.argtypes = [p, p, i64, i64, p, i64, p, p, i64]
        lib.oracle_iq3s_linear.restype = ctypes.c_int
        _lib = lib
    return _lib


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def dequantize_iq3s(raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    n_blocks = raw.size // IQ3_S_BLOCK_BYTES
    out = np.empty(n_blocks * IQ3_S_BLOCK_VALUES, dtype=np.float32)
    grid = iq3s_grid_u32()
    _load().oracle_iq3s_dequant(_ptr(raw), n_blocks, _ptr(grid), _ptr(out))
    return out.reshape(raw.shape[0], -1) if raw.ndim == 3 else out.reshape(raw.shape[:-1] + (IQ3_S_BLOCK_VALUES,))


def quantize_mxfp8(x: np.ndarray, rounding: str = "rne") -> tuple[np.ndarray, np.ndarray]:
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    q = np.empty((m, k), dtype=np.uint8)
    s = np.empty((m, k // 32), dtype=np.uint8)
    _load().oracle_mxfp8_quantize(_ptr(x), m, k, 0 if rounding == "rne" else 1, _ptr(q), _ptr(s))
    return q, s


def iq3s_linear_f64(xq: np.ndarray, xs: np.ndarray, raw: np.ndarray, threads: int | None = None) -> np.ndarray:
    """float64 [M,N] on `threads` host threads (row-split over N)."""
    xq = np.ascontiguousarray(xq, dtype=np.uint8)
    xs = np.ascontiguousarray(xs, dtype=np.uint8)
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    m, k = xq.shape
    n = raw.shape[0]
    out = np.empty((m, n), dtype=np.float64)
    grid = iq3s_grid_u32()
    lib = _load()
    threads = max(1, min(threads or os.cpu_count() or 1, n))
    bounds = np.linspace(0, n, threads + 1).astype(np.int64)
    row_bytes = raw.strides[0]

    def work(i: int) -> int:
        r0, r1 = int(bounds[i]), int(bounds[i + 1])
        if r1 <= r0:
            return 0
        return lib.oracle_iq3s_linear(_ptr(xq), _ptr(xs), m, k, _ptr(raw) + r0 * row_bytes, r1 - r0,
                                      _ptr(grid), _ptr(out) + r0 * 8, n)

    with ThreadPoolExecutor(max_workers=threads) as pool:
        codes = list(pool.map(work, range(threads)))
    if any(codes):
        raise MemoryError("C oracle could not allocate its row buffer")
    return out
