"""ctypes binding of libmambo_b200.so (the sm_100a C ABI in include/mambo_b200.h).

The library is built in-tree (``make -C mambo_b200/csrc`` or
``__graft_entry__.build()``). There is no fallback: if the library is missing
or the device is not sm_100, every operator raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libmambo_b200.so"

MAMBO_OK = 0
MAMBO_EINVAL = 1
MAMBO_ENOTSUPPORTED = 2
MAMBO_ECUDA = 3
MAMBO_ETIMEOUT = 4
MAMBO_EWORKSPACE = 5

MAMBO_F32 = 0
MAMBO_BF16 = 1

MAMBO_ROUND_NEAREST_EVEN = 0
MAMBO_ROUND_TIES_DOWN = 1

MAMBO_KERNEL_AUTO = 0
MAMBO_KERNEL_GEMV = 1
MAMBO_KERNEL_GEMM = 2
MAMBO_KERNEL_GEMV_SYNC = 3
MAMBO_KERNEL_GEMM_F16 = 4
MAMBO_KERNEL_GEMM_F16_PAIR = 5
MAMBO_KERNEL_GEMM_F16_FOLD = 6
MAMBO_KERNEL_GEMM_F16_WIDE = 7

# Every symbol include/mambo_b200.h declares.
EXPORTED_SYMBOLS = (
    "mambo_version",
    "mambo_last_error",
    "mambo_device_check",
    "mambo_iq3s_prepare",
    "mambo_iq3s_packed_bytes",
    "mambo_iq3s_pack",
    "mambo_iq3s_decode",
    "mambo_quantize_mxfp8",
    "mambo_iq3s_linear",
    "mambo_iq3s_linear_workspace_bytes",
    "mambo_iq3s_linear_noalloc",
    "mambo_iq3s_linear_fused",
    "mambo_iq3s_linear_fused_workspace_bytes",
    "mambo_iq3s_linear_group",
    "mambo_iq3s_linear_group_workspace_bytes",
    "mambo_iq3s_linear_q",
    "mambo_iq3s_linear_fused_q",
    "mambo_iq3s_linear_group_q",
    "mambo_num_configs",
    "mambo_config_at",
    "mambo_default_config",
    "mambo_device_status",
    "mambo_set_wait_limit_ns",
    "mambo_selftest_wait_timeout",
    "mambo_q4k_packed_bytes",
    "mambo_q4k_pack",
    "mambo_quantize_mxfp8_sums",
    "mambo_q4k_linear_workspace_bytes",
    "mambo_q4k_linear",
    "mambo_q4k_linear_fused_workspace_bytes",
    "mambo_q4k_linear_fused",
    "mambo_q4k_linear_group_workspace_bytes",
    "mambo_q4k_linear_group",
    "mambo_ar_comm_create",
    "mambo_ar_comm_connect",
    "mambo_ar_comm_destroy",
    "mambo_iq3s_linear_fused_ar",
)

MAMBO_AR_HANDLE_BYTES = 64


class MamboIQ3SWeight(ctypes.Structure):
    _fields_ = [
        ("d", ctypes.c_void_p),
        ("qs", ctypes.c_void_p),
        ("qh", ctypes.c_void_p),
        ("signs", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("n_rows", ctypes.c_int64),
        ("n_blocks", ctypes.c_int64),
        ("packed", ctypes.c_void_p),
    ]


class MamboLinearItem(ctypes.Structure):
    """One linear of mambo_iq3s_linear_group (x [m,K] times w into out [m,N])."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("x_dtype", ctypes.c_int),
        ("ldx", ctypes.c_int64),
        ("m", ctypes.c_int64),
        ("w", ctypes.POINTER(MamboIQ3SWeight)),
        ("out", ctypes.c_void_p),
        ("out_dtype", ctypes.c_int),
        ("ldo", ctypes.c_int64),
    ]


MAMBO_MAX_GROUP = 32


class MamboQ4KItem(ctypes.Structure):
    """One Q4_K linear of mambo_q4k_linear_group (x [m,K] times the packed weight into out [m,N])."""

    _fields_ = [
        ("x", ctypes.c_void_p),
        ("x_dtype", ctypes.c_int),
        ("ldx", ctypes.c_int64),
        ("m", ctypes.c_int64),
        ("packed", ctypes.c_void_p),
        ("n_rows", ctypes.c_int64),
        ("n_blocks", ctypes.c_int64),
        ("out", ctypes.c_void_p),
        ("out_dtype", ctypes.c_int),
        ("ldo", ctypes.c_int64),
    ]


class MamboQuantOut(ctypes.Structure):
    """A linear's output quantized to MXFP8 for the next linear: q [M,N] E4M3, s [M,N/32] UE8M0."""

    _fields_ = [
        ("q", ctypes.c_void_p),
        ("ldq", ctypes.c_int64),
        ("s", ctypes.c_void_p),
        ("lds", ctypes.c_int64),
    ]


class MamboLinearConfig(ctypes.Structure):
    _fields_ = [
        ("kernel", ctypes.c_int),
        ("warps", ctypes.c_int),
        ("stages", ctypes.c_int),
        ("ctas_per_sm", ctypes.c_int),
        ("split", ctypes.c_int),
        ("loader", ctypes.c_int),
        ("prefetch", ctypes.c_int),
        ("reserved", ctypes.c_int),
    ]

    FIELDS = ("kernel", "warps", "stages", "ctas_per_sm", "split", "loader", "prefetch")

    def to_dict(self) -> dict:
        return {name: int(getattr(self, name)) for name in self.FIELDS}

    @classmethod
    def from_dict(cls, cfg: dict) -> "MamboLinearConfig":
        c = cls()
        for name in cls.FIELDS:
            if name in cfg:
                setattr(c, name, int(cfg[name]))
        return c


class MamboError(RuntimeError):
    """A C-ABI call failed; ``code`` is the MAMBO_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load libmambo_b200.so once; raise if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = os.environ.get("MAMBO_B200_LIB", str(LIB_PATH))
        if not Path(path).is_file():
            raise ImportError(
                f"libmambo_b200.so not found at {path}; build it with `make -C mambo_b200/csrc` "
                "(there is no CPU fallback)"
            )
        lib = ctypes.CDLL(path)
        vp, i64, i32, u64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_ulonglong
        sigs = {
            "mambo_version": ([], ctypes.c_char_p),
            "mambo_last_error": ([ctypes.c_char_p, ctypes.c_size_t], i32),
            "mambo_device_check": ([], i32),
            "mambo_iq3s_prepare": ([vp, i64, i64, i64, i64, i64, vp, vp, vp, vp, vp, vp], i32),
            "mambo_iq3s_packed_bytes": ([i64, i64], ctypes.c_size_t),
            "mambo_iq3s_pack": ([ctypes.POINTER(MamboIQ3SWeight), vp, vp], i32),
            "mambo_iq3s_decode": ([ctypes.POINTER(MamboIQ3SWeight), vp, vp, vp, vp], i32),
            "mambo_quantize_mxfp8": ([vp, i32, i64, i64, i64, vp, i64, vp, i64, i32, vp], i32),
            "mambo_iq3s_linear": (
                [vp, i64, vp, i64, i64, ctypes.POINTER(MamboIQ3SWeight), vp, vp, i32, i64,
                 ctypes.POINTER(MamboLinearConfig), vp, ctypes.c_size_t, vp],
                i32,
            ),
            "mambo_iq3s_linear_workspace_bytes": ([i64, i64, i64, ctypes.POINTER(MamboLinearConfig)], ctypes.c_size_t),
            "mambo_iq3s_linear_noalloc": (
                [vp, i64, vp, i64, i64, ctypes.POINTER(MamboIQ3SWeight), vp, vp, i32, i64,
                 ctypes.POINTER(MamboLinearConfig), vp],
                i32,
            ),
            "mambo_iq3s_linear_fused": (
                [vp, i32, i64, i64, ctypes.POINTER(MamboIQ3SWeight), vp, vp, i32, i64,
                 ctypes.POINTER(MamboLinearConfig), vp, ctypes.c_size_t, vp],
                i32,
            ),
            "mambo_iq3s_linear_fused_workspace_bytes": (
                [i64, i64, i64, ctypes.POINTER(MamboLinearConfig)], ctypes.c_size_t),
            "mambo_iq3s_linear_group": (
                [ctypes.POINTER(MamboLinearItem), i32, vp, vp, ctypes.c_size_t, vp], i32),
            "mambo_iq3s_linear_group_workspace_bytes": ([ctypes.POINTER(MamboLinearItem), i32], ctypes.c_size_t),
            "mambo_iq3s_linear_q": (
                [vp, i64, vp, i64, i64, ctypes.POINTER(MamboIQ3SWeight), vp, vp, i32, i64,
                 ctypes.POINTER(MamboQuantOut), ctypes.POINTER(MamboLinearConfig), vp, ctypes.c_size_t, vp],
                i32,
            ),
            "mambo_iq3s_linear_fused_q": (
                [vp, i32, i64, i64, ctypes.POINTER(MamboIQ3SWeight), vp, vp, i32, i64,
                 ctypes.POINTER(MamboQuantOut), ctypes.POINTER(MamboLinearConfig), vp, ctypes.c_size_t, vp],
                i32,
            ),
            "mambo_iq3s_linear_group_q": (
                [ctypes.POINTER(MamboLinearItem), ctypes.POINTER(MamboQuantOut), i32, vp, vp, ctypes.c_size_t, vp],
                i32),
            "mambo_num_configs": ([i32], i32),
            "mambo_config_at": ([i32, i32, ctypes.POINTER(MamboLinearConfig)], i32),
            "mambo_default_config": ([i64, i64, i64, ctypes.POINTER(MamboLinearConfig)], i32),
            "mambo_device_status": ([i32, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32)], i32),
            "mambo_set_wait_limit_ns": ([u64], i32),
            "mambo_selftest_wait_timeout": ([u64, vp], i32),
            "mambo_q4k_packed_bytes": ([i64, i64], ctypes.c_size_t),
            "mambo_q4k_pack": ([vp, i64, i64, i64, i64, i64, vp, vp], i32),
            "mambo_quantize_mxfp8_sums": ([vp, i32, i64, i64, i64, vp, i64, vp, i64, vp, i64, i32, vp], i32),
            "mambo_q4k_linear_workspace_bytes": ([i64, i64, i64, ctypes.POINTER(MamboLinearConfig)],
                                                 ctypes.c_size_t),
            "mambo_q4k_linear": (
                [vp, i64, vp, i64, vp, i64, i64, vp, i64, i64, vp, i32, i64, ctypes.POINTER(MamboLinearConfig), vp,
                 ctypes.c_size_t, vp],
                i32,
            ),
            "mambo_q4k_linear_fused_workspace_bytes": ([i64, i64, i64, ctypes.POINTER(MamboLinearConfig)],
                                                       ctypes.c_size_t),
            "mambo_q4k_linear_fused": (
                [vp, i32, i64, i64, vp, i64, i64, vp, i32, i64, ctypes.POINTER(MamboLinearConfig), vp,
                 ctypes.c_size_t, vp],
                i32,
            ),
            "mambo_q4k_linear_group_workspace_bytes": ([ctypes.POINTER(MamboQ4KItem), i32], ctypes.c_size_t),
            "mambo_q4k_linear_group": ([ctypes.POINTER(MamboQ4KItem), i32, vp, ctypes.c_size_t, vp], i32),
            "mambo_ar_comm_create": ([i32, i32, i64, ctypes.POINTER(vp), vp], i32),
            "mambo_ar_comm_connect": ([vp, vp], i32),
            "mambo_ar_comm_destroy": ([vp], i32),
            "mambo_iq3s_linear_fused_ar": (
                [vp, i32, i64, i64, ctypes.POINTER(MamboIQ3SWeight), vp, vp, i32, i64, vp,
                 ctypes.POINTER(MamboLinearConfig), vp, ctypes.c_size_t, vp],
                i32,
            ),
        }
        for name, (args, res) in sigs.items():
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = res
        _lib = lib
        return lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    load().mambo_last_error(buf, len(buf))
    return buf.value.decode("utf-8", "replace")


def check(status: int, what: str = "") -> None:
    """Map a MAMBO_* status to the reference's exception types."""
    if status == MAMBO_OK:
        return
    msg = last_error() or f"status {status}"
    if what:
        msg = f"{what}: {msg}"
    if status == MAMBO_EINVAL:
        raise ValueError(msg)
    if status == MAMBO_ENOTSUPPORTED:
        raise RuntimeError(msg)
    raise MamboError(status, msg)


def device_status(reset: bool = False) -> tuple[int, int, int]:
    code, where, block = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    check(load().mambo_device_status(1 if reset else 0, ctypes.byref(code), ctypes.byref(where), ctypes.byref(block)))
    return code.value, where.value, block.value
