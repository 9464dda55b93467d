"""IQ3_S weights split into per-field arrays for the sm_100a kernels.

Drop-in for src/python/mambo/utils/iq3_s_weight.py (Menooker/Mambo): the class,
field names, dtypes, shapes and exception types are the reference's API; the
arrays are torch CUDA tensors and the split itself is a kernel of
libmambo_b200 (``mambo_iq3s_prepare``).

A GGUF IQ3_S tensor stores, for each row, one 110-byte record per 256 weights
along K. The record starts with the FP16 scale d, followed by 64 bytes that
give the low eight bits of the 64 nine-bit codebook indices (one index per
four weights), 8 bytes of ninth index bits, 32 bytes of sign bits (one per
weight) and 4 bytes holding eight 4-bit group scales. A weight of group g
(32 weights) is sign * codebook magnitude * d * (1 + 2 * scale_g).
"""

from __future__ import annotations

import dataclasses
from dataclasses import dataclass

import torch

from .. import _lib, _runtime


@dataclass(frozen=True)
class IQ3SFields:
    """The fields of every record, each in its own array indexed [K block, row, ...] (iq3_s_weight.py:10-22).

    The bytes are the GGUF ones, regrouped: d as float16 [B,N], the index low
    bytes as uint32 [B,N,16], the ninth bits as uint16 [B,N,4], the sign bits
    as int32 [B,N,8] and the group scales as uint32 [B,N] (B = K/256). Built
    once by prepare_iq3_s_fields and then passed to every launch.
    """

    d: torch.Tensor
    qs: torch.Tensor
    qh: torch.Tensor
    signs: torch.Tensor
    scales: torch.Tensor
    # Addition of this build: the same bytes in tile-major records (one copy per
    # GEMV work unit), made by prepare_iq3_s_fields; None when not built.
    packed: torch.Tensor | None = None


def prepare_iq3_s_fields(iq3_weight, *, stream=None, packed: bool = True, soa: bool = True) -> IQ3SFields:
    """Split GGUF uint8 [N,B,110] blocks into aligned SoA fields once (iq3_s_weight.py:25-54).

    Accepts any strides and address alignment of the source view. The copy is
    outside kernel timing. With ``packed`` (and N % 8 == 0) it also builds the
    tile-major copy the tcgen05 GEMV streams with one copy per work unit; that
    doubles the weight memory. ``soa=False`` (needs ``packed`` and N % 8 == 0)
    keeps only the packed copy plus the small d and scales fields: qs, qh and
    signs become empty [B,N,0] tensors (104 of the 110 bytes per block freed).
    Every linear runs on such a weight; the standalone decoder
    (launch_dequant_iq3_s) and the legacy MAMBO_KERNEL_GEMV_SYNC kernel need
    the SoA fields and raise.
    """
    raw = _runtime.as_cuda_tensor(iq3_weight)
    if raw.ndim != 3 or raw.dtype != torch.uint8 or raw.shape[2] != 110:
        raise ValueError("IQ3_S weight must be uint8 [N,K/256,110]")
    n, blocks, _ = raw.shape
    if n < 1 or blocks < 1:
        raise ValueError("IQ3_S weight must have positive N and K")
    if not soa and (not packed or n % 8):
        raise ValueError("soa=False keeps only the packed copy: it needs packed=True and N % 8 == 0")
    dev = raw.device
    _runtime.require_device(dev)
    mk = lambda *shape: torch.empty(shape, dtype=torch.uint8, device=dev)  # noqa: E731
    d, qs, qh, signs, scales = mk(blocks, n, 2), mk(blocks, n, 64), mk(blocks, n, 8), mk(blocks, n, 32), mk(blocks, n, 4)
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        _lib.check(
            _lib.load().mambo_iq3s_prepare(
                raw.data_ptr(), n, blocks, raw.stride(0), raw.stride(1), raw.stride(2),
                d.data_ptr(), qs.data_ptr(), qh.data_ptr(), signs.data_ptr(), scales.data_ptr(), st,
            ),
            "prepare_iq3_s_fields",
        )
    fields = IQ3SFields(
        d.view(torch.float16).reshape(blocks, n),
        qs.view(torch.uint32),
        qh.view(torch.uint16),
        signs.view(torch.int32),
        scales.view(torch.uint32).reshape(blocks, n),
    )
    if packed and n % 8 == 0:
        fields = pack_iq3_s_fields(fields, stream=stream)
    if not soa:
        # The packed copy holds every byte; keep d and scales (dimensions, C-ABI checks) and free the rest.
        fields = dataclasses.replace(
            fields, qs=torch.empty((blocks, n, 0), dtype=torch.uint32, device=dev),
            qh=torch.empty((blocks, n, 0), dtype=torch.uint16, device=dev),
            signs=torch.empty((blocks, n, 0), dtype=torch.int32, device=dev))
    return fields


def has_soa_fields(iq3_weight: IQ3SFields) -> bool:
    """False for weights prepared with soa=False (only the packed copy carries qs, qh and signs)."""
    return iq3_weight.qs.numel() > 0


def pack_iq3_s_fields(fields: IQ3SFields, *, stream=None) -> IQ3SFields:
    """Return ``fields`` with the tile-major packed copy built (mambo_iq3s_pack)."""
    n, blocks = _weight_dimensions(fields)
    lib = _lib.load()
    dev = fields.d.device
    buf = torch.empty(lib.mambo_iq3s_packed_bytes(n, blocks), dtype=torch.uint8, device=dev)
    w = weight_struct(fields)
    with torch.cuda.device(dev):
        _lib.check(lib.mambo_iq3s_pack(w, buf.data_ptr(), _runtime.stream_handle(stream, dev)), "pack_iq3_s_fields")
    return dataclasses.replace(fields, packed=buf)


def _weight_dimensions(iq3_weight: IQ3SFields) -> tuple[int, int]:
    """(rows N, K blocks B) of prepared fields; TypeError for anything else (iq3_s_weight.py:57-62)."""
    if not isinstance(iq3_weight, IQ3SFields):
        raise TypeError("prepare IQ3_S weights with prepare_iq3_s_fields before launch")
    blocks, n_rows = iq3_weight.d.shape
    return n_rows, blocks


def _weight_kernel_args(iq3_weight: IQ3SFields) -> tuple[torch.Tensor, ...]:
    return (iq3_weight.d, iq3_weight.qs, iq3_weight.qh, iq3_weight.signs, iq3_weight.scales)


def _large_weight_kernel_args(iq3_weight: IQ3SFields) -> tuple[torch.Tensor, ...]:
    """The fields with the ninth bits viewed as uint32 [B,N,2] and the signs flattened per K block
    to int32 [B,N*8], without copying (iq3_s_weight.py:69-77)."""
    return (iq3_weight.d, iq3_weight.qs, iq3_weight.qh.view(torch.uint32),
            iq3_weight.signs.reshape(iq3_weight.signs.shape[0], -1), iq3_weight.scales)


def weight_struct(iq3_weight: IQ3SFields) -> _lib.MamboIQ3SWeight:
    """The C-ABI view of prepared fields (validates contiguity and shapes)."""
    n, b = _weight_dimensions(iq3_weight)
    expect = {
        "d": ((b, n), torch.float16),
        "qs": ((b, n, 16), torch.uint32),
        "qh": ((b, n, 4), torch.uint16),
        "signs": ((b, n, 8), torch.int32),
        "scales": ((b, n), torch.uint32),
    }
    packed = getattr(iq3_weight, "packed", None)
    dropped = packed is not None and iq3_weight.qs.numel() == 0  # prepared with soa=False
    for name, (shape, dtype) in expect.items():
        t = getattr(iq3_weight, name)
        if dropped and name in ("qs", "qh", "signs"):
            shape = shape[:2] + (0,)
        if tuple(t.shape) != shape or t.dtype != dtype or not t.is_contiguous() or not t.is_cuda:
            raise ValueError(f"IQ3SFields.{name} must be a contiguous CUDA {dtype} tensor of shape {shape}")
    w = _lib.MamboIQ3SWeight()
    w.d, w.scales = iq3_weight.d.data_ptr(), iq3_weight.scales.data_ptr()
    if not dropped:
        w.qs, w.qh, w.signs = iq3_weight.qs.data_ptr(), iq3_weight.qh.data_ptr(), iq3_weight.signs.data_ptr()
    w.n_rows, w.n_blocks = n, b
    w.packed = packed.data_ptr() if packed is not None else None
    return w


def fields_nbytes(iq3_weight: IQ3SFields) -> int:
    return sum(t.numel() * t.element_size() for t in _weight_kernel_args(iq3_weight))


__all__ = ["IQ3SFields", "prepare_iq3_s_fields", "weight_struct", "fields_nbytes"]
