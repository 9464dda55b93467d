"""Tensor-parallel IQ3_S x MXFP8 linears: one process per GPU, NCCL collectives.

The projection shards without splitting a quantization block:

* column split (QKV, gate, up): rank r holds weight rows [n0, n1) -- a slice
  of every IQ3_S block row, no exchange inside the linear -- and produces
  out[:, n0:n1]; an all-gather along N gives the full output when asked.
* row split (O, down): rank r holds K blocks [b0, b1) of every row (super-
  blocks of 256 weights, so an MXFP8 group of 32 never straddles ranks) and
  the matching K slice of the activations, and produces an FP32 partial of
  the full output; an all-reduce (sum) combines the partials.

Shard sizes: N is split into multiples of 8 rows (the packed weight records),
K into whole 256-weight blocks; ``K % (256 * world) == 0`` and
``N % (8 * world) == 0`` are required, as for every Llama-3 shape.

The collectives go through ``torch.distributed`` (NCCL on GPUs, gloo in the
CPU tests). The per-rank compute is the single-GPU path of this package;
``linear``/``quantize`` can be replaced (the CPU tests plug in a restatement).

At decode sizes (M < 32) a row split can instead run its all-reduce inside the
GEMV launch (:class:`FusedAllReduce`, ``TensorParallelIQ3SLinear.fused``):
each row tile's partial goes straight into every rank's exchange buffer over
NVLink and every rank sums all partials in rank order, with no NCCL call.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist

COLUMN = "column"
ROW = "row"


class FusedAllReduce:
    """This rank's side of the fused row-split all-reduce.

    Allocates an exchange buffer on the current GPU for outputs of up to
    ``max_rows`` rows (the C ABI's mambo_ar_comm_create), all-gathers the
    buffers' CUDA IPC handles over ``group`` and maps every peer's buffer
    (mambo_ar_comm_connect). Every rank must then issue the same sequence of
    fused linears on it (same shapes), on one stream per rank. ``close()``
    releases the mappings and the buffer.
    """

    def __init__(self, max_rows: int, group=None):
        import ctypes

        from . import _lib

        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.max_rows = (max_rows + 127) // 128 * 128
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        handle = ctypes.create_string_buffer(_lib.MAMBO_AR_HANDLE_BYTES)
        comm = ctypes.c_void_p()
        _lib.check(lib.mambo_ar_comm_create(self.world, self.rank, self.max_rows, ctypes.byref(comm), handle),
                   "mambo_ar_comm_create")
        self.handle = comm
        handles = [bytes(handle.raw)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
        try:
            _lib.check(lib.mambo_ar_comm_connect(comm, b"".join(handles)), "mambo_ar_comm_connect")
        except Exception:
            lib.mambo_ar_comm_destroy(comm)
            self.handle = None
            raise

    def close(self) -> None:
        if self.handle is not None:
            from . import _lib

            _lib.load().mambo_ar_comm_destroy(self.handle)
            self.handle = None


def shard_range(total: int, rank: int, world: int, unit: int) -> tuple[int, int]:
    """[start, end) of rank's equal share of `total` items, in whole `unit`s."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} is not in a world of {world}")
    if total % (unit * world):
        raise ValueError(f"{total} does not split into {world} shards of whole {unit}-item units")
    per = total // world
    return rank * per, (rank + 1) * per


def shard_iq3_s_blocks(raw: torch.Tensor, mode: str, rank: int, world: int) -> torch.Tensor:
    """This rank's slice of GGUF IQ3_S blocks uint8 [N, K/256, 110] (a view; prepare it afterwards)."""
    if raw.ndim != 3 or raw.shape[2] != 110:
        raise ValueError("IQ3_S weight must be uint8 [N,K/256,110]")
    if mode == COLUMN:
        n0, n1 = shard_range(raw.shape[0], rank, world, 8)
        return raw[n0:n1]
    if mode == ROW:
        b0, b1 = shard_range(raw.shape[1], rank, world, 1)
        return raw[:, b0:b1]
    raise ValueError(f"mode must be {COLUMN!r} or {ROW!r}")


def _default_quantize(x: torch.Tensor):
    from .kernels.quantize_fp8 import launch_quantize_fp8

    return launch_quantize_fp8(x)


def _default_linear(xq: torch.Tensor, xs: torch.Tensor, fields, out_dtype: torch.dtype) -> torch.Tensor:
    from .kernels.iq3_s_fp8 import launch_iq3_s_fp8_matmul

    return launch_iq3_s_fp8_matmul(xq, xs, fields, out_dtype=out_dtype)


def _default_prepare(raw: torch.Tensor):
    from .utils.iq3_s_weight import prepare_iq3_s_fields

    return prepare_iq3_s_fields(raw)


@dataclass
class CollectiveTimes:
    """Device time of the last forward's collective (ms), when timing was asked for."""

    collective_ms: float = 0.0


class TensorParallelIQ3SLinear:
    """One rank's shard of an IQ3_S x MXFP8 linear y = x @ W^T.

    ``raw``: the FULL uint8 [N, K/256, 110] weight (each rank keeps only its
    slice) or, with ``raw_is_shard``, this rank's slice already.
    ``mode``: COLUMN or ROW. ``gather_output`` (COLUMN): all-gather the
    [M, N/P] shards into [M, N]. ``input_is_sharded`` (ROW): the activation
    passed to forward is this rank's K slice [M, K/P] instead of [M, K].
    """

    def __init__(self, raw: torch.Tensor, mode: str, *, group=None, raw_is_shard: bool = False,
                 gather_output: bool = True, input_is_sharded: bool = False,
                 out_dtype: torch.dtype = torch.bfloat16,
                 prepare: Callable | None = None, quantize: Callable | None = None, linear: Callable | None = None):
        if mode not in (COLUMN, ROW):
            raise ValueError(f"mode must be {COLUMN!r} or {ROW!r}")
        if out_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
        self.mode = mode
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.gather_output = gather_output
        self.input_is_sharded = input_is_sharded
        self.out_dtype = out_dtype
        self._quantize = quantize or _default_quantize
        self._linear = linear or _default_linear
        # With the library's own kernels, quantization and linear are one call
        # (one launch at decode sizes: the GEMV quantizes its bf16 rows itself).
        self._fused = quantize is None and linear is None
        if raw_is_shard:
            local = raw
            full_n = raw.shape[0] * (self.world if mode == COLUMN else 1)
            full_b = raw.shape[1] * (self.world if mode == ROW else 1)
        else:
            local = shard_iq3_s_blocks(raw, mode, self.rank, self.world)
            full_n, full_b = raw.shape[0], raw.shape[1]
        self.n, self.k = full_n, full_b * 256
        self.local_n, self.local_k = local.shape[0], local.shape[1] * 256
        if mode == COLUMN:
            self.n0 = self.rank * self.local_n
            self.k0 = 0
        else:
            self.n0 = 0
            self.k0 = self.rank * self.local_k
        self.fields = (prepare or _default_prepare)(local)
        self.times = CollectiveTimes()

    def forward(self, x: torch.Tensor, *, time_collective: bool = False, gather: bool | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """x: [M, K] (or [M, K/P] for a row split with sharded input) -> [M, N] (or [M, N/P]).

        ``gather`` (COLUMN) and ``out_dtype`` override the instance's settings for this call.
        """
        return self.combine(self.local(x, out_dtype=out_dtype), time_collective=time_collective, gather=gather,
                            out_dtype=out_dtype)

    def local(self, x: torch.Tensor, *, out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """This rank's compute: COLUMN -> out[:, n0:n1] in out_dtype; ROW -> the FP32 partial [M, N]."""
        if x.ndim != 2:
            raise ValueError("activation must be [M,K]")
        if self.mode == COLUMN:
            if x.shape[1] != self.k:
                raise ValueError(f"column-split activation must be [M,{self.k}]")
            return self._quantized_linear(x, out_dtype or self.out_dtype)
        # Row split: this rank's K slice (whole 256-weight blocks: MXFP8 groups stay intact).
        if self.input_is_sharded:
            if x.shape[1] != self.local_k:
                raise ValueError(f"sharded row-split activation must be [M,{self.local_k}]")
            return self._quantized_linear(x, torch.float32)
        if x.shape[1] != self.k:
            raise ValueError(f"row-split activation must be [M,{self.k}]")
        return self._quantized_linear(x[:, self.k0:self.k0 + self.local_k], torch.float32)

    def _quantized_linear(self, x: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
        if self._fused and x.dtype in (torch.float32, torch.bfloat16):
            from .kernels.iq3_s_fp8 import iq3_s_fp8_linear

            return iq3_s_fp8_linear(x, self.fields, out_dtype=out_dtype)
        xq, xs = self._quantize(x)
        return self._linear(xq, xs, self.fields, out_dtype)

    def combine(self, y: torch.Tensor, *, time_collective: bool = False, gather: bool | None = None,
                out_dtype: torch.dtype | None = None) -> torch.Tensor:
        """The exchange step on local()'s result: all-gather (COLUMN, when asked) or all-reduce (ROW)."""
        if self.mode == COLUMN:
            if not (self.gather_output if gather is None else gather) or self.world == 1:
                return y
            return self._timed(time_collective, lambda: self._gather_columns(y))
        if self.world > 1:
            self._timed(time_collective, lambda: dist.all_reduce(y, op=dist.ReduceOp.SUM, group=self.group))
        dtype = out_dtype or self.out_dtype
        return y if dtype == torch.float32 else y.to(dtype)

    __call__ = forward

    def fused(self, x: torch.Tensor, comm: FusedAllReduce, *, out_dtype: torch.dtype | None = None,
              out: torch.Tensor | None = None) -> torch.Tensor:
        """Row split at decode sizes: this rank's GEMV and the sum over ranks in one launch.

        ``x``: [M, K] (or [M, K/P] with ``input_is_sharded``), bf16, M < 32.
        Returns the full [M, N] output, identical on every rank.
        """
        from .kernels.iq3_s_fp8 import fused_linear_ar_into

        if self.mode != ROW:
            raise ValueError("the fused all-reduce applies to a row split")
        if x.ndim != 2 or x.dtype != torch.bfloat16:
            raise ValueError("activation must be bf16 [M,K]")
        if not self.input_is_sharded:
            if x.shape[1] != self.k:
                raise ValueError(f"row-split activation must be [M,{self.k}]")
            x = x[:, self.k0:self.k0 + self.local_k]
        elif x.shape[1] != self.local_k:
            raise ValueError(f"sharded row-split activation must be [M,{self.local_k}]")
        dtype = out_dtype or self.out_dtype
        if out is None:
            out = torch.empty((x.shape[0], self.n), dtype=dtype, device=x.device)
        return fused_linear_ar_into(x, self.fields, out, comm)

    def _gather_columns(self, y: torch.Tensor) -> torch.Tensor:
        if dist.get_backend(self.group) == "nccl":
            # One buffer: the [M, N/P] shards land as [P, M, N/P]; one permuting copy makes [M, N].
            m, nl = y.shape
            parts = torch.empty((self.world, m, nl), dtype=y.dtype, device=y.device)
            dist.all_gather_into_tensor(parts, y.contiguous(), group=self.group)
            return parts.permute(1, 0, 2).reshape(m, self.world * nl)
        parts = [torch.empty_like(y) for _ in range(self.world)]
        dist.all_gather(parts, y.contiguous(), group=self.group)
        return torch.cat(parts, dim=1)

    def _timed(self, on: bool, fn):
        if not on or not torch.cuda.is_available():
            return fn()
        dev = torch.cuda.current_device()
        s = torch.cuda.current_stream(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        out = fn()
        e1.record(s)
        e1.synchronize()
        self.times.collective_ms = e0.elapsed_time(e1)
        return out


def local_group(linears, x: torch.Tensor) -> list:
    """local() of several COLUMN shards that read the same activation (gate and
    up, or separate Q, K, V weights) as one grouped launch on this rank.

    Returns each shard's [M, N/P] output; pass each to its own combine().
    Falls back to one local() per shard unless all use the library's kernels.
    """
    if not linears:
        return []
    if any(lin.mode != COLUMN or not lin._fused or lin.k != linears[0].k for lin in linears) \
            or x.dtype not in (torch.float32, torch.bfloat16):
        return [lin.local(x) for lin in linears]
    if x.ndim != 2 or x.shape[1] != linears[0].k:
        raise ValueError(f"column-split activation must be [M,{linears[0].k}]")
    from .kernels.iq3_s_fp8 import group_linear_into

    if x.stride(1) != 1:
        x = x.contiguous()
    outs = [torch.empty((x.shape[0], lin.local_n), dtype=lin.out_dtype, device=x.device) for lin in linears]
    return group_linear_into([x] * len(linears), [lin.fields for lin in linears], outs)


def gather_columns_group(linears, ys: list) -> list:
    """combine(gather=True) of several COLUMN shards' outputs with ONE all-gather.

    ``ys[i]``: linears[i]'s [M, N_i/P] output (same M and dtype for all).
    Returns the [M, N_i] outputs, in order.
    """
    if not ys:
        return []
    lin0 = linears[0]
    if lin0.world == 1:
        return list(ys)
    m, dtype = ys[0].shape[0], ys[0].dtype
    widths = [y.shape[1] for y in ys]
    send = torch.cat([y.reshape(-1) for y in ys])
    parts = torch.empty((lin0.world, send.numel()), dtype=dtype, device=send.device)
    if dist.get_backend(lin0.group) == "nccl":
        dist.all_gather_into_tensor(parts, send, group=lin0.group)
    else:
        chunks = list(parts.unbind(0))
        dist.all_gather(chunks, send, group=lin0.group)
    outs, off = [], 0
    for w in widths:
        blk = parts[:, off:off + m * w].reshape(lin0.world, m, w)
        outs.append(blk.permute(1, 0, 2).reshape(m, lin0.world * w))
        off += m * w
    return outs
