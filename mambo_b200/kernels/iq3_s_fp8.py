"""IQ3_S block decode and IQ3_S x MXFP8 projection on sm_100a (B200).

Mirror of src/python/mambo/kernels/iq3_s_fp8.py (Menooker/Mambo): the same
constants, codebook helpers, launch wrappers, errors and benchmark-case
factory. The kernels are hand-written CUDA in libmambo_b200.so:

* decode-sized M (< LARGE_TOKEN_THRESHOLD): a weight-streaming tcgen05 GEMV
  that bulk-copies tile-major IQ3_S records, decodes them into E4M3 bytes in
  tensor memory and splits K across all SMs (stream-K with a deterministic
  fixup, or a thread-block-cluster K split). Each 32-weight group is one
  block-scaled FP8 MMA (the activation's UE8M0 scale applied by the tensor
  core) and its FP32 partial is scaled by d*(1+2*nibble) in the epilogue --
  the reference's arithmetic.
* prefill-sized M (>= LARGE_TOKEN_THRESHOLD): by default a tcgen05 GEMM with
  FP16 operands over 128-row x 128-token tiles. The group factor (1+2*nibble)
  is folded into the FP16 weight operand and the activations enter as FP16
  relative to each token's largest MXFP8 scale (both exact), so one FP32
  accumulator covers a whole 256-wide K block and the epilogue applies d per
  block. The reference's per-group decomposition (one block-scaled FP8 MMA
  per group, FP32 rescale) is the non-default ``MAMBO_KERNEL_GEMM``.
* the standalone decoder used by the bit-exactness tests.

Layout of one GGUF IQ3_S block (256 consecutive weights of a row, 110 bytes):
the FP16 base scale d first (2 bytes); then the low eight bits of the 64
codebook indices (one byte each, 64 bytes); then their ninth bits packed
eight to a byte (8 bytes); then one sign bit per weight (32 bytes); and last
the eight 4-bit group scales (4 bytes).
"""

from __future__ import annotations

import ctypes
import dataclasses
import json
import os
import re
import threading
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

from .. import _lib, _runtime
from ..utils.iq3_s_weight import (
    IQ3SFields,
    _weight_dimensions,
    prepare_iq3_s_fields,
    weight_struct,
)

IQ3_S_BLOCK_BYTES = 110
IQ3_S_BLOCK_VALUES = 256
IQ3_S_SCALE_VALUES = 32

# Tuned on B200 for the Llama-3-8B projection shapes (decode M <= 8). Keys
# follow the reference convention: GPU SM version, then medium/large by M.
BEST_CONFIGS = {
    "sm100": {
        # split: the thread-block-cluster K split while every 128-row tile gets
        # its own CTAs (select_config), stream-K beyond that.
        "medium": {"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": 8, "ctas_per_sm": 1, "split": 2,
                   "prefetch": 0},
        # AUTO: the GEMM where it applies (packed weights, 16-byte aligned
        # activation rows), else the GEMV in 32-token chunks.
        "large": {"kernel": _lib.MAMBO_KERNEL_AUTO, "warps": 8, "stages": 4, "ctas_per_sm": 1, "split": 0},
    },
}
LARGE_TOKEN_THRESHOLD = 32

_IQ3_TABLES: dict[int, torch.Tensor] = {}
_TABLE_LOCK = threading.Lock()
_TUNED: dict[tuple[int, int, int], dict] = {}


# ----------------------------------------------------------------------------
# Codebook
# ----------------------------------------------------------------------------
@lru_cache(maxsize=1)
def iq3_s_table() -> np.ndarray:
    """The 512-entry IQ3_S codebook (uint32, four magnitude bytes each).

    Like the reference (iq3_s_fp8.py:63-74) it is read from llama.cpp's
    ``ggml-common.h`` when MAMBO_LLAMA_SOURCE_DIR points at a llama.cpp tree;
    otherwise from the installed gguf-py, whose IQ3_S grid is the same table.
    """
    src = os.environ.get("MAMBO_LLAMA_SOURCE_DIR")
    if src:
        header = Path(src) / "ggml" / "src" / "ggml-common.h"
        if header.is_file():
            text = header.read_text(encoding="utf-8")
            match = re.search(r"GGML_TABLE_BEGIN\(uint32_t, iq3s_grid, 512\)(.*?)GGML_TABLE_END\(\)", text, re.S)
            if match is None:
                raise ValueError(f"IQ3_S lookup table was not found in {header}")
            values = np.asarray([int(s, 16) for s in re.findall(r"0x[0-9a-fA-F]+", match.group(1))], dtype=np.uint32)
            if values.shape != (512,):
                raise ValueError(f"expected 512 IQ3_S table entries, got {values.size}")
            return values
    from gguf.quants import IQ3_S  # the GGUF format's own Python package

    IQ3_S.init_grid()
    grid = np.asarray(IQ3_S.grid, dtype=np.float32).reshape(512, 4).astype(np.uint32)
    return (grid[:, 0] | (grid[:, 1] << 8) | (grid[:, 2] << 16) | (grid[:, 3] << 24)).astype(np.uint32)


def _e4m3_bits(value: int) -> int | None:
    """Bit pattern of a positive integer in FP8 E4M3 (bias 7, 3 mantissa bits), None if it is not exact.

    value = 2^p * (8 + m) / 8 with m < 8 gives exponent field p + 7 and mantissa m.
    """
    if value < 1:
        return None
    p = value.bit_length() - 1
    if p > 8 or (p > 3 and value % (1 << (p - 3))):
        return None
    m = (value << 3 >> p) - 8
    return ((p + 7) << 3) | m


@lru_cache(maxsize=1)
def iq3_s_fp8_table() -> np.ndarray:
    """The codebook with each magnitude byte replaced by its E4M3 bit pattern (iq3_s_fp8.py:77-94).

    The IQ3_S magnitudes are small odd integers, all exact in E4M3; the sign
    bit (bit 7) stays clear and the kernels set it from the weight's sign bit.
    """
    encode = np.zeros(256, dtype=np.uint32)
    exact = np.zeros(256, dtype=np.bool_)
    for v in range(1, 256):
        bits = _e4m3_bits(v)
        if bits is not None:
            encode[v], exact[v] = bits, True
    table = iq3_s_table()
    out = np.zeros(table.shape, dtype=np.uint32)
    for byte in range(4):
        mag = (table >> (8 * byte)) & 0xFF
        if not exact[mag].all():
            raise ValueError("IQ3_S codebook contains a magnitude without an E4M3 encoding")
        out |= encode[mag] << (8 * byte)
    return out


def _get_iq3_table(device: torch.device | None = None) -> torch.Tensor:
    """Upload the FP8-encoded codebook once per CUDA device (iq3_s_fp8.py:97-102)."""
    index = torch.cuda.current_device() if device is None or device.index is None else device.index
    with _TABLE_LOCK:
        table = _IQ3_TABLES.get(index)
        if table is None:
            host = torch.from_numpy(iq3_s_fp8_table().view(np.int32).copy())
            table = host.to(torch.device("cuda", index)).view(torch.uint32)
            _IQ3_TABLES[index] = table
    return table


def _power_of_two(value: int, name: str) -> None:
    if value < 1 or value & (value - 1):
        raise ValueError(f"{name} must be a positive power of two")


# ----------------------------------------------------------------------------
# Standalone decoder
# ----------------------------------------------------------------------------
def launch_dequant_iq3_s(iq3_weight: IQ3SFields, *, tile_n: int = 1, stream=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Return [N,K] E4M3 bit patterns and [N,K/32] original F32 scales (iq3_s_fp8.py:341-351)."""
    _power_of_two(tile_n, "tile_n")
    n_rows, blocks = _weight_dimensions(iq3_weight)
    if iq3_weight.qs.numel() == 0:
        raise ValueError("the decoder reads the SoA fields, which a weight prepared with soa=False does not keep")
    w = weight_struct(iq3_weight)
    dev = iq3_weight.d.device
    _runtime.require_device(dev)
    values = torch.empty((n_rows, blocks * 256), dtype=torch.uint8, device=dev)
    scales = torch.empty((n_rows, blocks * 8), dtype=torch.float32, device=dev)
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        _lib.check(_lib.load().mambo_iq3s_decode(w, _get_iq3_table(dev).data_ptr(), values.data_ptr(),
                                                  scales.data_ptr(), st), "launch_dequant_iq3_s")
    return values, scales


# ----------------------------------------------------------------------------
# Linear
# ----------------------------------------------------------------------------
def _sm_key(device: torch.device) -> str:
    major, minor = torch.cuda.get_device_capability(device)
    return f"sm{major}{minor}"


def _m_bucket(m: int) -> int:
    """Token counts that share a tuned configuration: up to 8, 16 and 31 (the GEMV's
    token tiles), then powers of two from LARGE_TOKEN_THRESHOLD (the GEMM)."""
    if m <= 8:
        return 8
    if m <= 16:
        return 16
    if m < LARGE_TOKEN_THRESHOLD:
        return LARGE_TOKEN_THRESHOLD - 1
    b = LARGE_TOKEN_THRESHOLD
    while b < m:
        b *= 2
    return b


def register_tuned_config(m: int, n: int, k: int, config: dict) -> None:
    """Record the autotuner's choice for a shape; launches consult it before BEST_CONFIGS."""
    _TUNED[(_m_bucket(m), int(n), int(k))] = dict(config)


def load_tuned_configs(path: str | os.PathLike) -> int:
    """Load a JSON list of {"m","n","k","config"} records written by the autotuner."""
    records = json.loads(Path(path).read_text())
    for rec in records:
        register_tuned_config(rec["m"], rec["n"], rec["k"], rec["config"])
    return len(records)


# Configurations tuned on B200 by ``python -m mambo_b200.utils.kernel_benchmark`` for the
# Llama-3 projection shapes; loaded the first time a configuration is selected.
TUNED_CONFIGS_PATH = Path(__file__).resolve().parent / "tuned_sm100.json"
_TUNED_LOADED = False


def _load_packaged_tuned() -> None:
    global _TUNED_LOADED
    if _TUNED_LOADED:
        return
    _TUNED_LOADED = True
    if TUNED_CONFIGS_PATH.is_file():
        # Records registered explicitly before this point take precedence.
        explicit = dict(_TUNED)
        load_tuned_configs(TUNED_CONFIGS_PATH)
        _TUNED.update(explicit)


def select_config(m: int, n: int, k: int, device: torch.device, *, tuned: bool = True) -> dict:
    """The configuration a launch uses: the autotuner's record for (M bucket, N, K) if any, else BEST_CONFIGS."""
    if tuned and _sm_key(device) == "sm100":
        _load_packaged_tuned()
    rec = _TUNED.get((_m_bucket(m), n, k)) if tuned else None
    if rec is not None:
        return rec
    sm = _sm_key(device)
    if sm not in BEST_CONFIGS:
        raise RuntimeError(f"IQ3_S FP8 matmul has no tuned config for {sm}")
    cfg = BEST_CONFIGS[sm]["medium" if m < LARGE_TOKEN_THRESHOLD else "large"]
    if cfg.get("split") == 2 and (n + 127) // 128 > _sm_count(device):
        cfg = dict(cfg, split=0)
    return cfg


@lru_cache(maxsize=None)
def _sm_count(device: torch.device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


def _quant_out_struct(qout) -> "_lib.MamboQuantOut | None":
    """(q uint8 [M,N], s uint8 [M,N/32]) -> the C ABI's MamboQuantOut (None: no quantized output)."""
    if qout is None:
        return None
    q, sc = qout
    qo = _lib.MamboQuantOut()
    qo.q, qo.ldq, qo.s, qo.lds = q.data_ptr(), q.stride(0), sc.data_ptr(), sc.stride(0)
    return qo


def _new_quant_out(m: int, n: int, dev) -> tuple[torch.Tensor, torch.Tensor]:
    if n % IQ3_S_SCALE_VALUES:
        raise ValueError("quantize_output needs N divisible by 32")
    return (torch.empty((m, n), dtype=torch.uint8, device=dev),
            torch.empty((m, n // IQ3_S_SCALE_VALUES), dtype=torch.uint8, device=dev))


def linear_into(x_values: torch.Tensor, x_scales: torch.Tensor, iq3_weight: IQ3SFields, out: torch.Tensor,
                config: dict | None = None, stream=None, qout=None) -> torch.Tensor:
    """Launch the linear into a preallocated out [M,N] (f32 or bf16). No validation of x beyond the C ABI's."""
    n_rows, blocks = _weight_dimensions(iq3_weight)
    m = x_values.shape[0]
    dev = x_values.device
    cfg = _lib.MamboLinearConfig.from_dict(config if config is not None else select_config(m, n_rows, blocks * 256,
                                                                                              dev))
    w = weight_struct(iq3_weight)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        need = lib.mambo_iq3s_linear_workspace_bytes(m, n_rows, blocks, cfg)
        ws = _runtime.workspace(dev, st, need)
        out_dtype = _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32
        _lib.check(
            lib.mambo_iq3s_linear_q(
                x_values.data_ptr(), x_values.stride(0), x_scales.data_ptr(), x_scales.stride(0), m, w,
                _get_iq3_table(dev).data_ptr(), out.data_ptr(), out_dtype, out.stride(0), _quant_out_struct(qout),
                cfg, ws.data_ptr(), ws.numel(), st,
            ),
            "launch_iq3_s_fp8_matmul",
        )
    return out


def launch_iq3_s_fp8_matmul(x_values, x_scales, iq3_weight: IQ3SFields, *, stream=None,
                            out_dtype: torch.dtype = torch.float32, config: dict | None = None,
                            quantize_output: bool = False):
    """Multiply prepared SoA weights by prequantized MXFP8 activations (iq3_s_fp8.py:364-399).

    Returns float32 [M,N] by default (``out_dtype=torch.bfloat16`` for the bf16
    epilogue). Activation views with a non-unit column stride are copied to
    contiguous memory first. ``quantize_output``: also return the output's
    MXFP8 quantization for the next linear, ``(out, (q, s))`` -- what
    ``launch_quantize_fp8(out)`` gives, formed in the GEMV's epilogue below 32
    tokens (N divisible by 32).
    """
    n_rows, k_blocks = _weight_dimensions(iq3_weight)
    k = k_blocks * 256
    x_values = _runtime.as_cuda_tensor(x_values)
    x_scales = _runtime.as_cuda_tensor(x_scales)
    if x_values.ndim != 2 or x_values.dtype != torch.uint8 or x_values.shape[0] < 1 or x_values.shape[1] != k:
        raise ValueError("x_values must be uint8 [M,K]")
    if tuple(x_scales.shape) != (x_values.shape[0], k // 32) or x_scales.dtype != torch.uint8:
        raise ValueError("x_scales must be uint8 [M,K/32]")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    dev = x_values.device
    if _sm_key(dev) not in BEST_CONFIGS:
        raise RuntimeError(f"IQ3_S FP8 matmul has no tuned config for {_sm_key(dev)}")
    _runtime.require_device(dev)
    if x_values.stride(1) != 1:
        x_values = x_values.contiguous()
    if x_scales.stride(1) != 1:
        x_scales = x_scales.contiguous()
    out = torch.empty((x_values.shape[0], n_rows), dtype=out_dtype, device=dev)
    if quantize_output:
        qout = _new_quant_out(x_values.shape[0], n_rows, dev)
        return linear_into(x_values, x_scales, iq3_weight, out, config=config, stream=stream, qout=qout), qout
    return linear_into(x_values, x_scales, iq3_weight, out, config=config, stream=stream)


def fused_linear_into(x: torch.Tensor, iq3_weight: IQ3SFields, out: torch.Tensor, config: dict | None = None,
                      stream=None, qout=None) -> torch.Tensor:
    """Quantize (round to nearest even) and multiply in one C-ABI call into a preallocated out [M,N].

    Below 32 tokens with bf16 rows the tcgen05 GEMV quantizes the activations
    itself (one launch); otherwise the quantizer runs into the workspace first.
    """
    n_rows, blocks = _weight_dimensions(iq3_weight)
    m = x.shape[0]
    dev = x.device
    cfg = _lib.MamboLinearConfig.from_dict(config if config is not None else select_config(m, n_rows, blocks * 256,
                                                                                              dev))
    w = weight_struct(iq3_weight)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        need = lib.mambo_iq3s_linear_fused_workspace_bytes(m, n_rows, blocks, cfg)
        ws = _runtime.workspace(dev, st, need)
        x_dtype = _lib.MAMBO_BF16 if x.dtype == torch.bfloat16 else _lib.MAMBO_F32
        out_dtype = _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32
        _lib.check(
            lib.mambo_iq3s_linear_fused_q(
                x.data_ptr(), x_dtype, x.stride(0), m, w, _get_iq3_table(dev).data_ptr(), out.data_ptr(), out_dtype,
                out.stride(0), _quant_out_struct(qout), cfg, ws.data_ptr(), ws.numel(), st,
            ),
            "iq3_s_fp8_linear",
        )
    return out


def fused_linear_ar_into(x: torch.Tensor, iq3_weight: IQ3SFields, out: torch.Tensor, comm, config: dict | None = None,
                         stream=None) -> torch.Tensor:
    """A row-split linear and its all-reduce in one launch (mambo_iq3s_linear_fused_ar).

    ``x``: this rank's bf16 K slice [M, K/world] (M < 32); ``iq3_weight``: its
    shard [N, K/world]; ``comm``: a :class:`mambo_b200.sharding.FusedAllReduce`.
    ``out`` [M, N] receives the sum over all ranks (identical on every rank).
    """
    n_rows, blocks = _weight_dimensions(iq3_weight)
    m = x.shape[0]
    dev = x.device
    cfg = _lib.MamboLinearConfig.from_dict(config if config is not None else select_config(m, n_rows, blocks * 256,
                                                                                              dev))
    w = weight_struct(iq3_weight)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        need = lib.mambo_iq3s_linear_fused_workspace_bytes(m, n_rows, blocks, cfg)
        ws = _runtime.workspace(dev, st, need)
        out_dtype = _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32
        _lib.check(
            lib.mambo_iq3s_linear_fused_ar(
                x.data_ptr(), _lib.MAMBO_BF16, x.stride(0), m, w, _get_iq3_table(dev).data_ptr(), out.data_ptr(),
                out_dtype, out.stride(0), comm.handle, cfg, ws.data_ptr(), ws.numel(), st,
            ),
            "fused all-reduce linear",
        )
    return out


def iq3_s_fp8_linear(x, iq3_weight: IQ3SFields, *, stream=None, out_dtype: torch.dtype = torch.bfloat16,
                     rounding: str = "nearest_even", config: dict | None = None, quantize_output: bool = False):
    """bf16/f32 activations [M,K] -> MXFP8 -> IQ3_S linear -> out_dtype [M,N] (quantize + matmul).

    Round-to-nearest-even goes through the fused entry point (quantization inside
    the decode GEMV below 32 tokens, inside the GEMM's FP16 pass from 32); the
    other rounding modes quantize first. ``quantize_output``: return
    ``(out, (q, s))`` with the output's MXFP8 quantization for the next linear
    (see launch_iq3_s_fp8_matmul).
    """
    from .quantize_fp8 import launch_quantize_fp8

    if rounding != "nearest_even":
        xq, xs = launch_quantize_fp8(x, stream=stream, rounding=rounding)
        return launch_iq3_s_fp8_matmul(xq, xs, iq3_weight, stream=stream, out_dtype=out_dtype, config=config,
                                       quantize_output=quantize_output)
    n_rows, k_blocks = _weight_dimensions(iq3_weight)
    x = _runtime.as_cuda_tensor(x)
    if x.ndim != 2 or x.dtype not in (torch.float32, torch.bfloat16) or x.shape[0] < 1 or x.shape[1] != k_blocks * 256:
        raise ValueError("activation must be float32 or bfloat16 [M,K] with K = 256 * weight blocks")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    dev = x.device
    if _sm_key(dev) not in BEST_CONFIGS:
        raise RuntimeError(f"IQ3_S FP8 matmul has no tuned config for {_sm_key(dev)}")
    _runtime.require_device(dev)
    if x.stride(1) != 1:
        x = x.contiguous()
    out = torch.empty((x.shape[0], n_rows), dtype=out_dtype, device=dev)
    if quantize_output:
        qout = _new_quant_out(x.shape[0], n_rows, dev)
        return fused_linear_into(x, iq3_weight, out, config=config, stream=stream, qout=qout), qout
    return fused_linear_into(x, iq3_weight, out, config=config, stream=stream)


def group_linear_into(xs, iq3_weights, outs, stream=None, qouts=None) -> list:
    """Independent linears ``outs[i] = linear(xs[i], iq3_weights[i])`` in one C-ABI call.

    Each is what ``iq3_s_fp8_linear`` computes. With bf16 activations in
    16-byte aligned rows, M < 32 and packed weights this is one persistent GEMV
    launch for the whole group (up to ``MAMBO_MAX_GROUP`` linears); otherwise
    the linears run one after another. No output may overlap another linear's
    input. No validation beyond the C ABI's. ``qouts``: per linear None or
    ``(q, s)`` buffers for the output's MXFP8 quantization (formed in the
    grouped launch's epilogue).
    """
    count = len(xs)
    items = (_lib.MamboLinearItem * count)()
    keep = []  # the weight structs must outlive the call
    for i, (x, w, out) in enumerate(zip(xs, iq3_weights, outs)):
        ws = weight_struct(w)
        keep.append(ws)
        items[i].x = x.data_ptr()
        items[i].x_dtype = _lib.MAMBO_BF16 if x.dtype == torch.bfloat16 else _lib.MAMBO_F32
        items[i].ldx = x.stride(0)
        items[i].m = x.shape[0]
        items[i].w = ctypes.pointer(ws)
        items[i].out = out.data_ptr()
        items[i].out_dtype = _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32
        items[i].ldo = out.stride(0)
    dev = xs[0].device
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        need = lib.mambo_iq3s_linear_group_workspace_bytes(items, count)
        ws = _runtime.workspace(dev, st, need)
        qarr = None
        if qouts is not None:
            qarr = (_lib.MamboQuantOut * count)()
            for i, qo in enumerate(qouts):
                if qo is not None:
                    qarr[i] = _quant_out_struct(qo)
        _lib.check(lib.mambo_iq3s_linear_group_q(items, qarr, count, _get_iq3_table(dev).data_ptr(), ws.data_ptr(),
                                                 ws.numel(), st), "iq3_s_fp8_linear_group")
    return outs


def iq3_s_fp8_linear_group(xs, iq3_weights, *, stream=None, out_dtype: torch.dtype = torch.bfloat16) -> list:
    """Several independent ``iq3_s_fp8_linear`` calls as one (see ``group_linear_into``).

    ``xs[i]``: float32 or bfloat16 [M_i, K_i]; ``iq3_weights[i]``: prepared
    fields with K_i = 256 * blocks. Returns the list of out_dtype [M_i, N_i].
    """
    if len(xs) != len(iq3_weights) or not xs:
        raise ValueError("xs and iq3_weights must be non-empty lists of the same length")
    if len(xs) > _lib.MAMBO_MAX_GROUP:
        raise ValueError(f"at most {_lib.MAMBO_MAX_GROUP} linears per group")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    xs = [_runtime.as_cuda_tensor(x) for x in xs]
    dev = xs[0].device
    outs, ready = [], []
    for x, w in zip(xs, iq3_weights):
        n_rows, k_blocks = _weight_dimensions(w)
        if x.ndim != 2 or x.dtype not in (torch.float32, torch.bfloat16) or x.shape[0] < 1 \
                or x.shape[1] != k_blocks * 256:
            raise ValueError("activation must be float32 or bfloat16 [M,K] with K = 256 * weight blocks")
        if x.device != dev:
            raise ValueError("all activations must be on one device")
        if x.stride(1) != 1:
            x = x.contiguous()
        ready.append(x)
        outs.append(torch.empty((x.shape[0], n_rows), dtype=out_dtype, device=dev))
    if _sm_key(dev) not in BEST_CONFIGS:
        raise RuntimeError(f"IQ3_S FP8 matmul has no tuned config for {_sm_key(dev)}")
    _runtime.require_device(dev)
    return group_linear_into(ready, iq3_weights, outs, stream=stream)


# ----------------------------------------------------------------------------
# Autotuning cases (iq3_s_fp8.py:402-465)
# ----------------------------------------------------------------------------
def config_search_space(kernel: int = _lib.MAMBO_KERNEL_GEMV) -> list[dict]:
    lib = _lib.load()
    out = []
    for i in range(lib.mambo_num_configs(kernel)):
        c = _lib.MamboLinearConfig()
        _lib.check(lib.mambo_config_at(kernel, i, c))
        out.append(c.to_dict())
    return out


# At most this many weight copies rotate through a tuning case (and at least as
# many launches are captured per timed graph, kernel_benchmark.MIN_GRAPH_LAUNCHES).
MAX_TUNING_COPIES = 32


def make_benchmark_cases(iq3_weight, ms: tuple[int, ...] = (4, 128), seed: int = 0, *,
                         bf16_input: bool = True) -> list:
    """Prepare SoA weights and inputs once; benchmark the linear (iq3_s_fp8.py:402-465).

    ``bf16_input``: time what a model calls, bf16 activations through the fused
    entry point (below 32 tokens the GEMV quantizes them itself; from 32 the
    quantizer is part of the GEMM's FP16 pass). False: the matmul alone on
    prequantized MXFP8 activations, as the reference's cases do.
    """
    from ..utils.kernel_benchmark import BenchmarkCase
    from .quantize_fp8 import launch_quantize_fp8

    if not isinstance(iq3_weight, IQ3SFields):
        iq3_weight = prepare_iq3_s_fields(iq3_weight)
    n_rows, k_blocks = _weight_dimensions(iq3_weight)
    k = k_blocks * IQ3_S_BLOCK_VALUES
    dev = iq3_weight.d.device
    # A stream of its own: candidates are timed as launches captured into a CUDA graph.
    stream = torch.cuda.Stream(dev)
    gen = torch.Generator(device=dev).manual_seed(seed)

    # Copies of the weight that together exceed twice the L2, taken in turn by
    # successive launches: every timed launch streams its weights from HBM, as
    # a model's linears do (one weight replayed would stay in L2).
    l2 = getattr(torch.cuda.get_device_properties(dev), "L2_cache_size", 126 * 2 ** 20) or 126 * 2 ** 20
    wbytes = sum(t.numel() * t.element_size() for t in (iq3_weight.d, iq3_weight.qs, iq3_weight.qh,
                                                         iq3_weight.signs, iq3_weight.scales))
    copies = max(1, min(MAX_TUNING_COPIES, -(-2 * l2 // wbytes)))
    weights = [iq3_weight] + [dataclasses.replace(
        iq3_weight, **{f: getattr(iq3_weight, f).clone() for f in ("d", "qs", "qh", "signs", "scales")},
        packed=None if iq3_weight.packed is None else iq3_weight.packed.clone()) for _ in range(copies - 1)]
    turn = [0]

    def next_weight() -> IQ3SFields:
        w = weights[turn[0] % len(weights)]
        turn[0] += 1
        return w

    def make_case(m: int) -> BenchmarkCase:
        x = torch.randn((m, k), generator=gen, device=dev, dtype=torch.float32)
        stream.wait_stream(torch.cuda.current_stream(dev))
        if bf16_input:
            xb = x.to(torch.bfloat16)
            stream.wait_stream(torch.cuda.current_stream(dev))
            out = torch.empty((m, n_rows), dtype=torch.bfloat16, device=dev)

            def run(config: dict) -> None:
                fused_linear_into(xb, next_weight(), out, config=config, stream=stream)
        else:
            x_values, x_scales = launch_quantize_fp8(x, stream=stream)
            out = torch.empty((m, n_rows), dtype=torch.float32, device=dev)

            def run(config: dict) -> None:
                linear_into(x_values, x_scales, next_weight(), out, config=config, stream=stream)

        # The untuned default first (the tuner never ends up slower than it), then the
        # kernel's space: below the threshold the tcgen05 GEMV (decoder warps x weight
        # stages x L2 prefetch x split mode); from it the FP16 GEMM (weight stages x K
        # split) and the same on CTA pairs (weight stages).
        default = dict(select_config(m, n_rows, k, dev, tuned=False))
        if m >= LARGE_TOKEN_THRESHOLD:
            space = config_search_space(_lib.MAMBO_KERNEL_GEMM_F16) + \
                config_search_space(_lib.MAMBO_KERNEL_GEMM_F16_PAIR)
        else:
            space = config_search_space(_lib.MAMBO_KERNEL_GEMV)
        return BenchmarkCase(
            name=f"M={m} N={n_rows} K={k}", stream=stream, kernel=run,
            search_space=[default] + [c for c in space if c != default],
            grid_fn=lambda config: (config.get("ctas_per_sm", 1),),
            args_fn=lambda config: (config,),
            hints_fn=None,
            summary_keys=("kernel", "stages", "split"),
            shape=(m, n_rows, k),
        )

    return [make_case(m) for m in ms]
