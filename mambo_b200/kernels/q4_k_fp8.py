"""Q4_K x MXFP8 linear on the sm_100a tcgen05 GEMV.

Q4_K is the next GGUF block type of the reference's tensor-type table
(src/python/mambo/utils/gguf_manifest.py:30-42); the reference loads it but
has no kernel for it. This module gives it the interface of the IQ3_S path
(src/python/mambo/kernels/iq3_s_fp8.py:364-399): weights prepared once on the
device, activations quantized to MXFP8, one linear launch.

Block layout (144 bytes per 256 weights): fp16 d, fp16 dmin, 12 bytes of eight
6-bit scales s_g and mins m_g, 128 bytes of 4-bit codes q; weight =
d*s_g*q - dmin*m_g = (d*s_g/2)*(2q - 15) + (7.5*d*s_g - dmin*m_g) for the
32-weight group g. The odd integers 2q - 15 are exact E4M3 operands (the
packed copy stores them in sign/magnitude form), so the tensor cores form each
group's partial product P_g with the MXFP8 activations as for IQ3_S; the FP32
epilogue adds (d*s_g/2)*P_g and the constant term times the token's sum of the
group's quantized activations, which the quantizer writes beside its codes.
"""

from __future__ import annotations

from typing import TypedDict

import torch

from .. import _lib, _runtime
from .quantize_fp8 import _ROUNDING

Q4_K_BLOCK_BYTES = 144
Q4_K_BLOCK_VALUES = 256
LARGE_TOKEN_THRESHOLD = 32


class Q4KFields(TypedDict):
    packed: torch.Tensor  # uint8, mambo_q4k_packed_bytes(N, B) bytes (tile-major records)
    n_rows: int
    n_blocks: int


def prepare_q4_k_fields(raw: torch.Tensor, *, stream=None) -> Q4KFields:
    """GGUF Q4_K bytes [N, B, 144] or [N, B*144] (uint8, any strides) -> the packed copy the GEMV streams."""
    raw = _runtime.as_cuda_tensor(raw)
    if raw.dtype != torch.uint8:
        raise ValueError("Q4_K weight must be uint8")
    if raw.ndim == 2:
        if raw.shape[1] % Q4_K_BLOCK_BYTES:
            raise ValueError("Q4_K row bytes must be a multiple of 144")
        if raw.stride(1) != 1:
            raw = raw.contiguous()
        raw = raw.view(raw.shape[0], raw.shape[1] // Q4_K_BLOCK_BYTES, Q4_K_BLOCK_BYTES)
    if raw.ndim != 3 or raw.shape[2] != Q4_K_BLOCK_BYTES or raw.shape[0] < 1 or raw.shape[1] < 1:
        raise ValueError("Q4_K weight must be uint8 [N, K/256, 144]")
    _runtime.require_device(raw.device)
    n_rows, n_blocks = int(raw.shape[0]), int(raw.shape[1])
    lib = _lib.load()
    packed = torch.empty(lib.mambo_q4k_packed_bytes(n_rows, n_blocks), dtype=torch.uint8, device=raw.device)
    with torch.cuda.device(raw.device):
        st = _runtime.stream_handle(stream, raw.device)
        _lib.check(lib.mambo_q4k_pack(raw.data_ptr(), n_rows, n_blocks, raw.stride(0), raw.stride(1), raw.stride(2),
                                      packed.data_ptr(), st), "prepare_q4_k_fields")
    return {"packed": packed, "n_rows": n_rows, "n_blocks": n_blocks}


def launch_quantize_fp8_sums(x, *, stream=None, rounding: str = "nearest_even"):
    """MXFP8 quantization plus each 32-value group's sum of its quantized values.

    Returns (values uint8 [M,K], scales uint8 [M,K/32], sums float32 [M,K/32]);
    values and scales equal launch_quantize_fp8's bit for bit.
    """
    x = _runtime.as_cuda_tensor(x)
    if x.ndim != 2 or x.dtype not in (torch.float32, torch.bfloat16) or x.shape[1] % 32 or x.shape[0] < 1:
        raise ValueError("activation must be float32 or bfloat16 [M,K] with K divisible by 32")
    if rounding not in _ROUNDING:
        raise ValueError(f"rounding must be one of {sorted(_ROUNDING)}")
    _runtime.require_device(x.device)
    if x.stride(1) != 1:
        x = x.contiguous()
    m, k = x.shape
    values = torch.empty((m, k), dtype=torch.uint8, device=x.device)
    scales = torch.empty((m, k // 32), dtype=torch.uint8, device=x.device)
    sums = torch.empty((m, k // 32), dtype=torch.float32, device=x.device)
    dtype = _lib.MAMBO_BF16 if x.dtype == torch.bfloat16 else _lib.MAMBO_F32
    with torch.cuda.device(x.device):
        st = _runtime.stream_handle(stream, x.device)
        _lib.check(_lib.load().mambo_quantize_mxfp8_sums(
            x.data_ptr(), dtype, m, k, x.stride(0), values.data_ptr(), values.stride(0), scales.data_ptr(),
            scales.stride(0), sums.data_ptr(), sums.stride(0), _ROUNDING[rounding], st), "launch_quantize_fp8_sums")
    return values, scales, sums


def _config(config: dict | None) -> _lib.MamboLinearConfig | None:
    return None if config is None else _lib.MamboLinearConfig.from_dict(config)


def launch_q4_k_fp8_matmul(x_values, x_scales, x_sums, weight: Q4KFields, *, stream=None,
                           out_dtype: torch.dtype = torch.float32, config: dict | None = None,
                           out: torch.Tensor | None = None) -> torch.Tensor:
    """Prequantized MXFP8 activations (with their group sums) times a prepared Q4_K weight -> out [M,N]."""
    n_rows, n_blocks = weight["n_rows"], weight["n_blocks"]
    k = n_blocks * Q4_K_BLOCK_VALUES
    x_values, x_scales, x_sums = (_runtime.as_cuda_tensor(t) for t in (x_values, x_scales, x_sums))
    m = x_values.shape[0]
    if x_values.ndim != 2 or x_values.dtype != torch.uint8 or m < 1 or x_values.shape[1] != k:
        raise ValueError("x_values must be uint8 [M,K]")
    if tuple(x_scales.shape) != (m, k // 32) or x_scales.dtype != torch.uint8:
        raise ValueError("x_scales must be uint8 [M,K/32]")
    if tuple(x_sums.shape) != (m, k // 32) or x_sums.dtype != torch.float32:
        raise ValueError("x_sums must be float32 [M,K/32]")
    dev = x_values.device
    _runtime.require_device(dev)
    x_values, x_scales, x_sums = (t if t.stride(1) == 1 else t.contiguous() for t in (x_values, x_scales, x_sums))
    if out is None:
        if out_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
        out = torch.empty((m, n_rows), dtype=out_dtype, device=dev)
    cfg = _config(config)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        ws = _runtime.workspace(dev, st, lib.mambo_q4k_linear_workspace_bytes(m, n_rows, n_blocks, cfg))
        _lib.check(lib.mambo_q4k_linear(
            x_values.data_ptr(), x_values.stride(0), x_scales.data_ptr(), x_scales.stride(0), x_sums.data_ptr(),
            x_sums.stride(0), m, weight["packed"].data_ptr(), n_rows, n_blocks, out.data_ptr(),
            _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32, out.stride(0), cfg, ws.data_ptr(),
            ws.numel(), st), "launch_q4_k_fp8_matmul")
    return out


def q4_k_fp8_linear(x, weight: Q4KFields, *, stream=None, out_dtype: torch.dtype = torch.bfloat16,
                    config: dict | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16/f32 activations [M,K] -> MXFP8 (round to nearest even, with group sums) -> Q4_K linear, one C-ABI call."""
    x = _runtime.as_cuda_tensor(x)
    n_rows, n_blocks = weight["n_rows"], weight["n_blocks"]
    if x.ndim != 2 or x.dtype not in (torch.float32, torch.bfloat16) or x.shape[0] < 1 \
            or x.shape[1] != n_blocks * Q4_K_BLOCK_VALUES:
        raise ValueError("activation must be float32 or bfloat16 [M,K] with K = 256 * blocks")
    dev = x.device
    _runtime.require_device(dev)
    if x.stride(1) != 1:
        x = x.contiguous()
    m = x.shape[0]
    if out is None:
        if out_dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
        out = torch.empty((m, n_rows), dtype=out_dtype, device=dev)
    cfg = _config(config)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        ws = _runtime.workspace(dev, st, lib.mambo_q4k_linear_fused_workspace_bytes(m, n_rows, n_blocks, cfg))
        _lib.check(lib.mambo_q4k_linear_fused(
            x.data_ptr(), _lib.MAMBO_BF16 if x.dtype == torch.bfloat16 else _lib.MAMBO_F32, x.stride(0), m,
            weight["packed"].data_ptr(), n_rows, n_blocks, out.data_ptr(),
            _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32, out.stride(0), cfg, ws.data_ptr(),
            ws.numel(), st), "q4_k_fp8_linear")
    return out


def q4_k_linear_group_into(xs, weights, outs, *, stream=None) -> list:
    """Independent Q4_K linears ``outs[i] = q4_k_fp8_linear(xs[i], weights[i])`` in one C-ABI call.

    With bf16 activations in 16-byte aligned rows, 1 <= M < 32 and N % 8 == 0
    for every item, this is a quantization pre-pass (codes and group sums of all
    items at once) and one persistent GEMV launch over all items' weights;
    otherwise the items run one after another. No output may overlap another
    item's input.
    """
    count = len(xs)
    if count < 1 or len(weights) != count or len(outs) != count:
        raise ValueError("xs, weights and outs must be non-empty lists of the same length")
    if count > _lib.MAMBO_MAX_GROUP:
        raise ValueError(f"at most {_lib.MAMBO_MAX_GROUP} linears per group")
    items = (_lib.MamboQ4KItem * count)()
    for i, (x, w, out) in enumerate(zip(xs, weights, outs)):
        n_rows, n_blocks = w["n_rows"], w["n_blocks"]
        if x.ndim != 2 or x.dtype not in (torch.float32, torch.bfloat16) or x.shape[1] != n_blocks * Q4_K_BLOCK_VALUES \
                or x.stride(1) != 1:
            raise ValueError(f"xs[{i}] must be float32 or bfloat16 [M,K] with unit column stride")
        if tuple(out.shape) != (x.shape[0], n_rows) or out.dtype not in (torch.float32, torch.bfloat16) \
                or out.stride(1) != 1:
            raise ValueError(f"outs[{i}] must be float32 or bfloat16 [M,N] with unit column stride")
        items[i].x, items[i].ldx, items[i].m = x.data_ptr(), x.stride(0), x.shape[0]
        items[i].x_dtype = _lib.MAMBO_BF16 if x.dtype == torch.bfloat16 else _lib.MAMBO_F32
        items[i].packed, items[i].n_rows, items[i].n_blocks = w["packed"].data_ptr(), n_rows, n_blocks
        items[i].out, items[i].ldo = out.data_ptr(), out.stride(0)
        items[i].out_dtype = _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32
    dev = xs[0].device
    _runtime.require_device(dev)
    lib = _lib.load()
    with torch.cuda.device(dev):
        st = _runtime.stream_handle(stream, dev)
        ws = _runtime.workspace(dev, st, lib.mambo_q4k_linear_group_workspace_bytes(items, count))
        _lib.check(lib.mambo_q4k_linear_group(items, count, ws.data_ptr(), ws.numel(), st), "q4_k_linear_group")
    return outs


def q4_k_fp8_linear_group(xs, weights, *, stream=None, out_dtype: torch.dtype = torch.bfloat16) -> list:
    """Several independent ``q4_k_fp8_linear`` calls as one (see ``q4_k_linear_group_into``)."""
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be torch.float32 or torch.bfloat16")
    outs = [torch.empty((x.shape[0], w["n_rows"]), dtype=out_dtype, device=x.device) for x, w in zip(xs, weights)]
    return q4_k_linear_group_into(xs, weights, outs, stream=stream)
