"""GPU parity of the fused quantize + linear entry point (mambo_iq3s_linear_fused).

The reference runs launch_quantize_fp8 then launch_iq3_s_fp8_matmul
(src/python/mambo/kernels/quantize_fp8.py:67-84, iq3_s_fp8.py:364-399). Below
32 tokens the tcgen05 GEMV here quantizes bf16 rows itself with the standalone
quantizer's arithmetic; from 32 tokens the quantization is part of the pass
that writes the FP16 GEMM's activation operand. Either way the output must
equal the two-step path bit for bit under the same configuration.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import iq3s_oracle as O
from mambo_b200 import _lib
from mambo_b200.kernels.iq3_s_fp8 import iq3_s_fp8_linear, launch_iq3_s_fp8_matmul
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

pytestmark = pytest.mark.gpu

ORACLE_FROB_TOL = 1e-4  # vs the float64 oracle on the same MXFP8 inputs (FP32 accumulation only)


def _weight(dev, n, k, seed):
    raw = O.make_synthetic_iq3s(n, k, seed)
    return raw, prepare_iq3_s_fields(torch.from_numpy(raw).to(dev))


def _activations(dev, m, k, seed, outliers=True):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if outliers:
        cols = rng.permutation(k)[: max(1, k // 100)]
        x[:, cols] *= 50.0
    return torch.from_numpy(x).to(dev).to(torch.bfloat16)


def _two_step(x, fields, out_dtype, config):
    xq, xs = launch_quantize_fp8(x)
    return launch_iq3_s_fp8_matmul(xq, xs, fields, out_dtype=out_dtype, config=config)


def _same_bits(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.dtype != b.dtype or a.shape != b.shape:
        return False
    iview = torch.int32 if a.dtype == torch.float32 else torch.int16
    return torch.equal(a.contiguous().view(iview), b.contiguous().view(iview))


def _our_kernels(fn) -> list[str]:
    """Names of this library's kernels that fn launches (CUDA activity of the profiler)."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    return [n for n in names if "iq3s" in n or "mxfp8" in n]


def _assert_fused(fn) -> None:
    kernels = _our_kernels(fn)
    if kernels:  # an empty list: the profiler saw no kernel activity at all
        assert len(kernels) == 1 and "gemv_tm" in kernels[0], kernels


GEMV = {"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": 6, "ctas_per_sm": 1, "prefetch": 0}


@pytest.mark.parametrize("m", [1, 2, 5, 8, 9, 16, 17, 31])
@pytest.mark.parametrize("split", [0, 1, 2])
def test_fused_equals_two_step_bitwise(cuda_device, m, split):
    raw, fields = _weight(cuda_device, 1024, 2048, seed=300 + m)
    x = _activations(cuda_device, m, 2048, seed=400 + m + split)
    cfg = dict(GEMV, split=split)
    fused = iq3_s_fp8_linear(x, fields, out_dtype=torch.float32, config=cfg)
    assert _same_bits(fused, _two_step(x, fields, torch.float32, cfg))
    _assert_fused(lambda: iq3_s_fp8_linear(x, fields, out_dtype=torch.float32, config=cfg))
    xq, xs = O.quantize_mxfp8(x.float().cpu().numpy())
    ref = O.iq3s_linear_f64(xq, xs, raw)
    assert O.relative_frobenius(fused.cpu().numpy(), ref) < ORACLE_FROB_TOL


@pytest.mark.parametrize("warps,stages", [(8, 8), (16, 4)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_fused_decoder_warps_and_output_types(cuda_device, warps, stages, out_dtype):
    _, fields = _weight(cuda_device, 2048, 4096, seed=11)
    x = _activations(cuda_device, 8, 4096, seed=12)
    cfg = dict(GEMV, warps=warps, stages=stages, split=0)
    fused = iq3_s_fp8_linear(x, fields, out_dtype=out_dtype, config=cfg)
    assert fused.dtype == out_dtype
    assert _same_bits(fused, _two_step(x, fields, out_dtype, cfg))
    _assert_fused(lambda: iq3_s_fp8_linear(x, fields, out_dtype=out_dtype, config=cfg))


def test_fused_default_config_and_ragged_k(cuda_device):
    """Default (tuned) configuration; K of 3 blocks (odd: the last scale row is half used)."""
    raw, fields = _weight(cuda_device, 264, 768, seed=21)
    x = _activations(cuda_device, 3, 768, seed=22)
    fused = iq3_s_fp8_linear(x, fields, out_dtype=torch.float32)
    assert _same_bits(fused, _two_step(x, fields, torch.float32, None))
    _assert_fused(lambda: iq3_s_fp8_linear(x, fields, out_dtype=torch.float32))
    xq, xs = O.quantize_mxfp8(x.float().cpu().numpy())
    assert O.relative_frobenius(fused.cpu().numpy(), O.iq3s_linear_f64(xq, xs, raw)) < ORACLE_FROB_TOL


def test_fused_strided_rows(cuda_device):
    """Rows of a wider buffer: 16-byte aligned strides stay fused, others take the two-step path."""
    _, fields = _weight(cuda_device, 512, 1024, seed=31)
    for pad in (64, 8, 3):
        big = _activations(cuda_device, 6, 1024 + pad, seed=32 + pad)
        x = big[:, :1024]
        assert x.stride(0) == 1024 + pad
        fused = iq3_s_fp8_linear(x, fields, out_dtype=torch.float32, config=dict(GEMV, split=0))
        assert _same_bits(fused, _two_step(x.contiguous(), fields, torch.float32, dict(GEMV, split=0)))
        kernels = _our_kernels(lambda: iq3_s_fp8_linear(x, fields, config=dict(GEMV, split=0)))
        assert not kernels or len(kernels) == (1 if pad % 8 == 0 else 2), (pad, kernels)


def test_fused_nan_and_zero_rows(cuda_device):
    """A NaN row and an all-zero row give what the standalone quantizer gives, other rows untouched."""
    raw, fields = _weight(cuda_device, 256, 512, seed=41)
    x = _activations(cuda_device, 4, 512, seed=42)
    x[1, 7] = float("nan")
    x[2] = 0
    cfg = dict(GEMV, split=0)
    fused = iq3_s_fp8_linear(x, fields, out_dtype=torch.float32, config=cfg)
    two = _two_step(x, fields, torch.float32, cfg)
    assert _same_bits(fused, two)
    assert torch.equal(fused[2], torch.zeros_like(fused[2]))
    assert torch.isfinite(fused[[0, 3]]).all()


@pytest.mark.parametrize("m", [32, 40, 130, 300])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_fused_prefill_quantizes_in_the_fp16_pass(cuda_device, m, out_dtype):
    """From 32 tokens: the quantizer is part of the pass that writes the GEMM's FP16 activations
    (iq3s_x16_quant_kernel), then the GEMM -- two launches, the same bits as quantize + linear."""
    raw, fields = _weight(cuda_device, 264, 1024, seed=51 + m)
    x = _activations(cuda_device, m, 1024, seed=52 + m)
    x[1, 7] = float("nan")  # a NaN group and an all-zero row go through as the standalone quantizer has them
    x[2] = 0
    stream = torch.cuda.Stream(cuda_device)  # fresh stream: the workspace query covers this path
    with torch.cuda.stream(stream):
        fused = iq3_s_fp8_linear(x, fields, out_dtype=out_dtype, stream=stream)
    stream.synchronize()
    assert _same_bits(fused, _two_step(x, fields, out_dtype, None))
    kernels = _our_kernels(lambda: iq3_s_fp8_linear(x, fields, out_dtype=out_dtype))
    if kernels:
        assert len(kernels) == 2 and any("x16_quant" in k for k in kernels) \
            and any("gemm_f16" in k for k in kernels), kernels
    keep = [i for i in range(m) if i != 1]
    xq, xs = O.quantize_mxfp8(x[keep].float().cpu().numpy())
    ref = O.iq3s_linear_f64(xq, xs, raw)
    tol = ORACLE_FROB_TOL if out_dtype == torch.float32 else 4e-3
    assert O.relative_frobenius(fused[keep].float().cpu().numpy(), ref) < tol


def test_fused_prefill_f32_and_strided_rows(cuda_device):
    """f32 activations take the same fused pass; rows not 16-byte aligned fall back to two steps."""
    _, fields = _weight(cuda_device, 256, 1024, seed=71)
    x32 = _activations(cuda_device, 64, 1024, seed=72).float() * 1.0001  # not representable in bf16
    assert _same_bits(iq3_s_fp8_linear(x32, fields, out_dtype=torch.float32),
                      _two_step(x32, fields, torch.float32, None))
    kernels = _our_kernels(lambda: iq3_s_fp8_linear(x32, fields))
    assert not kernels or len(kernels) == 2, kernels
    for pad in (8, 3):
        big = _activations(cuda_device, 48, 1024 + pad, seed=73 + pad)
        x = big[:, :1024]
        fused = iq3_s_fp8_linear(x, fields, out_dtype=torch.float32)
        assert _same_bits(fused, _two_step(x.contiguous(), fields, torch.float32, None)), pad
        kernels = _our_kernels(lambda: iq3_s_fp8_linear(x, fields))
        assert not kernels or len(kernels) == (2 if pad % 8 == 0 else 3), (pad, kernels)


def test_fused_f32_activations(cuda_device):
    _, fields = _weight(cuda_device, 256, 1024, seed=61)
    x = _activations(cuda_device, 5, 1024, seed=62).float() * 1.0001  # not representable in bf16
    fused = iq3_s_fp8_linear(x, fields, out_dtype=torch.float32)
    assert _same_bits(fused, _two_step(x, fields, torch.float32, None))


@pytest.mark.parametrize("proj", [(6144, 4096), (4096, 4096), (14336, 4096), (4096, 14336)])
def test_fused_decode_is_one_launch(cuda_device, proj):
    """Llama-3-8B projections with the tuned decode configurations: the GEMV alone, no quantizer kernel."""
    n, k = proj
    gen = torch.Generator(device=cuda_device).manual_seed(n + k)
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=cuda_device, generator=gen)
    raw[..., :2] = torch.full((n, k // 256), 1e-3, device=cuda_device).half().view(torch.uint8).view(n, k // 256, 2)
    fields = prepare_iq3_s_fields(raw)
    for m in (1, 2, 4, 8):
        x = torch.randn((m, k), device=cuda_device, generator=gen).to(torch.bfloat16)
        iq3_s_fp8_linear(x, fields)  # workspace allocation outside the profiled region
        kernels = _our_kernels(lambda: iq3_s_fp8_linear(x, fields))
        if not kernels:
            pytest.skip("profiler recorded no kernel activity")
        assert len(kernels) == 1 and "gemv_tm" in kernels[0], (m, kernels)
