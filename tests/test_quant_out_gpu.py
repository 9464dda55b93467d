"""The next linear's MXFP8 quantization formed in this linear's epilogue (mambo_iq3s_linear*_q).

The reference quantizes every linear's input in a pass of its own
(launch_quantize_fp8, src/python/mambo/kernels/quantize_fp8.py:42-52,67-84).
Here a linear can hand the next one its output already quantized: on the
tcgen05 GEMV a warp owns 32 consecutive output features, one MXFP8 group per
token, and quantizes them where their value is final. The codes must equal
launch_quantize_fp8 of the stored output (bf16 or f32) bit for bit, on every
path: the fused GEMV (each split mode), the prequantized GEMV, the grouped
launch, and the paths that quantize after the linear (GEMM, unpacked weights).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mambo_b200 import _lib
from mambo_b200.kernels.iq3_s_fp8 import group_linear_into, iq3_s_fp8_linear, launch_iq3_s_fp8_matmul
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields
from oracle import iq3s_oracle as O

pytestmark = pytest.mark.gpu

GEMV = {"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": 6, "ctas_per_sm": 1, "prefetch": 0}


def _weight(dev, n, k, seed, packed=True):
    raw = O.make_synthetic_iq3s(n, k, seed)
    return raw, prepare_iq3_s_fields(torch.from_numpy(raw).to(dev), packed=packed)


def _x(dev, m, k, seed):
    x = np.random.default_rng(seed).standard_normal((m, k)).astype(np.float32)
    x[:, np.random.default_rng(seed + 1).permutation(k)[: max(1, k // 100)]] *= 50.0
    return torch.from_numpy(x).to(dev).to(torch.bfloat16)


def _assert_codes_of(out: torch.Tensor, q: torch.Tensor, s: torch.Tensor) -> None:
    eq, es = launch_quantize_fp8(out)
    torch.cuda.synchronize()
    bad = (q != eq).nonzero()[:8].tolist()
    detail = [(t, n, int(q[t, n]), int(eq[t, n]), float(out[t, n]), int(s[t, n // 32]), int(es[t, n // 32]))
              for t, n in bad]
    assert torch.equal(q, eq), f"{int((q != eq).sum())} codes differ (token, feature, got, expected, value, " \
                               f"scale got, scale expected): {detail}"
    assert torch.equal(s, es), int((s != es).sum())


def _kernels(fn) -> list[str]:
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    return [n for n in names if "iq3s" in n or "mxfp8" in n]


@pytest.mark.parametrize("m", [1, 2, 5, 8, 13, 31])
@pytest.mark.parametrize("split", [0, 1, 2])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_fused_gemv_epilogue_codes_equal_the_quantizer(cuda_device, m, split, out_dtype):
    _, w = _weight(cuda_device, 1024, 2048, seed=500 + m)
    x = _x(cuda_device, m, 2048, seed=600 + m + split)
    cfg = dict(GEMV, split=split)
    out, (q, s) = iq3_s_fp8_linear(x, w, out_dtype=out_dtype, config=cfg, quantize_output=True)
    plain = iq3_s_fp8_linear(x, w, out_dtype=out_dtype, config=cfg)
    assert torch.equal(out, plain)  # the output itself is unchanged
    _assert_codes_of(out, q, s)


def test_one_launch_on_the_gemv(cuda_device):
    _, w = _weight(cuda_device, 4096, 4096, seed=7)
    x = _x(cuda_device, 8, 4096, seed=8)
    iq3_s_fp8_linear(x, w, quantize_output=True)  # workspace outside the profiled region
    kernels = _kernels(lambda: iq3_s_fp8_linear(x, w, quantize_output=True))
    if kernels:
        assert len(kernels) == 1 and "gemv_tm" in kernels[0], kernels


@pytest.mark.parametrize("m", [1, 8, 20])
def test_prequantized_gemv_epilogue_codes(cuda_device, m):
    _, w = _weight(cuda_device, 6144, 4096, seed=11 + m)
    xq, xs = launch_quantize_fp8(_x(cuda_device, m, 4096, seed=12 + m))
    out, (q, s) = launch_iq3_s_fp8_matmul(xq, xs, w, out_dtype=torch.bfloat16, quantize_output=True)
    assert torch.equal(out, launch_iq3_s_fp8_matmul(xq, xs, w, out_dtype=torch.bfloat16))
    _assert_codes_of(out, q, s)


def test_grouped_launch_epilogue_codes(cuda_device):
    """Items with and without quantized outputs in one grouped launch (M 1..8, mixed output types)."""
    shapes = [(6144, 4096, 1), (4096, 4096, 2), (14336, 4096, 4), (4096, 14336, 8), (1024, 2048, 3)]
    xs, ws, outs, qouts = [], [], [], []
    for i, (n, k, m) in enumerate(shapes):
        _, w = _weight(cuda_device, n, k, seed=40 + i)
        xs.append(_x(cuda_device, m, k, seed=50 + i))
        ws.append(w)
        outs.append(torch.empty((m, n), dtype=torch.bfloat16 if i % 2 == 0 else torch.float32, device=cuda_device))
        qouts.append(None if i == 1 else (torch.empty((m, n), dtype=torch.uint8, device=cuda_device),
                                          torch.empty((m, n // 32), dtype=torch.uint8, device=cuda_device)))
    group_linear_into(xs, ws, outs, qouts=qouts)
    plain = [torch.empty_like(o) for o in outs]
    group_linear_into(xs, ws, plain)
    torch.cuda.synchronize()
    for i, (o, p, qo) in enumerate(zip(outs, plain, qouts)):
        assert torch.equal(o, p), i
        if qo is not None:
            _assert_codes_of(o, *qo)


@pytest.mark.parametrize("m", [32, 130])
def test_gemm_path_quantizes_after(cuda_device, m):
    raw, w = _weight(cuda_device, 512, 2048, seed=70 + m)
    x = _x(cuda_device, m, 2048, seed=71 + m)
    out, (q, s) = iq3_s_fp8_linear(x, w, out_dtype=torch.bfloat16, quantize_output=True)
    _assert_codes_of(out, q, s)


def test_unpacked_weights_quantize_after(cuda_device):
    _, w = _weight(cuda_device, 512, 1024, seed=81, packed=False)
    x = _x(cuda_device, 4, 1024, seed=82)
    out, (q, s) = iq3_s_fp8_linear(x, w, out_dtype=torch.float32, quantize_output=True)
    _assert_codes_of(out, q, s)


def test_nan_and_zero_groups(cuda_device):
    """A NaN output group gets the scale code 0xFF and an all-zero row code 127, as the quantizer gives them."""
    raw = O.make_synthetic_iq3s(256, 1024, 91)
    raw[3, 0, :2] = np.array([np.nan], dtype=np.float16).view(np.uint8)  # row 3's first block scale: NaN
    w = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))
    x = _x(cuda_device, 3, 1024, seed=92)
    x[1] = 0
    out, (q, s) = iq3_s_fp8_linear(x, w, out_dtype=torch.float32, config=dict(GEMV, split=0),
                                   quantize_output=True)
    _assert_codes_of(out, q, s)
    assert torch.isnan(out[:, 3]).all()      # d = NaN reaches every token, the zero row included
    assert (s[:, 0] == 0xFF).all()           # the group holding feature 3
    assert (s[1, 1:] == 127).all()           # the zero row's other groups


def test_chained_linears_take_the_epilogue_codes(cuda_device):
    """linear 1 -> its epilogue's MXFP8 -> linear 2 equals linear 2 on linear 1's stored output."""
    _, w1 = _weight(cuda_device, 4096, 4096, seed=101)
    raw2, w2 = _weight(cuda_device, 14336, 4096, seed=102)
    x = _x(cuda_device, 8, 4096, seed=103)
    y1, (q1, s1) = iq3_s_fp8_linear(x, w1, out_dtype=torch.bfloat16, quantize_output=True)
    y2 = launch_iq3_s_fp8_matmul(q1, s1, w2, out_dtype=torch.float32)
    ref = iq3_s_fp8_linear(y1, w2, out_dtype=torch.float32)
    assert torch.equal(y2, ref)
    err = O.relative_frobenius(y2.cpu().numpy(), O.iq3s_linear_f64(q1.cpu().numpy(), s1.cpu().numpy(), raw2))
    assert err < 1e-4


def test_rejects_n_not_divisible_by_32(cuda_device):
    _, w = _weight(cuda_device, 264, 512, seed=111)
    x = _x(cuda_device, 2, 512, seed=112)
    with pytest.raises(ValueError):
        iq3_s_fp8_linear(x, w, quantize_output=True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_standalone_quantizer_flags_nan_and_inf_groups(cuda_device, dtype):
    """The quantizer's rule for non-finite groups: a NaN or an infinity among a group's 32 values gives the
    scale code 0xFF; the other groups of the row are unaffected."""
    x = torch.randn((2, 128), device=cuda_device).to(dtype)
    x[0, 3] = float("nan")
    x[1, 70] = float("inf")
    q, s = launch_quantize_fp8(x)
    torch.cuda.synchronize()
    ref_q, ref_s = O.quantize_mxfp8(torch.nan_to_num(x.float(), nan=0.0, posinf=0.0).cpu().numpy())
    assert int(s[0, 0]) == 0xFF, s[0].tolist()
    assert int(s[1, 2]) == 0xFF, s[1].tolist()
    keep = [(0, 1), (0, 2), (0, 3), (1, 0), (1, 1), (1, 3)]
    assert all(int(s[r, g]) == int(ref_s[r, g]) for r, g in keep)
