"""GPU parity of the tcgen05 prefill GEMM (M >= LARGE_TOKEN_THRESHOLD) against the oracle.

The reference's large-token kernel (iq3_s_fp8.py:225-276) forms every
32-weight group's block-scaled E4M3 product in FP32 and accumulates it scaled
by d*(1+2*nibble); the cases below follow test_iq3_s_fp8.py's matmul tests
(ragged M and N, f32 output) and add the prefill shapes of the north star with
the outlier activations it names.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import iq3s_oracle as O
from mambo_b200 import _lib
from mambo_b200.kernels.iq3_s_fp8 import launch_dequant_iq3_s, launch_iq3_s_fp8_matmul
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

pytestmark = pytest.mark.gpu

REL_FROB_TOL = 1e-3    # north star: vs fp32/f64 matmul of the dequantized operands
ORACLE_FROB_TOL = 1e-4  # vs the float64 oracle on the same MXFP8 inputs (FP32 accumulation only)
GEMM = {"kernel": _lib.MAMBO_KERNEL_GEMM, "warps": 8, "stages": 4}
GEMM_F16 = {"kernel": _lib.MAMBO_KERNEL_GEMM_F16, "warps": 8, "stages": 4}
GEMM_F16_PAIR = {"kernel": _lib.MAMBO_KERNEL_GEMM_F16_PAIR, "warps": 8, "stages": 4}
# The per-group FP8 kernel (the reference's decomposition), the FP16-operand kernel (group scale folded
# into the weight operand, one accumulator per K block) and the same on CTA pairs (256-row tiles).
KINDS = {"fp8_groups": GEMM, "f16": GEMM_F16, "f16_pair": GEMM_F16_PAIR}


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def _case(dev, m, n, k, seed, outliers=False):
    raw = O.make_synthetic_iq3s(n, k, seed)
    rng = np.random.default_rng(seed + 1)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if outliers:
        cols = rng.permutation(k)[: max(1, round(0.01 * k))]
        x[:, cols] *= 50.0
    xq, xs = O.quantize_mxfp8(x)
    ref = O.iq3s_linear_f64(xq, xs, raw)
    fields = prepare_iq3_s_fields(torch.from_numpy(raw).to(dev))
    return fields, torch.from_numpy(xq).to(dev), torch.from_numpy(xs).to(dev), ref


@pytest.mark.parametrize("m,n,k,outliers", [(32, 256, 512, False), (128, 128, 256, False), (130, 384, 1024, True),
                                            (257, 136, 512, False), (64, 640, 1536, True), (300, 256, 2048, True)])
@pytest.mark.parametrize("stages", [2, 3, 4])
@pytest.mark.parametrize("kind", sorted(KINDS))
def test_gemm_matches_oracle(cuda_device, m, n, k, outliers, stages, kind):
    fields, xq, xs, ref = _case(cuda_device, m, n, k, seed=900 + m + n + stages, outliers=outliers)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, config=dict(KINDS[kind], stages=stages))
    got = to_np(out).astype(np.float64)
    assert O.relative_frobenius(got, ref) < ORACLE_FROB_TOL
    np.testing.assert_allclose(got, ref, rtol=5e-4, atol=5e-4 * np.abs(ref).max())


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_gemm_bf16_output(cuda_device, kind):
    fields, xq, xs, ref = _case(cuda_device, 160, 512, 1024, seed=7)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, out_dtype=torch.bfloat16, config=KINDS[kind])
    assert out.dtype == torch.bfloat16
    assert O.relative_frobenius(to_np(out.float()), ref) < 4e-3  # bf16 output rounding


@pytest.mark.parametrize("m,n,k", [(32, 256, 512), (130, 384, 1024), (257, 136, 512), (300, 640, 1536), (2048, 1024, 1024)])
@pytest.mark.parametrize("kind", sorted(KINDS))
def test_gemm_bf16_output_is_the_rounded_f32_output(cuda_device, m, n, k, kind):
    """bf16 tiles leave through shared memory and a TMA store (partial tiles clipped): bit for bit the f32 result rounded."""
    fields, xq, xs, _ = _case(cuda_device, m, n, k, seed=500 + m + n)
    f32 = launch_iq3_s_fp8_matmul(xq, xs, fields, config=KINDS[kind])
    bf16 = launch_iq3_s_fp8_matmul(xq, xs, fields, out_dtype=torch.bfloat16, config=KINDS[kind])
    assert torch.equal(bf16.view(torch.int16), f32.to(torch.bfloat16).view(torch.int16))


def test_default_config_picks_the_gemm_at_large_m(cuda_device):
    lib = _lib.load()
    for m, kind in ((8, _lib.MAMBO_KERNEL_GEMV), (31, _lib.MAMBO_KERNEL_GEMV), (32, _lib.MAMBO_KERNEL_GEMM_F16),
                    (4096, _lib.MAMBO_KERNEL_GEMM_F16)):
        c = _lib.MamboLinearConfig()
        _lib.check(lib.mambo_default_config(m, 4096, 16, c))
        assert c.kernel == kind, (m, c.kernel)
    # and the default path gives the oracle's result
    fields, xq, xs, ref = _case(cuda_device, 96, 256, 768, seed=21)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields)
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_gemm_agrees_with_chunked_gemv(cuda_device, kind):
    """Independent kernels, exact products: only the FP32 summation order differs."""
    fields, xq, xs, ref = _case(cuda_device, 96, 1024, 2048, seed=33, outliers=True)
    a = launch_iq3_s_fp8_matmul(xq, xs, fields, config=KINDS[kind])
    b = launch_iq3_s_fp8_matmul(xq, xs, fields, config={"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": 4})
    assert O.relative_frobenius(to_np(a), to_np(b).astype(np.float64)) < 1e-5


@pytest.mark.parametrize("kind", sorted(KINDS))
def test_gemm_is_deterministic(cuda_device, kind):
    fields, xq, xs, _ = _case(cuda_device, 200, 384, 1024, seed=44)
    a = launch_iq3_s_fp8_matmul(xq, xs, fields, config=KINDS[kind])
    b = launch_iq3_s_fp8_matmul(xq, xs, fields, config=KINDS[kind])
    assert torch.equal(a, b)


def test_unaligned_activations_fall_back_or_raise(cuda_device):
    """The GEMM's TMA needs 16-byte aligned rows: the default path falls back to the GEMV; an explicit GEMM raises."""
    fields, xq, xs, ref = _case(cuda_device, 48, 256, 512, seed=55)
    buf = torch.empty(xq.numel() + 1, dtype=torch.uint8, device=cuda_device)
    odd = buf[1:].view(xq.shape)
    odd.copy_(xq)
    out = launch_iq3_s_fp8_matmul(odd, xs, fields)
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL
    for cfg in KINDS.values():
        with pytest.raises(ValueError):
            launch_iq3_s_fp8_matmul(odd, xs, fields, config=cfg)


def test_gemm_without_packed_weights_falls_back(cuda_device):
    raw = O.make_synthetic_iq3s(256, 512, 66)
    soa = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device), packed=False)
    rng = np.random.default_rng(67)
    xq, xs = O.quantize_mxfp8(rng.standard_normal((40, 512)).astype(np.float32))
    ref = O.iq3s_linear_f64(xq, xs, raw)
    out = launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device), soa)
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL


LLAMA3_8B = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (14336, 4096), "down": (4096, 14336)}


@pytest.mark.parametrize("proj", sorted(LLAMA3_8B))
@pytest.mark.parametrize("m", [512, 2048])
@pytest.mark.parametrize("kind", sorted(KINDS))
def test_full_size_prefill_frobenius(cuda_device, proj, m, kind):
    """Prefill shapes with 1% outlier columns (x50): GPU float64 reference of the dequantized operands."""
    n, k = LLAMA3_8B[proj]
    gen = torch.Generator(device=cuda_device).manual_seed(101 + m)
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=cuda_device, generator=gen)
    d = (torch.rand((n, k // 256), device=cuda_device, generator=gen) * 9e-3 + 1e-3).half()
    raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
    fields = prepare_iq3_s_fields(raw)
    x = torch.randn((m, k), device=cuda_device, generator=gen)
    cols = torch.randperm(k, device=cuda_device, generator=gen)[: round(0.01 * k)]
    x[:, cols] *= 50.0
    xq, xs = launch_quantize_fp8(x.to(torch.bfloat16))
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, config=KINDS[kind])
    bits, scales = launch_dequant_iq3_s(fields)
    lut = torch.from_numpy(O.decode_e4m3(np.arange(256, dtype=np.uint8))).to(cuda_device)
    w = (lut[bits.long()] * scales.repeat_interleave(32, dim=1)).double()
    del bits, scales
    xe = lut[xq.long()].double() * torch.exp2(xs.double() - 127).repeat_interleave(32, dim=1)
    ref = xe @ w.t()
    err = (torch.linalg.norm(out.double() - ref) / torch.linalg.norm(ref)).item()
    assert err < REL_FROB_TOL, err


def test_gemv_after_gemm_on_one_stream(cuda_device):
    """The GEMM and the GEMV share the per-stream workspace; the GEMV's split-K counters must stay zero."""
    fields, xq, xs, _ = _case(cuda_device, 256, 1024, 2048, seed=77)
    raw = O.make_synthetic_iq3s(1024, 2048, 77)
    rng = np.random.default_rng(78)
    for _ in range(2):
        launch_iq3_s_fp8_matmul(xq, xs, fields, config=GEMM)
        launch_iq3_s_fp8_matmul(xq, xs, fields, config=GEMM_F16)
        x8q, x8s = O.quantize_mxfp8(rng.standard_normal((8, 2048)).astype(np.float32))
        ref = O.iq3s_linear_f64(x8q, x8s, raw)
        out = launch_iq3_s_fp8_matmul(torch.from_numpy(x8q).to(cuda_device), torch.from_numpy(x8s).to(cuda_device),
                                      fields)
        assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL


def test_f16_operands_exact_across_wide_scale_ranges(cuda_device):
    """Groups up to 2^12 below the token's largest scale stay exact in the FP16 activation operand."""
    raw = O.make_synthetic_iq3s(256, 2048, 88)
    rng = np.random.default_rng(89)
    x = rng.standard_normal((64, 2048)).astype(np.float32)
    x *= np.exp2(rng.integers(-12, 1, size=(64, 2048 // 32)).repeat(32, axis=1)).astype(np.float32)
    xq, xs = O.quantize_mxfp8(x)
    ref = O.iq3s_linear_f64(xq, xs, raw)
    fields = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))
    out = launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device), fields,
                                  config=GEMM_F16)
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL


def test_default_path_sizes_its_workspace_on_a_fresh_stream(cuda_device):
    """The workspace query resolves the automatic kernel choice the way the call does."""
    fields, xq, xs, ref = _case(cuda_device, 300, 256, 4096, seed=91)
    stream = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(stream):
        out = launch_iq3_s_fp8_matmul(xq, xs, fields, stream=stream)
    stream.synchronize()
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL


@pytest.mark.parametrize("m,n,k,outliers", [(32, 256, 2048, False), (130, 384, 4096, True), (257, 136, 3072, False),
                                            (64, 1024, 7168, True)])
@pytest.mark.parametrize("split", [2, 3, 8])
def test_gemm_k_split_matches_oracle(cuda_device, m, n, k, outliers, split):
    """The FP16 GEMM with each output tile's K blocks split over CTAs (partials summed in K order)."""
    fields, xq, xs, ref = _case(cuda_device, m, n, k, seed=1300 + m + n + split, outliers=outliers)
    cfg = dict(GEMM_F16, split=split)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, config=cfg)
    got = to_np(out).astype(np.float64)
    assert O.relative_frobenius(got, ref) < ORACLE_FROB_TOL
    np.testing.assert_allclose(got, ref, rtol=5e-4, atol=5e-4 * np.abs(ref).max())
    # Deterministic (the sum order does not depend on which part arrives last), and the counters
    # are left zero: a second call and a GEMV call after it give the same answers.
    again = launch_iq3_s_fp8_matmul(xq, xs, fields, config=cfg)
    assert torch.equal(out, again)
    bf = launch_iq3_s_fp8_matmul(xq, xs, fields, config=cfg, out_dtype=torch.bfloat16)
    assert O.relative_frobenius(to_np(bf.float()), ref) < 4e-3
    x8 = xq[:8].contiguous(), xs[:8].contiguous()
    small = launch_iq3_s_fp8_matmul(*x8, fields)
    assert O.relative_frobenius(to_np(small), ref[:8]) < ORACLE_FROB_TOL


def test_default_split_on_few_tiles_matches_oracle(cuda_device):
    """Llama-3-70B O projection at 64 tokens: 64 output tiles, so the default config splits K."""
    from mambo_b200.kernels.iq3_s_fp8 import select_config

    fields, xq, xs, ref = _case(cuda_device, 64, 8192, 8192, seed=1401, outliers=True)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields)
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL
    assert select_config(64, 8192, 8192, cuda_device)["kernel"] in (_lib.MAMBO_KERNEL_AUTO,
                                                                    _lib.MAMBO_KERNEL_GEMM_F16,
                                                                    _lib.MAMBO_KERNEL_GEMM_F16_PAIR)


GEMM_F16_FOLD = {"kernel": _lib.MAMBO_KERNEL_GEMM_F16_FOLD, "warps": 8, "stages": 4}
FOLD_FROB_TOL = 1e-3  # north star bound; each folded weight carries one or two FP16 roundings (~4e-4 RMS)


@pytest.mark.parametrize("m,n,k,outliers", [(32, 256, 512, False), (130, 384, 1024, True), (257, 136, 512, False),
                                            (64, 640, 1536, True), (300, 256, 2048, True)])
@pytest.mark.parametrize("stages,split", [(2, 1), (3, 1), (4, 1), (4, 3)])
def test_folded_gemm_within_north_star_bound(cuda_device, m, n, k, outliers, stages, split):
    fields, xq, xs, ref = _case(cuda_device, m, n, k, seed=1700 + m + n + stages + split, outliers=outliers)
    cfg = dict(GEMM_F16_FOLD, stages=stages, split=split)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, config=cfg)
    got = to_np(out).astype(np.float64)
    err = O.relative_frobenius(got, ref)
    assert err < FOLD_FROB_TOL, err
    np.testing.assert_allclose(got, ref, rtol=4e-3, atol=2e-3 * np.abs(ref).max())
    assert torch.equal(out, launch_iq3_s_fp8_matmul(xq, xs, fields, config=cfg))  # deterministic


def test_folded_gemm_wide_scale_ranges(cuda_device):
    """Block scales spread over 2^10 within a row, and a zero block: the per-row exponent keeps every
    folded weight in FP16's normal range."""
    raw = O.make_synthetic_iq3s(256, 4096, 1801)
    rng = np.random.default_rng(1802)
    d = (np.exp2(rng.integers(-16, -6, size=(256, 16))) * rng.uniform(1, 2, size=(256, 16))).astype("<f2")
    d[5, 3] = 0
    raw[..., :2] = d.view(np.uint8).reshape(256, 16, 2)
    xq, xs = O.quantize_mxfp8(rng.standard_normal((96, 4096)).astype(np.float32))
    ref = O.iq3s_linear_f64(xq, xs, raw)
    fields = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))
    out = launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device),
                                  fields, config=GEMM_F16_FOLD)
    assert O.relative_frobenius(to_np(out), ref) < FOLD_FROB_TOL


@pytest.mark.parametrize("proj", sorted(LLAMA3_8B))
def test_folded_full_size_prefill(cuda_device, proj):
    """Llama-3-8B shapes at M = 2048 with 1 % outlier columns (x50) against a float64 GPU reference."""
    n, k = LLAMA3_8B[proj]
    m = 2048
    gen = torch.Generator(device=cuda_device).manual_seed(1901 + n)
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=cuda_device, generator=gen)
    d = (torch.rand((n, k // 256), device=cuda_device, generator=gen) * 9e-3 + 1e-3).half()
    raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
    fields = prepare_iq3_s_fields(raw)
    x = torch.randn((m, k), device=cuda_device, generator=gen)
    x[:, torch.randperm(k, device=cuda_device, generator=gen)[: round(0.01 * k)]] *= 50.0
    xq, xs = launch_quantize_fp8(x.to(torch.bfloat16))
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, config=GEMM_F16_FOLD)
    bits, scales = launch_dequant_iq3_s(fields)
    lut = torch.from_numpy(O.decode_e4m3(np.arange(256, dtype=np.uint8))).to(cuda_device)
    w = (lut[bits.long()] * scales.repeat_interleave(32, dim=1)).double()
    del bits, scales
    xe = lut[xq.long()].double() * torch.exp2(xs.double() - 127).repeat_interleave(32, dim=1)
    ref = xe @ w.t()
    err = (torch.linalg.norm(out.double() - ref) / torch.linalg.norm(ref)).item()
    assert err < FOLD_FROB_TOL, err


GEMM_F16_WIDE = {"kernel": _lib.MAMBO_KERNEL_GEMM_F16_WIDE, "warps": 8, "stages": 4}


@pytest.mark.parametrize("m,n,k,outliers", [(32, 256, 512, False), (130, 384, 1024, True), (257, 136, 512, False),
                                            (300, 256, 2048, True), (513, 520, 1024, True), (64, 1032, 768, False)])
@pytest.mark.parametrize("stages", [2, 3, 4])
def test_wide_gemm_within_north_star_bound(cuda_device, m, n, k, outliers, stages):
    """256 x 256-token tiles on CTA pairs (block scale folded): ragged M and N, a lone last row tile of a
    pair, token tiles past M; within the folded bound, deterministic, and equal to the single-CTA folded
    kernel to FP32 rounding."""
    fields, xq, xs, ref = _case(cuda_device, m, n, k, seed=2100 + m + n + stages, outliers=outliers)
    cfg = dict(GEMM_F16_WIDE, stages=stages)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, config=cfg)
    got = to_np(out).astype(np.float64)
    err = O.relative_frobenius(got, ref)
    assert err < FOLD_FROB_TOL, err
    np.testing.assert_allclose(got, ref, rtol=4e-3, atol=2e-3 * np.abs(ref).max())
    assert torch.equal(out, launch_iq3_s_fp8_matmul(xq, xs, fields, config=cfg))  # deterministic
    fold = launch_iq3_s_fp8_matmul(xq, xs, fields, config=dict(GEMM_F16_FOLD, stages=stages))
    assert O.relative_frobenius(got, to_np(fold).astype(np.float64)) < 1e-5


@pytest.mark.parametrize("m,n,k", [(600, 1024, 1024), (2048, 512, 2048)])
def test_wide_gemm_bf16_output_is_the_rounded_f32_output(cuda_device, m, n, k):
    """bf16 output leaves through the staging tile and TMA stores, two per 256-token tile."""
    fields, xq, xs, _ = _case(cuda_device, m, n, k, seed=2200 + m)
    f32 = launch_iq3_s_fp8_matmul(xq, xs, fields, config=GEMM_F16_WIDE)
    b16 = launch_iq3_s_fp8_matmul(xq, xs, fields, config=GEMM_F16_WIDE, out_dtype=torch.bfloat16)
    assert torch.equal(b16, f32.to(torch.bfloat16))


@pytest.mark.parametrize("proj", sorted(LLAMA3_8B))
def test_wide_full_size_prefill(cuda_device, proj):
    """Llama-3-8B shapes at M = 2048 with 1 % outlier columns (x50) against a float64 GPU reference."""
    n, k = LLAMA3_8B[proj]
    m = 2048
    gen = torch.Generator(device=cuda_device).manual_seed(2301 + n)
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=cuda_device, generator=gen)
    d = (torch.rand((n, k // 256), device=cuda_device, generator=gen) * 9e-3 + 1e-3).half()
    raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
    fields = prepare_iq3_s_fields(raw)
    x = torch.randn((m, k), device=cuda_device, generator=gen)
    x[:, torch.randperm(k, device=cuda_device, generator=gen)[: round(0.01 * k)]] *= 50.0
    xq, xs = launch_quantize_fp8(x.to(torch.bfloat16))
    out = launch_iq3_s_fp8_matmul(xq, xs, fields, config=GEMM_F16_WIDE)
    bits, scales = launch_dequant_iq3_s(fields)
    lut = torch.from_numpy(O.decode_e4m3(np.arange(256, dtype=np.uint8))).to(cuda_device)
    w = (lut[bits.long()] * scales.repeat_interleave(32, dim=1)).double()
    del bits, scales
    xe = lut[xq.long()].double() * torch.exp2(xs.double() - 127).repeat_interleave(32, dim=1)
    ref = xe @ w.t()
    err = (torch.linalg.norm(out.double() - ref) / torch.linalg.norm(ref)).item()
    assert err < FOLD_FROB_TOL, err
