"""GPU parity: sm_100a kernels against the oracle and the reference's golden vectors.

Mirrors the reference's tests/python/test_iq3_s_fp8.py case by case and adds
B200-specific coverage (TMA and plain loaders, stream-K split, bf16 output,
full-size Llama-3 shapes through size-independent properties).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import iq3s_oracle as O
from mambo_b200 import _lib
from mambo_b200.kernels.iq3_s_fp8 import (
    iq3_s_fp8_linear,
    iq3_s_fp8_table,
    iq3_s_table,
    launch_dequant_iq3_s,
    launch_iq3_s_fp8_matmul,
)
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

pytestmark = pytest.mark.gpu

# GEMM output bound of the north star: relative Frobenius error vs an fp32/f64
# matmul of the dequantized operands.
REL_FROB_TOL = 1e-3
# Against the float64 oracle on the same MXFP8 inputs: only FP32 accumulation
# error remains (each 32-weight group is summed by the tensor core, then scaled
# and accumulated in FP32).
ORACLE_FROB_TOL = 1e-4


def to_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def gpu_weight(raw: np.ndarray, device):
    return prepare_iq3_s_fields(torch.from_numpy(np.ascontiguousarray(raw)).to(device))


def test_fp8_codebook_preserves_every_iq3_s_magnitude():
    raw = iq3_s_table()
    encoded = iq3_s_fp8_table()
    assert raw.shape == encoded.shape == (512,)
    shifts = (0, 8, 16, 24)
    mags = np.stack([(raw >> s) & 0xFF for s in shifts], axis=-1).astype(np.float32)
    bits = np.stack([(encoded >> s) & 0xFF for s in shifts], axis=-1).astype(np.uint8)
    np.testing.assert_array_equal(O.decode_e4m3(bits), mags)
    np.testing.assert_array_equal(O.decode_e4m3(bits | np.uint8(0x80)), -mags)


def test_iq3_s_decode_matches_gguf_py(golden, cuda_device):
    g = golden["iq3s_decode"]
    raw = g["synth_raw"]
    n_rows, k = raw.shape[0], raw.shape[1] * 256
    q_t, s_t = launch_dequant_iq3_s(gpu_weight(raw, cuda_device), tile_n=4)
    q, scales = to_np(q_t), to_np(s_t)
    assert q.dtype == np.uint8 and q.shape == (n_rows, k)
    assert scales.dtype == np.float32 and scales.shape == (n_rows, k // 32)
    decoded = O.decode_e4m3(q) * np.repeat(scales, 32, axis=1)
    np.testing.assert_array_equal(decoded, g["synth_deq"])
    oq, os_ = O.decode_iq3s_fp8(raw)
    np.testing.assert_array_equal(q, oq)
    np.testing.assert_array_equal(scales, os_)


def test_packed_decode_all_codes_and_sign_nibbles(golden, cuda_device):
    g = golden["iq3s_decode"]
    raw = g["allcodes_raw"]
    expected = g["allcodes_deq"]
    aligned = torch.from_numpy(raw).to(cuda_device)
    # odd-address and strided source views (test_iq3_s_fp8.py:118-131)
    allocation = torch.empty(raw.size + 1, dtype=torch.uint8, device=cuda_device)
    unaligned = allocation[1:].view(raw.shape)
    unaligned.copy_(aligned)
    strided_alloc = torch.empty((raw.shape[0], raw.shape[1], 220), dtype=torch.uint8, device=cuda_device)
    strided = strided_alloc[..., ::2]
    strided.copy_(aligned)
    for source in (aligned, unaligned, strided):
        fields = prepare_iq3_s_fields(source)
        bits, scales = launch_dequant_iq3_s(fields, tile_n=4)
        actual = O.decode_e4m3(to_np(bits)) * np.repeat(to_np(scales), 32, axis=1)
        np.testing.assert_array_equal(actual, expected)


@pytest.mark.parametrize("n_rows,blocks", [(7, 3), (1, 1), (256, 2)])
def test_soa_fields_preserve_every_byte(cuda_device, n_rows, blocks):
    raw = O.make_synthetic_iq3s(n_rows, blocks * 256, seed=0x50A, d_low=0.002, d_high=0.04)
    fields = gpu_weight(raw, cuda_device)
    rec = np.empty_like(raw)
    for t, start, end in ((fields.d, 0, 2), (fields.qs, 2, 66), (fields.qh, 66, 74), (fields.signs, 74, 106),
                          (fields.scales, 106, 110)):
        assert t.is_contiguous() and t.data_ptr() % t.element_size() == 0
        data = to_np(t.contiguous().view(torch.uint8)).reshape(blocks, n_rows, end - start)
        rec[..., start:end] = data.transpose(1, 0, 2)
    np.testing.assert_array_equal(rec, raw)
    assert sum(t.numel() * t.element_size() for t in (fields.d, fields.qs, fields.qh, fields.signs,
                                                         fields.scales)) == raw.nbytes
    assert fields.d.dtype == torch.float16 and fields.qs.dtype == torch.uint32 and fields.qh.dtype == torch.uint16
    assert fields.signs.dtype == torch.int32 and fields.scales.dtype == torch.uint32


@pytest.mark.parametrize("tokens", [5, 33, 128])
def test_f32_to_mxfp8_quantization_matches_reference(golden, cuda_device, tokens):
    g = golden["mxfp8"]
    x = g[f"x_{tokens}"]
    for rounding in ("nearest_even", "ties_down"):
        q_t, s_t = launch_quantize_fp8(torch.from_numpy(x).to(cuda_device), rounding=rounding)
        q, s = to_np(q_t), to_np(s_t)
        assert q.dtype == np.uint8 and q.shape == (tokens, 160)
        assert s.dtype == np.uint8 and s.shape == (tokens, 5)
        np.testing.assert_array_equal(q, g[f"q_{tokens}"])
        np.testing.assert_array_equal(s, g[f"s_{tokens}"])
        assert np.count_nonzero(O.decode_mxfp8(q, s)[0]) == 0


def test_bf16_mxfp8_both_tie_rules_bit_exact(golden, cuda_device):
    g = golden["mxfp8"]
    bits = torch.from_numpy(g["xbf16_bits"].astype(np.int16)).to(cuda_device)
    xb = bits.view(torch.bfloat16)
    q, s = launch_quantize_fp8(xb)
    np.testing.assert_array_equal(to_np(q), g["q_bf16_rne"])
    np.testing.assert_array_equal(to_np(s), g["s_bf16"])
    q, s = launch_quantize_fp8(xb, rounding="ties_down")
    np.testing.assert_array_equal(to_np(q), g["q_bf16_ties_down"])
    # the same values given as f32 quantize identically
    q32, _ = launch_quantize_fp8(xb.float(), rounding="ties_down")
    np.testing.assert_array_equal(to_np(q32), g["q_bf16_ties_down"])


def test_mxfp8_wide_range_and_strided_rows(cuda_device):
    rng = np.random.default_rng(7)
    x = (rng.standard_normal((37, 1024)) * np.exp2(rng.integers(-140, 120, size=(37, 1024)))).astype(np.float32)
    x[3, :64] = 0.0
    x[4, 32:64] = -0.0
    xt = torch.from_numpy(x).to(cuda_device)
    for rounding, orr in (("nearest_even", "rne"), ("ties_down", "ties_down")):
        q, s = launch_quantize_fp8(xt, rounding=rounding)
        eq, es = O.quantize_mxfp8(x, orr)
        np.testing.assert_array_equal(to_np(s), es)
        np.testing.assert_array_equal(to_np(q), eq)
    wide = torch.zeros((37, 2048), device=cuda_device)
    wide[:, :1024] = xt
    q, s = launch_quantize_fp8(wide[:, :1024])  # row stride 2048
    np.testing.assert_array_equal(to_np(q), O.quantize_mxfp8(x)[0])


@pytest.mark.parametrize("m", [3, 4, 5, 8, 9, 33, 128, 129])
def test_synthetic_iq3_s_fp8_matmul_matches_gguf_py(golden, cuda_device, m):
    g = golden["linear"]
    raw = g["raw"]
    fields = gpu_weight(raw, cuda_device)
    rng = np.random.default_rng(20261016)
    x = torch.from_numpy(rng.standard_normal((m, 768), dtype=np.float32)).to(cuda_device)
    xq, xs = launch_quantize_fp8(x)
    np.testing.assert_array_equal(to_np(xq), g[f"q_{m}"])
    np.testing.assert_array_equal(to_np(xs), g[f"s_{m}"])
    expected = g[f"out_{m}"]
    out = launch_iq3_s_fp8_matmul(xq, xs, fields)
    assert out.dtype == torch.float32 and tuple(out.shape) == (m, raw.shape[0])
    np.testing.assert_allclose(to_np(out), expected, rtol=5e-4, atol=5e-3)
    # strided activations (test_iq3_s_fp8.py:202-210)
    sv = torch.empty((m, 2 * 768), dtype=torch.uint8, device=cuda_device)
    sv[:, ::2] = xq
    ss = torch.empty((m, 2 * 768 // 32), dtype=torch.uint8, device=cuda_device)
    ss[:, ::2] = xs
    out2 = launch_iq3_s_fp8_matmul(sv[:, ::2], ss[:, ::2], fields)
    np.testing.assert_allclose(to_np(out2), expected, rtol=5e-4, atol=5e-3)


def _linear_case(cuda_device, m, n, k, seed, outliers=False):
    raw = O.make_synthetic_iq3s(n, k, seed)
    rng = np.random.default_rng(seed + 1)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if outliers:
        cols = rng.permutation(k)[: max(1, round(0.01 * k))]
        x[:, cols] *= 50.0
    xq, xs = O.quantize_mxfp8(x)
    ref = O.iq3s_linear_f64(xq, xs, raw)
    return raw, x, xq, xs, ref


KERNELS = {  # (kernel kind, weight loader)
    "tcgen05": (_lib.MAMBO_KERNEL_GEMV, 0),
    "tcgen05_w16": (_lib.MAMBO_KERNEL_GEMV, 0, 16),
    "sync_tma": (_lib.MAMBO_KERNEL_GEMV_SYNC, 0),
    "sync_plain": (_lib.MAMBO_KERNEL_GEMV_SYNC, 1),
}


@pytest.mark.parametrize("m,n,k", [(1, 256, 512), (2, 384, 1024), (8, 1024, 2048), (13, 512, 768), (32, 640, 1536),
                                   (40, 128, 256), (17, 136, 512)])
@pytest.mark.parametrize("kernel", sorted(KERNELS))
@pytest.mark.parametrize("split", [0, 1, 2])
def test_linear_kernels_and_splits_match_oracle(cuda_device, m, n, k, kernel, split):
    if split == 2 and not KERNELS[kernel][0] == _lib.MAMBO_KERNEL_GEMV:
        pytest.skip("cluster K-split is a tcgen05 GEMV mode")
    raw, _, xq, xs, ref = _linear_case(cuda_device, m, n, k, seed=1000 + m + n)
    fields = gpu_weight(raw, cuda_device)
    kind, loader, *warps = KERNELS[kernel]
    cfg = {"kernel": kind, "warps": warps[0] if warps else 8, "stages": 4 if m <= 16 else 3, "ctas_per_sm": 1,
           "split": split, "loader": loader}
    out = launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device),
                                  fields, config=cfg)
    got = to_np(out).astype(np.float64)
    assert O.relative_frobenius(got, ref) < ORACLE_FROB_TOL
    np.testing.assert_allclose(got, ref, rtol=5e-4, atol=5e-4 * np.abs(ref).max())


@pytest.mark.parametrize("kind,warps,stages,ctas,prefetch", [
    (_lib.MAMBO_KERNEL_GEMV_SYNC, 4, 3, 1, 0), (_lib.MAMBO_KERNEL_GEMV_SYNC, 16, 3, 1, 0),
    (_lib.MAMBO_KERNEL_GEMV_SYNC, 12, 6, 1, 0), (_lib.MAMBO_KERNEL_GEMV, 8, 2, 1, 0), (_lib.MAMBO_KERNEL_GEMV, 16, 3, 1, 8),
    (_lib.MAMBO_KERNEL_GEMV, 8, 3, 1, 0), (_lib.MAMBO_KERNEL_GEMV, 16, 4, 1, 4), (_lib.MAMBO_KERNEL_GEMV, 8, 8, 1, 2)])
@pytest.mark.parametrize("m", [8, 16])
def test_linear_all_warp_stage_configs(cuda_device, kind, warps, stages, ctas, prefetch, m):
    raw, _, xq, xs, ref = _linear_case(cuda_device, m, 1024, 4096, seed=77)
    fields = gpu_weight(raw, cuda_device)
    cfg = {"kernel": kind, "warps": warps, "stages": stages, "ctas_per_sm": ctas, "split": 0, "prefetch": prefetch}
    out = launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device),
                                  fields, config=cfg)
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL


def test_bf16_epilogue_and_fused_entry(cuda_device):
    raw, x, xq, xs, ref = _linear_case(cuda_device, 4, 512, 2048, seed=5)
    fields = gpu_weight(raw, cuda_device)
    out = launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device),
                                  fields, out_dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    assert O.relative_frobenius(to_np(out.float()), ref) < 4e-3  # bf16 output rounding
    out2 = iq3_s_fp8_linear(torch.from_numpy(x).to(cuda_device), fields, out_dtype=torch.float32)
    assert O.relative_frobenius(to_np(out2), ref) < ORACLE_FROB_TOL


def test_deterministic_and_workspace_reusable(cuda_device):
    raw, _, xq, xs, ref = _linear_case(cuda_device, 8, 2048, 4096, seed=9)
    fields = gpu_weight(raw, cuda_device)
    xq_t, xs_t = torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device)
    outs = [launch_iq3_s_fp8_matmul(xq_t, xs_t, fields) for _ in range(4)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    assert O.relative_frobenius(to_np(outs[0]), ref) < ORACLE_FROB_TOL


def test_config_that_does_not_fit_is_a_value_error(cuda_device):
    raw, _, xq, xs, _ = _linear_case(cuda_device, 32, 256, 512, seed=3)
    fields = gpu_weight(raw, cuda_device)
    with pytest.raises(ValueError):
        launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device), fields,
                                config={"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": 12})


@pytest.mark.parametrize("m", [5, 13])
@pytest.mark.parametrize("which", ["values", "scales", "both"])
def test_unaligned_activation_rows_match_oracle(cuda_device, m, which):
    """Activations at odd addresses: the tcgen05 path copies them to 16-byte aligned rows first."""
    raw, _, xq, xs, ref = _linear_case(cuda_device, m, 512, 1024, seed=31 + m)
    fields = gpu_weight(raw, cuda_device)

    def odd(a):
        buf = torch.empty(a.size + 1, dtype=torch.uint8, device=cuda_device)
        view = buf[1:].view(a.shape)
        view.copy_(torch.from_numpy(a).to(cuda_device))
        return view

    q = odd(xq) if which in ("values", "both") else torch.from_numpy(xq).to(cuda_device)
    sc = odd(xs) if which in ("scales", "both") else torch.from_numpy(xs).to(cuda_device)
    out = launch_iq3_s_fp8_matmul(q, sc, fields)
    assert O.relative_frobenius(to_np(out), ref) < ORACLE_FROB_TOL


def _permute_sign_words(w: np.ndarray) -> np.ndarray:
    """Packed-record sign words: bit 4c+j (weight j of code c) moves to bit 8j+7-c."""
    o = np.zeros_like(w)
    for c in range(8):
        for j in range(4):
            o |= ((w >> np.uint32(4 * c + j)) & np.uint32(1)) << np.uint32(8 * j + 7 - c)
    return o


def _permute_qh_words(w: np.ndarray) -> np.ndarray:
    """Packed-record qh words (4 groups): bit 8g+4h+j moves to bit 8j+7-(2g+h)."""
    o = np.zeros_like(w)
    for g in range(4):
        for h in range(2):
            for j in range(4):
                o |= ((w >> np.uint32(8 * g + 4 * h + j)) & np.uint32(1)) << np.uint32(8 * j + 7 - (2 * g + h))
    return o


@pytest.mark.parametrize("m,n,k", [(8, 520, 768), (3, 1024, 2048), (13, 136, 512)])
def test_packed_layout_and_results_match_soa(cuda_device, m, n, k):
    """Tile-major packed records hold the block bytes (sign and qh words bit-permuted); both weight paths
    give identical outputs."""
    raw, _, xq, xs, ref = _linear_case(cuda_device, m, n, k, seed=55 + n)
    soa = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device), packed=False)
    packed = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))
    assert soa.packed is None and packed.packed is not None
    blocks, tiles = k // 256, (n + 127) // 128
    buf = to_np(packed.packed)
    rec = buf[: tiles * blocks * 14080].reshape(tiles, blocks, 14080)
    # Tail: per row of whole tiles, floor(log2(max |d|)) over the row's finite block scales (0 past N).
    d = np.abs(raw[:, :, 0:2].copy().view("<f2")[..., 0].astype(np.float64))
    d[~np.isfinite(d)] = 0
    dmax = d.max(axis=1)
    expect_exp = np.zeros(tiles * 128, dtype=np.int8)
    expect_exp[:n] = np.where(dmax > 0, np.floor(np.log2(np.where(dmax > 0, dmax, 1))), 0).astype(np.int8)
    np.testing.assert_array_equal(buf[tiles * blocks * 14080:][: tiles * 128].view(np.int8), expect_exp)
    pad = np.zeros((tiles * 128, blocks, 110), dtype=np.uint8)
    pad[:n] = raw
    for t in range(tiles):
        rows = pad[t * 128:(t + 1) * 128].transpose(1, 0, 2)  # [B, 128, 110]
        chunk_major = lambda f, w: f.reshape(blocks, 128, -1, w).transpose(0, 2, 1, 3).reshape(blocks, -1)  # noqa: E731
        signs = _permute_sign_words(np.ascontiguousarray(rows[:, :, 74:106]).view("<u4")).view(np.uint8)
        qh = _permute_qh_words(np.ascontiguousarray(rows[:, :, 66:74]).view("<u4")).view(np.uint8)
        expect = np.concatenate([chunk_major(rows[:, :, 2:66], 16), chunk_major(signs, 16),
                                 chunk_major(qh, 4), rows[:, :, 0:2].reshape(blocks, -1),
                                 rows[:, :, 106:110].reshape(blocks, -1)], axis=1)
        np.testing.assert_array_equal(rec[t], expect, err_msg=f"tile {t}")
    xq_t, xs_t = torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device)
    a = launch_iq3_s_fp8_matmul(xq_t, xs_t, soa)
    b = launch_iq3_s_fp8_matmul(xq_t, xs_t, packed)
    assert torch.equal(a, b)
    assert O.relative_frobenius(to_np(b), ref) < ORACLE_FROB_TOL


def test_errors_match_reference(cuda_device):
    fields = gpu_weight(O.make_synthetic_iq3s(8, 256, 1), cuda_device)
    good_q = torch.zeros((2, 256), dtype=torch.uint8, device=cuda_device)
    good_s = torch.zeros((2, 8), dtype=torch.uint8, device=cuda_device)
    with pytest.raises(ValueError):
        launch_iq3_s_fp8_matmul(good_q[:, :128], good_s, fields)
    with pytest.raises(ValueError):
        launch_iq3_s_fp8_matmul(good_q, good_s[:, :4], fields)
    with pytest.raises(TypeError):
        launch_iq3_s_fp8_matmul(good_q, good_s, object())
    with pytest.raises(ValueError):
        launch_quantize_fp8(torch.zeros((2, 33), device=cuda_device))
    with pytest.raises(ValueError):
        launch_quantize_fp8(torch.zeros((2, 64), device=cuda_device), tile_m=3)
    with pytest.raises(ValueError):
        prepare_iq3_s_fields(torch.zeros((2, 1, 109), dtype=torch.uint8, device=cuda_device))
    with pytest.raises(ValueError):
        launch_dequant_iq3_s(fields, tile_n=3)


LLAMA3_8B = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (14336, 4096), "down": (4096, 14336)}


@pytest.mark.parametrize("proj", sorted(LLAMA3_8B))
@pytest.mark.parametrize("m", [1, 8])
def test_full_size_llama3_projection_frobenius(cuda_device, proj, m):
    """Full-size shapes: decode on GPU (bit-exact tested above) -> fp32 matmul reference; <= 1e-3 rel. Frobenius."""
    n, k = LLAMA3_8B[proj]
    gen = torch.Generator(device=cuda_device).manual_seed(11 + m)
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=cuda_device, generator=gen)
    d = (torch.rand((n, k // 256), device=cuda_device, generator=gen) * 9e-3 + 1e-3).half()
    raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
    fields = prepare_iq3_s_fields(raw)
    x = torch.randn((m, k), device=cuda_device, generator=gen).to(torch.bfloat16)
    xq, xs = launch_quantize_fp8(x)
    out = launch_iq3_s_fp8_matmul(xq, xs, fields)
    bits, scales = launch_dequant_iq3_s(fields)
    lut = torch.from_numpy(O.decode_e4m3(np.arange(256, dtype=np.uint8))).to(cuda_device)
    w = lut[bits.long()] * scales.repeat_interleave(32, dim=1)
    xe = lut[xq.long()].double() * torch.exp2(xs.double() - 127).repeat_interleave(32, dim=1)
    ref = xe @ w.double().t()
    err = (torch.linalg.norm(out.double() - ref) / torch.linalg.norm(ref)).item()
    assert err < REL_FROB_TOL, err


def test_bounded_wait_reports_timeout_without_faulting(cuda_device):
    lib = _lib.load()
    _lib.device_status(reset=True)
    _lib.check(lib.mambo_selftest_wait_timeout(2_000_000, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    code, where, _ = _lib.device_status(reset=True)
    assert code == _lib.MAMBO_ETIMEOUT and where == 9
    # the context is still usable
    assert torch.ones(4, device=cuda_device).sum().item() == 4.0
    assert _lib.device_status()[0] == 0
