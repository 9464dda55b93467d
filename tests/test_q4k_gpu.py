"""Q4_K x MXFP8 linear on the tcgen05 GEMV against the Q4_K oracle.

The reference lists Q4_K in its GGUF tensor-type table
(src/python/mambo/utils/gguf_manifest.py:30-42) without a kernel; the oracle
(oracle/gguf_quants_oracle.py) restates the block decode and is pinned bit for
bit to gguf-py 0.19.0 (tests/test_gguf_quants_oracle.py). The kernel's
arithmetic is the oracle's group decomposition: per 32-weight group the tensor
cores' partial product of the exact E4M3 codes times d*s_g, minus dmin*m_g
times the token's group sum of the quantized activations. The bar is the one
of the IQ3_S linear: relative Frobenius error below 1e-4 against the float64
product of the same MXFP8 activations and the exact weights.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mambo_b200 import _lib
from mambo_b200.kernels.q4_k_fp8 import launch_q4_k_fp8_matmul, launch_quantize_fp8_sums, prepare_q4_k_fields, \
    q4_k_fp8_linear
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from oracle import gguf_quants_oracle as G
from oracle import iq3s_oracle as O

pytestmark = pytest.mark.gpu

ORACLE_FROB_TOL = 1e-4  # FP32 accumulation against the float64 product of the same operands


def _x(dev, m, k, seed):
    x = np.random.default_rng(seed).standard_normal((m, k)).astype(np.float32)
    x[:, np.random.default_rng(seed + 1).permutation(k)[: max(1, k // 100)]] *= 50.0
    return torch.from_numpy(x).to(dev).to(torch.bfloat16)


def _stored_codes(codes: np.ndarray) -> np.ndarray:
    """Code bytes [..., 128] -> the packed words' bytes: per 4 bytes, their low nibbles in the word's
    low half and their high nibbles in its high half, each q stored as 2q - 15 in sign/magnitude form
    ((v > 0) << 3 | (|v| - 1) / 2, i.e. q for q >= 8 and 7 - q below)."""
    c = codes.astype(np.uint32).reshape(*codes.shape[:-1], 32, 4)
    lo, hi = c & 15, c >> 4
    lo, hi = np.where(lo >= 8, lo, 7 - lo), np.where(hi >= 8, hi, 7 - hi)
    shift = np.arange(4, dtype=np.uint32) * 4
    word = (lo << shift).sum(axis=-1) | ((hi << shift).sum(axis=-1) << 16)
    return word.astype("<u4").view(np.uint8).reshape(codes.shape)


def _packed_layout(raw: np.ndarray) -> np.ndarray:
    """The documented record layout, restated in NumPy: per (128-row tile, K block) the stored codes
    [8 chunks][128 rows][16 B], then [128 rows] d|dmin (4 B), then [128 rows] 12 scale bytes."""
    n, b, _ = raw.shape
    tiles = (n + 127) // 128
    pad = np.zeros((tiles * 128, b, 144), dtype=np.uint8)
    pad[:n] = raw
    out = []
    for t in range(tiles):
        rows = pad[t * 128:(t + 1) * 128]
        for kb in range(b):
            blk = rows[:, kb]
            codes = _stored_codes(blk[:, 16:144]).reshape(128, 8, 16).transpose(1, 0, 2).reshape(-1)
            out += [codes, blk[:, 0:4].reshape(-1), blk[:, 4:16].reshape(-1)]
    return np.concatenate(out)


@pytest.mark.parametrize("n,k", [(256, 512), (200, 768), (8, 256)])
def test_pack_layout(cuda_device, n, k):
    raw = G.make_synthetic_q4_k(n, k, seed=n + k)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    torch.cuda.synchronize()
    assert w["packed"].numel() == _lib.load().mambo_q4k_packed_bytes(n, k // 256)
    assert np.array_equal(w["packed"].cpu().numpy(), _packed_layout(raw))


def test_pack_from_strided_bytes(cuda_device):
    """A [N, B*144] view with a row stride larger than the row packs like the contiguous bytes."""
    raw = G.make_synthetic_q4_k(128, 512, seed=3)
    wide = torch.zeros((128, 2 * 144 + 40), dtype=torch.uint8, device=cuda_device)
    wide[:, :288] = torch.from_numpy(raw.reshape(128, -1)).to(cuda_device)
    a = prepare_q4_k_fields(wide[:, :288])
    b = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    assert torch.equal(a["packed"], b["packed"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantizer_group_sums_are_exact(cuda_device, dtype):
    x = _x(cuda_device, 7, 1024, seed=21).to(dtype)
    q, s, sums = launch_quantize_fp8_sums(x)
    eq, es = launch_quantize_fp8(x)
    torch.cuda.synchronize()
    assert torch.equal(q, eq) and torch.equal(s, es)
    xe = O.decode_mxfp8(q.cpu().numpy(), s.cpu().numpy()).astype(np.float64)
    ref = xe.reshape(7, 32, 32).sum(axis=2).astype(np.float32)  # exact in float64, then representable
    assert np.array_equal(sums.cpu().numpy(), ref)


def _oracle(xq, xs, raw):
    xe = O.decode_mxfp8(xq.cpu().numpy(), xs.cpu().numpy())
    return G.q4_k_linear_group_decomposed(xe, raw)


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9, 13, 16, 17, 31, 32, 33, 70])
def test_linear_matches_oracle(cuda_device, m):
    n, k = 384, 2048
    raw = G.make_synthetic_q4_k(n, k, seed=100 + m)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    xq, xs, xsum = launch_quantize_fp8_sums(_x(cuda_device, m, k, seed=200 + m))
    out = launch_q4_k_fp8_matmul(xq, xs, xsum, w)
    torch.cuda.synchronize()
    err = O.relative_frobenius(out.cpu().numpy(), _oracle(xq, xs, raw))
    assert err < ORACLE_FROB_TOL, err


@pytest.mark.parametrize("n,k", [(1000, 512), (8, 256), (136, 1280), (4096, 4096)])
def test_ragged_shapes(cuda_device, n, k):
    """N not a multiple of the 128-row tile (or of 8), a single K block, more K blocks than tiles."""
    raw = G.make_synthetic_q4_k(n, k, seed=n * 3 + k)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    xq, xs, xsum = launch_quantize_fp8_sums(_x(cuda_device, 4, k, seed=n))
    out = torch.full((4, n), float("nan"), device=cuda_device)
    launch_q4_k_fp8_matmul(xq, xs, xsum, w, out=out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert O.relative_frobenius(got, _oracle(xq, xs, raw)) < ORACLE_FROB_TOL


@pytest.mark.parametrize("stages,prefetch", [(2, 0), (4, 8), (8, 0), (10, 4)])
def test_pipeline_depths_give_one_result(cuda_device, stages, prefetch):
    """The stage ring's depth and the L2 prefetch distance change the schedule only: the stream-K ranges
    (set by the grid) and the order of every sum stay, so the results are bit-identical."""
    raw = G.make_synthetic_q4_k(1024, 4096, seed=77)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    xq, xs, xsum = launch_quantize_fp8_sums(_x(cuda_device, 8, 4096, seed=78))
    cfg = {"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": stages, "ctas_per_sm": 1, "split": 0,
           "prefetch": prefetch}
    base = launch_q4_k_fp8_matmul(xq, xs, xsum, w, config=dict(cfg, stages=6, prefetch=0))
    got = launch_q4_k_fp8_matmul(xq, xs, xsum, w, config=cfg)
    torch.cuda.synchronize()
    assert O.relative_frobenius(got.cpu().numpy(), _oracle(xq, xs, raw)) < ORACLE_FROB_TOL
    assert torch.equal(got, base)


@pytest.mark.parametrize("split", [0, 1, 2])
@pytest.mark.parametrize("n,k,m", [(14336, 4096, 1), (4096, 14336, 8), (1024, 2048, 20)])
def test_work_splits_match_oracle(cuda_device, split, n, k, m):
    """Stream-K (0), one CTA per row tile (1) and the cluster K-split (2) on shapes where each is used."""
    raw = G.make_synthetic_q4_k(n, k, seed=split + n + m)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    xq, xs, xsum = launch_quantize_fp8_sums(_x(cuda_device, m, k, seed=k + split))
    cfg = {"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": 6, "ctas_per_sm": 1, "split": split,
           "prefetch": 4}
    out = launch_q4_k_fp8_matmul(xq, xs, xsum, w, config=cfg)
    torch.cuda.synchronize()
    err = O.relative_frobenius(out.cpu().numpy(), _oracle(xq, xs, raw))
    assert err < ORACLE_FROB_TOL, err


@pytest.mark.parametrize("m", [1, 8, 40])
def test_fused_call_equals_quantize_then_linear(cuda_device, m):
    raw = G.make_synthetic_q4_k(512, 1024, seed=300 + m)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    x = _x(cuda_device, m, 1024, seed=301 + m)
    fused = q4_k_fp8_linear(x, w, out_dtype=torch.float32)
    xq, xs, xsum = launch_quantize_fp8_sums(x)
    two = launch_q4_k_fp8_matmul(xq, xs, xsum, w)
    bf = q4_k_fp8_linear(x, w)
    torch.cuda.synchronize()
    assert torch.equal(fused, two)
    assert bf.dtype == torch.bfloat16 and torch.equal(bf, fused.to(torch.bfloat16))


LLAMA3_8B = (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate", 14336, 4096), ("down", 4096, 14336))


@pytest.mark.parametrize("name,n,k", LLAMA3_8B)
@pytest.mark.parametrize("m", [1, 8])
def test_llama3_8b_decode_shapes_match_the_direct_product(cuda_device, name, n, k, m):
    """Full-size decode linears against the direct float64 product of the exact weights."""
    raw = G.make_synthetic_q4_k(n, k, seed=n + k + m)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    xq, xs, xsum = launch_quantize_fp8_sums(_x(cuda_device, m, k, seed=k + m))
    out = launch_q4_k_fp8_matmul(xq, xs, xsum, w)
    torch.cuda.synchronize()
    xe = O.decode_mxfp8(xq.cpu().numpy(), xs.cpu().numpy())
    err = O.relative_frobenius(out.cpu().numpy(), G.q4_k_linear_f64(xe, raw))
    assert err < ORACLE_FROB_TOL, f"{name}: {err}"


def test_zero_activation_rows_give_zero(cuda_device):
    raw = G.make_synthetic_q4_k(256, 512, seed=9)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    x = _x(cuda_device, 3, 512, seed=10)
    x[1] = 0
    out = q4_k_fp8_linear(x, w, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert (out[1] == 0).all()


def test_rejects_bad_inputs(cuda_device):
    raw = G.make_synthetic_q4_k(256, 512, seed=11)
    w = prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device))
    xq, xs, xsum = launch_quantize_fp8_sums(_x(cuda_device, 2, 512, seed=12))
    with pytest.raises(ValueError):
        launch_q4_k_fp8_matmul(xq[:, :256], xs, xsum, w)
    with pytest.raises(ValueError):
        launch_q4_k_fp8_matmul(xq, xs, xsum.double(), w)
    wide = {"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 16, "stages": 4, "ctas_per_sm": 1, "split": 0, "prefetch": 0}
    with pytest.raises(ValueError, match="8 decoder warps"):
        launch_q4_k_fp8_matmul(xq, xs, xsum, w, config=wide)
    with pytest.raises(ValueError, match="GEMV"):
        launch_q4_k_fp8_matmul(xq, xs, xsum, w, config=dict(wide, kernel=_lib.MAMBO_KERNEL_GEMM_F16, warps=8))
    misaligned = torch.empty(2 * 16 + 1, dtype=torch.float32, device=cuda_device)[1:].view(2, 16)
    misaligned.copy_(xsum)
    with pytest.raises(ValueError, match="16-byte aligned"):
        launch_q4_k_fp8_matmul(xq, xs, misaligned, w)
    with pytest.raises(ValueError):
        prepare_q4_k_fields(torch.zeros((4, 145), dtype=torch.uint8, device=cuda_device))


def test_grouped_q4k_linears_match_each_linear_and_the_oracle(cuda_device):
    """Independent Q4_K linears of 1 to 31 tokens in one call: a quantization pre-pass (codes and group
    sums) and one grouped GEMV launch. Each output equals the single fused call to FP32 rounding (the
    stream-K split differs) and the oracle's float64 product of the same MXFP8 operands."""
    from mambo_b200.kernels.q4_k_fp8 import q4_k_fp8_linear, q4_k_fp8_linear_group

    shapes = [(1, 256, 512), (8, 1024, 2048), (3, 384, 1024), (17, 512, 768), (5, 2048, 1024), (31, 128, 256)]
    raws, ws, xs = [], [], []
    for i, (m, n, k) in enumerate(shapes):
        raw = G.make_synthetic_q4_k(n, k, seed=700 + i)
        raws.append(raw)
        ws.append(prepare_q4_k_fields(torch.from_numpy(raw).to(cuda_device)))
        xs.append(_x(cuda_device, m, k, seed=800 + i))
    for _ in range(2):  # the second call reuses the workspace's tiles and sums
        outs = q4_k_fp8_linear_group(xs, ws, out_dtype=torch.float32)
        for x, w, raw, out in zip(xs, ws, raws, outs):
            one = q4_k_fp8_linear(x, w, out_dtype=torch.float32)
            assert O.relative_frobenius(out.cpu().numpy(), one.cpu().numpy().astype(np.float64)) < 1e-5
            xq, xs_ = launch_quantize_fp8(x)
            assert O.relative_frobenius(out.cpu().numpy(), _oracle(xq, xs_, raw)) < ORACLE_FROB_TOL
