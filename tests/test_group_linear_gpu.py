"""GPU parity of grouped linears (mambo_iq3s_linear_group): several independent
IQ3_S x MXFP8 linears in one persistent launch.

Each item must be what iq3_s_fp8_linear gives for it. The grouped launch
splits the concatenated units of all items by stream-K, so an item's FP32
partial sums may be added in another order than in its own launch: results
agree to FP32 rounding, and bit for bit when the split is the same (a group of
one against a single stream-K launch).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import iq3s_oracle as O
from mambo_b200 import _lib
from mambo_b200.kernels.iq3_s_fp8 import iq3_s_fp8_linear, iq3_s_fp8_linear_group
from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

pytestmark = pytest.mark.gpu

ORACLE_FROB_TOL = 1e-4
STREAM_K = {"kernel": _lib.MAMBO_KERNEL_GEMV, "warps": 8, "stages": 8, "ctas_per_sm": 1, "split": 0, "prefetch": 0}


def _weight(dev, n, k, seed):
    raw = O.make_synthetic_iq3s(n, k, seed)
    return raw, prepare_iq3_s_fields(torch.from_numpy(raw).to(dev))


def _x(dev, m, k, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    x[:, rng.permutation(k)[: max(1, k // 100)]] *= 50.0
    return torch.from_numpy(x).to(dev).to(torch.bfloat16)


def _oracle(x, raw):
    xq, xs = O.quantize_mxfp8(x.float().cpu().numpy())
    return O.iq3s_linear_f64(xq, xs, raw)


def _kernels(fn) -> list[str]:
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    return [e.name for e in prof.events()
            if e.device_type == torch.autograd.DeviceType.CUDA and ("iq3s" in e.name or "mxfp8" in e.name)]


@pytest.mark.parametrize("m", [1, 5, 8, 17])
def test_group_of_one_equals_single_stream_k_launch(cuda_device, m):
    _, w = _weight(cuda_device, 1024, 2048, seed=10 + m)
    x = _x(cuda_device, m, 2048, seed=20 + m)
    (g,) = iq3_s_fp8_linear_group([x], [w], out_dtype=torch.float32)
    single = iq3_s_fp8_linear(x, w, out_dtype=torch.float32, config=STREAM_K)
    assert torch.equal(g.view(torch.int32), single.view(torch.int32))


def test_mixed_group_matches_each_linear_and_the_oracle(cuda_device):
    shapes = [(1, 264, 512), (3, 1024, 2048), (8, 384, 768), (2, 136, 256), (5, 2048, 1024), (8, 520, 3072)]
    raws, ws, xs = [], [], []
    for i, (m, n, k) in enumerate(shapes):
        raw, w = _weight(cuda_device, n, k, seed=100 + i)
        raws.append(raw)
        ws.append(w)
        xs.append(_x(cuda_device, m, k, seed=200 + i))
    outs = iq3_s_fp8_linear_group(xs, ws, out_dtype=torch.float32)
    for x, w, raw, out in zip(xs, ws, raws, outs):
        one = iq3_s_fp8_linear(x, w, out_dtype=torch.float32)
        assert out.shape == one.shape
        assert O.relative_frobenius(out.cpu().numpy(), one.cpu().numpy().astype(np.float64)) < 1e-5
        assert O.relative_frobenius(out.cpu().numpy(), _oracle(x, raw)) < ORACLE_FROB_TOL


def test_group_mixes_token_tiles_and_output_types(cuda_device):
    """Items of 20 and 2 tokens share the 32-token tile; each keeps its own M and output dtype."""
    raw_a, wa = _weight(cuda_device, 512, 1024, seed=31)
    raw_b, wb = _weight(cuda_device, 256, 2048, seed=32)
    xa, xb = _x(cuda_device, 20, 1024, seed=33), _x(cuda_device, 2, 2048, seed=34)
    ya, yb = iq3_s_fp8_linear_group([xa, xb], [wa, wb], out_dtype=torch.bfloat16)
    assert ya.shape == (20, 512) and yb.shape == (2, 256) and ya.dtype == torch.bfloat16
    assert O.relative_frobenius(ya.float().cpu().numpy(), _oracle(xa, raw_a)) < 4e-3
    assert O.relative_frobenius(yb.float().cpu().numpy(), _oracle(xb, raw_b)) < 4e-3


def test_group_is_one_launch_and_deterministic(cuda_device):
    ws, xs = [], []
    for i, (n, k) in enumerate([(6144, 4096), (4096, 4096), (14336, 4096), (4096, 14336)]):
        ws.append(_weight(cuda_device, n, k, seed=40 + i)[1])
        xs.append(_x(cuda_device, 4, k, seed=50 + i))
    a = iq3_s_fp8_linear_group(xs, ws)
    kernels = _kernels(lambda: iq3_s_fp8_linear_group(xs, ws))
    if kernels:
        assert len(kernels) == 1 and "gemv_tm" in kernels[0], kernels
    b = iq3_s_fp8_linear_group(xs, ws)
    for ya, yb in zip(a, b):
        assert torch.equal(ya, yb)


def test_group_falls_back_per_item(cuda_device):
    """An f32 activation (or an unaligned row) sends the group down the per-item path: same results as alone."""
    _, w1 = _weight(cuda_device, 256, 1024, seed=61)
    _, w2 = _weight(cuda_device, 512, 512, seed=62)
    x1 = _x(cuda_device, 3, 1024, seed=63).float() * 1.0001
    big = _x(cuda_device, 4, 512 + 3, seed=64)
    x2 = big[:, :512]
    y1, y2 = iq3_s_fp8_linear_group([x1, x2], [w1, w2], out_dtype=torch.float32)
    assert torch.equal(y1, iq3_s_fp8_linear(x1, w1, out_dtype=torch.float32))
    assert torch.equal(y2, iq3_s_fp8_linear(x2, w2, out_dtype=torch.float32))


def test_group_size_limit(cuda_device):
    _, w = _weight(cuda_device, 8, 256, seed=71)
    xs = [_x(cuda_device, 1, 256, seed=72 + i) for i in range(_lib.MAMBO_MAX_GROUP)]
    outs = iq3_s_fp8_linear_group(xs, [w] * len(xs), out_dtype=torch.float32)
    for x, y in zip(xs, outs):
        assert torch.allclose(y, iq3_s_fp8_linear(x, w, out_dtype=torch.float32), rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        iq3_s_fp8_linear_group(xs + xs[:1], [w] * (len(xs) + 1))


def test_decode_sweep_as_one_group(cuda_device):
    """The 20 linears of the decode sweep (Llama-3-8B shapes, M in {1,2,4,8}) in one launch."""
    shapes = [(6144, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
    gen = torch.Generator(device=cuda_device).manual_seed(7)
    ws = []
    for n, k in shapes:
        raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=cuda_device, generator=gen)
        raw[..., :2] = (torch.rand((n, k // 256), device=cuda_device, generator=gen) * 9e-3 + 1e-3).half() \
            .view(torch.uint8).view(n, k // 256, 2)
        ws.append(prepare_iq3_s_fields(raw))
    xs, wl = [], []
    for m in (1, 2, 4, 8):
        for (n, k), w in zip(shapes, ws):
            xs.append(torch.randn((m, k), device=cuda_device, generator=gen).to(torch.bfloat16))
            wl.append(w)
    outs = iq3_s_fp8_linear_group(xs, wl, out_dtype=torch.float32)
    for x, w, y in zip(xs, wl, outs):
        one = iq3_s_fp8_linear(x, w, out_dtype=torch.float32)
        err = (torch.linalg.norm(y.double() - one.double()) / torch.linalg.norm(one.double())).item()
        assert err < 1e-5, err


def test_tensor_parallel_local_group_matches_separate_shards(cuda_device):
    """Column shards that read the same activation (gate and up) as one grouped launch on a rank."""
    from mambo_b200.sharding import COLUMN, TensorParallelIQ3SLinear, local_group

    gen = torch.Generator(device=cuda_device).manual_seed(81)
    lins = []
    for n in (1024, 1536):
        raw = torch.randint(0, 256, (n, 8, 110), dtype=torch.uint8, device=cuda_device, generator=gen)
        raw[..., :2] = (torch.rand((n, 8), device=cuda_device, generator=gen) * 9e-3 + 1e-3).half() \
            .view(torch.uint8).view(n, 8, 2)
        lins.append(TensorParallelIQ3SLinear(raw, COLUMN, out_dtype=torch.float32))
    x = torch.randn((4, 2048), device=cuda_device, generator=gen).to(torch.bfloat16)
    grouped = local_group(lins, x)
    for lin, y in zip(lins, grouped):
        one = lin.local(x)
        assert y.shape == one.shape
        err = (torch.linalg.norm(y.double() - one.double()) / torch.linalg.norm(one.double())).item()
        assert err < 1e-5, err


def test_time_balanced_split_with_unequal_items(cuda_device):
    """Items from 1 to 31 tokens: the launch cuts stream-K ranges by estimated time, so CTAs
    get very different unit counts and some ranges lie inside one row tile. Every item must
    still match its own launch, and repeated launches must agree bit for bit."""
    shapes = [(1, 1024, 2048), (31, 512, 1024), (2, 2048, 1024), (17, 256, 3072),
              (5, 1536, 512), (31, 768, 2048), (1, 136, 256), (9, 1024, 1024)]
    raws, ws, xs = [], [], []
    for i, (m, n, k) in enumerate(shapes):
        raw, w = _weight(cuda_device, n, k, seed=900 + i)
        raws.append(raw)
        ws.append(w)
        xs.append(_x(cuda_device, m, k, seed=950 + i))
    a = iq3_s_fp8_linear_group(xs, ws, out_dtype=torch.float32)
    b = iq3_s_fp8_linear_group(xs, ws, out_dtype=torch.float32)
    for x, w, raw, ya, yb in zip(xs, ws, raws, a, b):
        assert torch.equal(ya, yb)
        one = iq3_s_fp8_linear(x, w, out_dtype=torch.float32)
        assert O.relative_frobenius(ya.cpu().numpy(), one.cpu().numpy().astype(np.float64)) < 1e-5
    for i in (1, 6):
        assert O.relative_frobenius(a[i].cpu().numpy(), _oracle(xs[i], raws[i])) < ORACLE_FROB_TOL
