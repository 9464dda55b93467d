"""Row-split linear with its all-reduce fused into the GEMV (mambo_iq3s_linear_fused_ar) on one B200.

A one-rank communicator runs the whole device path (the partials written to
the exchange slots, the epoch-tagged flags, the rank-order sum and the epoch
advance between launches) without a peer; the two-GPU parity test lives in
tests/test_sharding_gpu.py. The result must equal the plain fused linear and
stay within the oracle bound, call after call (the exchange slots alternate
between two buffers by launch parity).
"""

from __future__ import annotations

import pytest
import torch

from oracle import iq3s_oracle as O

pytestmark = pytest.mark.gpu

FROB_TOL = 1e-3  # relative Frobenius error against the float64 oracle, as in the other linear tests


def _weight(n, k, seed, dev):
    gen = torch.Generator(device=dev).manual_seed(seed)
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
    raw[..., :2] = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half() \
        .view(torch.uint8).view(n, k // 256, 2)
    return raw


@pytest.fixture(scope="module")
def comm():
    from mambo_b200.sharding import FusedAllReduce

    c = FusedAllReduce(14336)
    yield c
    c.close()


@pytest.mark.parametrize("m", [1, 8, 13, 31])
@pytest.mark.parametrize("n,k", [(4096, 4096), (14336, 4096), (4096, 14336)])
def test_fused_allreduce_one_rank_matches_fused_linear(comm, m, n, k):
    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_ar_into, fused_linear_into, select_config
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    dev = torch.device("cuda", 0)
    raw = _weight(n, k, 100 + m, dev)
    w = prepare_iq3_s_fields(raw)
    gen = torch.Generator(device=dev).manual_seed(7 + m)
    x = torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16)
    # The plan the fused all-reduce runs: the tuned configuration on the tcgen05 GEMV with whole row tiles or
    # a cluster K split (each row's sum formed in one CTA), so the single-rank result is bit-identical.
    cfg = dict(select_config(m, n, k, dev), kernel=1, warps=8, loader=0)
    cfg["split"] = 1 if cfg["split"] == 1 else 2
    ref = torch.empty((m, n), dtype=torch.float32, device=dev)
    fused_linear_into(x, w, ref, config=cfg)
    for call in range(3):  # both slot buffers, then the first again
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device=dev)
        fused_linear_ar_into(x, w, out, comm, config=cfg)
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"call {call}"
    if m in (1, 13) and n == 4096 and k == 4096:
        expected = O.iq3s_linear_f64(*O.quantize_mxfp8(x.float().cpu().numpy()), raw.cpu().numpy())
        assert O.relative_frobenius(out.cpu().numpy(), expected) < FROB_TOL


def test_fused_allreduce_bf16_output_and_sharded_row_linear(comm):
    from mambo_b200.sharding import ROW, TensorParallelIQ3SLinear

    dev = torch.device("cuda", 0)
    n, k, m = 4096, 14336, 8
    raw = _weight(n, k, 5, dev)
    lin = TensorParallelIQ3SLinear(raw, ROW, out_dtype=torch.bfloat16)
    gen = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16)
    want = lin(x).float()  # local() + combine() (one rank: no collective); its own K split
    for _ in range(2):
        got = lin.fused(x, comm)
        torch.cuda.synchronize()
        assert got.dtype == torch.bfloat16 and got.shape == (m, n)
        err = (torch.linalg.norm((got.float() - want).double()) / torch.linalg.norm(want.double())).item()
        assert err < FROB_TOL, err


def test_fused_allreduce_rejects_bad_calls(comm):
    from mambo_b200 import _lib
    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_ar_into
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    dev = torch.device("cuda", 0)
    w = prepare_iq3_s_fields(_weight(16384, 4096, 3, dev))  # more rows than the communicator holds
    x = torch.randn((4, 4096), device=dev).to(torch.bfloat16)
    with pytest.raises(ValueError, match="exceeds the communicator"):
        fused_linear_ar_into(x, w, torch.empty((4, 16384), device=dev), comm)
    w = prepare_iq3_s_fields(_weight(4096, 4096, 4, dev))
    with pytest.raises(ValueError, match="1 to 31 tokens"):
        fused_linear_ar_into(torch.randn((32, 4096), device=dev).to(torch.bfloat16), w,
                             torch.empty((32, 4096), device=dev), comm)
    assert _lib.load().mambo_iq3s_linear_fused_ar(None, 0, 0, 0, None, None, None, 0, 0, None, None, None, 0,
                                                  None) == _lib.MAMBO_EINVAL
