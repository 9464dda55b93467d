"""Tensor-parallel sharding of the IQ3_S x MXFP8 linear: host logic on CPU (gloo, world size 2).

The per-rank compute is replaced by the oracle (float64 restatement of the
reference's decode + MXFP8 matmul), so these tests check the split, the
activation slicing and the collectives: the sharded result must equal the
unsharded one.
"""

from __future__ import annotations

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import iq3s_oracle as O
from mambo_b200.sharding import COLUMN, ROW, TensorParallelIQ3SLinear, shard_iq3_s_blocks, shard_range


def test_shard_range_splits_whole_units():
    assert [shard_range(4096, r, 4, 8) for r in range(4)] == [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]
    assert shard_range(56, 1, 8, 1) == (7, 14)  # Llama-3-8B down: 56 K blocks over 8 ranks
    with pytest.raises(ValueError):
        shard_range(100, 0, 8, 8)
    with pytest.raises(ValueError):
        shard_range(64, 2, 2, 8)


@pytest.mark.parametrize("mode", [COLUMN, ROW])
def test_shards_partition_the_weight(mode):
    raw = torch.from_numpy(O.make_synthetic_iq3s(64, 1024, 3))
    shards = [shard_iq3_s_blocks(raw, mode, r, 4) for r in range(4)]
    joined = torch.cat(shards, dim=0 if mode == COLUMN else 1)
    assert torch.equal(joined, raw)
    with pytest.raises(ValueError):
        shard_iq3_s_blocks(raw, "diagonal", 0, 4)


# --- two gloo ranks -----------------------------------------------------------

def _oracle_prepare(raw: torch.Tensor):
    return raw.contiguous().numpy()


def _oracle_quantize(x: torch.Tensor):
    xq, xs = O.quantize_mxfp8(x.contiguous().numpy().astype(np.float32))
    return torch.from_numpy(xq), torch.from_numpy(xs)


def _oracle_linear(xq, xs, raw, out_dtype):
    return torch.from_numpy(O.iq3s_linear_f64(xq.contiguous().numpy(), xs.contiguous().numpy(), raw)).to(out_dtype)


def _rank_main(rank, world, port, mode, input_sharded, path):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        raw = torch.from_numpy(O.make_synthetic_iq3s(128, 1024, 17))
        x = torch.from_numpy(np.random.default_rng(5).standard_normal((6, 1024)).astype(np.float32))
        lin = TensorParallelIQ3SLinear(raw, mode, input_is_sharded=input_sharded, out_dtype=torch.float32,
                                       prepare=_oracle_prepare, quantize=_oracle_quantize, linear=_oracle_linear)
        if mode == ROW and input_sharded:
            x = x[:, lin.k0:lin.k0 + lin.local_k]
        y = lin(x)
        if rank == 0:
            np.save(path, y.numpy())
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("mode,input_sharded", [(COLUMN, False), (ROW, False), (ROW, True)])
def test_two_rank_linear_matches_unsharded(mode, input_sharded):
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "y.npy")
        mp.spawn(_rank_main, args=(2, _free_port(), mode, input_sharded, path), nprocs=2, join=True)
        got = np.load(path)
    raw = O.make_synthetic_iq3s(128, 1024, 17)
    x = np.random.default_rng(5).standard_normal((6, 1024)).astype(np.float32)
    if mode == COLUMN:
        xq, xs = O.quantize_mxfp8(x)
        ref = O.iq3s_linear_f64(xq, xs, raw)
        np.testing.assert_array_equal(got, ref.astype(np.float32))  # disjoint output columns: bit-identical
    else:
        # Each rank quantizes its K slice (MXFP8 groups of 32 never straddle 256-weight blocks): the same
        # codes as quantizing the whole row, so only the FP32 sum of the two partials differs.
        xq, xs = O.quantize_mxfp8(x)
        ref = O.iq3s_linear_f64(xq, xs, raw)
        assert O.relative_frobenius(got.astype(np.float64), ref) < 1e-6


def _rank_group_main(rank, world, port, path):
    from mambo_b200.sharding import local_group

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        fakes = dict(prepare=_oracle_prepare, quantize=_oracle_quantize, linear=_oracle_linear)
        gate = TensorParallelIQ3SLinear(torch.from_numpy(O.make_synthetic_iq3s(128, 1024, 21)), COLUMN,
                                        out_dtype=torch.float32, **fakes)
        up = TensorParallelIQ3SLinear(torch.from_numpy(O.make_synthetic_iq3s(64, 1024, 22)), COLUMN,
                                      out_dtype=torch.float32, **fakes)
        down = TensorParallelIQ3SLinear(torch.from_numpy(O.make_synthetic_iq3s(64, 1024, 23)), ROW,
                                        out_dtype=torch.float32, **fakes)
        x = torch.from_numpy(np.random.default_rng(9).standard_normal((5, 1024)).astype(np.float32))
        g, u = local_group([gate, up], x)
        assert g.shape == (5, 64) and u.shape == (5, 32)
        # A row shard in a group runs its own local(): the FP32 partial of its K slice.
        (d,) = local_group([down], x)
        assert torch.equal(d, down.local(x))
        with pytest.raises(ValueError):
            local_group([gate, up], x[:, :512])
        if rank == 0:
            np.savez(path, gate=gate.combine(g).numpy(), up=up.combine(u).numpy())
        else:
            gate.combine(g)
            up.combine(u)
    finally:
        dist.destroy_process_group()


def test_two_rank_local_group_matches_unsharded():
    """Column shards that share an activation through local_group, then each shard's combine()."""
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "y.npz")
        mp.spawn(_rank_group_main, args=(2, _free_port(), path), nprocs=2, join=True)
        got = dict(np.load(path))
    x = np.random.default_rng(9).standard_normal((5, 1024)).astype(np.float32)
    xq, xs = O.quantize_mxfp8(x)
    for name, n, seed in (("gate", 128, 21), ("up", 64, 22)):
        ref = O.iq3s_linear_f64(xq, xs, O.make_synthetic_iq3s(n, 1024, seed))
        np.testing.assert_array_equal(got[name], ref.astype(np.float32))


def _rank_gather_group_main(rank, world, port, path):
    from mambo_b200.sharding import gather_columns_group

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        fakes = dict(prepare=_oracle_prepare, quantize=_oracle_quantize, linear=_oracle_linear)
        # Column shards that keep their outputs sharded (gather_output=False), as in a layer whose
        # next linear is a row split; a row split that takes its K slice as input.
        gate = TensorParallelIQ3SLinear(torch.from_numpy(O.make_synthetic_iq3s(128, 1024, 31)), COLUMN,
                                        gather_output=False, out_dtype=torch.float32, **fakes)
        up = TensorParallelIQ3SLinear(torch.from_numpy(O.make_synthetic_iq3s(64, 1024, 32)), COLUMN,
                                      gather_output=False, out_dtype=torch.float32, **fakes)
        down = TensorParallelIQ3SLinear(torch.from_numpy(O.make_synthetic_iq3s(64, 1024, 33)), ROW,
                                        input_is_sharded=True, out_dtype=torch.bfloat16, **fakes)
        x = torch.from_numpy(np.random.default_rng(11).standard_normal((3, 1024)).astype(np.float32))
        g, u = gate.local(x), up.local(x)
        assert gate.combine(g).shape == (3, 64)  # kept sharded
        full_g, full_u = gather_columns_group([gate, up], [g, u])
        assert torch.equal(full_g, gate.combine(g, gather=True))
        y = down(x[:, down.k0:down.k0 + down.local_k], out_dtype=torch.float32)
        assert y.dtype == torch.float32
        if rank == 0:
            np.savez(path, gate=full_g.numpy(), up=full_u.numpy(), down=y.numpy())
    finally:
        dist.destroy_process_group()


def test_two_rank_grouped_gather_and_overrides():
    """One all-gather for several column shards; per-call gather / output-dtype overrides."""
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "y.npz")
        mp.spawn(_rank_gather_group_main, args=(2, _free_port(), path), nprocs=2, join=True)
        got = dict(np.load(path))
    x = np.random.default_rng(11).standard_normal((3, 1024)).astype(np.float32)
    xq, xs = O.quantize_mxfp8(x)
    for name, n, seed in (("gate", 128, 31), ("up", 64, 32)):
        ref = O.iq3s_linear_f64(xq, xs, O.make_synthetic_iq3s(n, 1024, seed))
        np.testing.assert_array_equal(got[name], ref.astype(np.float32))
    ref = O.iq3s_linear_f64(xq, xs, O.make_synthetic_iq3s(64, 1024, 33))
    assert O.relative_frobenius(got["down"].astype(np.float64), ref) < 1e-6
