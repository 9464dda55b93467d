"""Tensor-parallel IQ3_S x MXFP8 linears on 2 B200s over NCCL: sharded == unsharded.

Skipped on a box with fewer than two GPUs. Each rank runs the single-GPU
kernels on its shard; rank 0 also runs the unsharded linear and compares.
"""

from __future__ import annotations

import datetime
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

SHAPES = {"column": (6144, 4096), "row": (4096, 14336)}  # Llama-3-8B QKV (column) and down (row)


def _rank_main(rank, world, port, mode, m, path):
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    try:
        from mambo_b200.kernels.iq3_s_fp8 import iq3_s_fp8_linear
        from mambo_b200.sharding import TensorParallelIQ3SLinear
        from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

        dev = torch.device("cuda", rank)
        n, k = SHAPES[mode]
        gen = torch.Generator(device=dev).manual_seed(2024)  # same weights and input on every rank
        raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
        raw[..., :2] = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half() \
            .view(torch.uint8).view(n, k // 256, 2)
        x = torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16)
        lin = TensorParallelIQ3SLinear(raw, mode, out_dtype=torch.float32)
        y = lin(x)
        torch.cuda.synchronize()
        if rank == 0:
            full = iq3_s_fp8_linear(x, prepare_iq3_s_fields(raw), out_dtype=torch.float32)
            err = (torch.linalg.norm((y - full).double()) / torch.linalg.norm(full.double())).item()
            np.save(path, np.array([err, float(y.shape[0]), float(y.shape[1])]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["column", "row"])
@pytest.mark.parametrize("m", [8, 256])
def test_two_gpu_tensor_parallel_matches_unsharded(mode, m):
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "r.npy")
        mp.spawn(_rank_main, args=(2, _free_port(), mode, m, path), nprocs=2, join=True)
        err, rows, cols = np.load(path)
    assert (rows, cols) == (m, SHAPES[mode][0])
    assert err < 1e-5, err


def _rank_main_fused(rank, world, port, m, path):
    """Row split with the all-reduce fused into the GEMV: every rank's result against the unsharded linear,
    and the ranks' results against each other (bit-identical: every rank sums the same partials in rank order)."""
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
    comm = None
    try:
        from mambo_b200.kernels.iq3_s_fp8 import iq3_s_fp8_linear
        from mambo_b200.sharding import ROW, FusedAllReduce, TensorParallelIQ3SLinear
        from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

        dev = torch.device("cuda", rank)
        n, k = SHAPES["row"]
        gen = torch.Generator(device=dev).manual_seed(2024)
        raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
        raw[..., :2] = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half() \
            .view(torch.uint8).view(n, k // 256, 2)
        x = torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16)
        lin = TensorParallelIQ3SLinear(raw, ROW, out_dtype=torch.float32)
        comm = FusedAllReduce(n)
        outs = [lin.fused(x, comm) for _ in range(3)]  # both slot buffers, then the first again
        torch.cuda.synchronize()
        same_calls = all(torch.equal(o, outs[0]) for o in outs)
        y = outs[0]
        gathered = [torch.empty_like(y) for _ in range(world)]
        dist.all_gather(gathered, y)
        same_ranks = all(torch.equal(g, gathered[0]) for g in gathered)
        if rank == 0:
            full = iq3_s_fp8_linear(x, prepare_iq3_s_fields(raw), out_dtype=torch.float32)
            err = (torch.linalg.norm((y - full).double()) / torch.linalg.norm(full.double())).item()
            np.save(path, np.array([err, float(same_calls), float(same_ranks)]))
        dist.barrier()
    finally:
        if comm is not None:
            torch.cuda.synchronize()
            dist.barrier()  # no rank unmaps a peer's buffer while that peer may still write into it
            comm.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("m", [1, 8, 31])
def test_two_gpu_fused_allreduce_matches_unsharded(m):
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "r.npy")
        mp.spawn(_rank_main_fused, args=(2, _free_port(), m, path), nprocs=2, join=True)
        err, same_calls, same_ranks = np.load(path)
    assert same_calls == 1.0 and same_ranks == 1.0
    assert err < 1e-5, err
