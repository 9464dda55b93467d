"""Weights prepared with soa=False keep only the tile-major packed copy (plus d and scales).

Every linear reads the packed records, so its results must be bit-identical to
those of the same weight with its SoA fields kept; the paths that read the SoA
fields (the standalone decoder, the legacy mma.sync kernel) refuse such a
weight instead of reading null pointers.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import iq3s_oracle as O
from mambo_b200 import _lib
from mambo_b200.kernels.iq3_s_fp8 import (config_search_space, iq3_s_fp8_linear, iq3_s_fp8_linear_group,
                                          launch_dequant_iq3_s, launch_iq3_s_fp8_matmul)
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from mambo_b200.utils.iq3_s_weight import fields_nbytes, has_soa_fields, prepare_iq3_s_fields

pytestmark = pytest.mark.gpu


def _pair(dev, n, k, seed):
    raw = torch.from_numpy(O.make_synthetic_iq3s(n, k, seed)).to(dev)
    return prepare_iq3_s_fields(raw), prepare_iq3_s_fields(raw, soa=False)


def _x(dev, m, k, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn((m, k), generator=g).to(torch.bfloat16).to(dev)


def test_packed_only_frees_the_soa_fields(cuda_device):
    full, lean = _pair(cuda_device, 1024, 2048, 11)
    assert has_soa_fields(full) and not has_soa_fields(lean)
    assert fields_nbytes(lean) * 18 < fields_nbytes(full)  # 6 of 110 bytes per block kept
    assert torch.equal(lean.packed, full.packed)


@pytest.mark.parametrize("m", [1, 4, 13, 64, 300])
def test_linears_on_packed_only_weights_are_bit_identical(cuda_device, m):
    full, lean = _pair(cuda_device, 1024, 2048, 20 + m)
    x = _x(cuda_device, m, 2048, 30 + m)
    assert torch.equal(iq3_s_fp8_linear(x, lean, out_dtype=torch.float32),
                       iq3_s_fp8_linear(x, full, out_dtype=torch.float32))
    xq, xs = launch_quantize_fp8(x)
    assert torch.equal(launch_iq3_s_fp8_matmul(xq, xs, lean), launch_iq3_s_fp8_matmul(xq, xs, full))
    if m >= 32:
        wide = {"kernel": _lib.MAMBO_KERNEL_GEMM_F16_WIDE, "warps": 8, "stages": 4}
        assert torch.equal(launch_iq3_s_fp8_matmul(xq, xs, lean, config=wide),
                           launch_iq3_s_fp8_matmul(xq, xs, full, config=wide))


def test_grouped_launch_on_packed_only_weights(cuda_device):
    pairs = [_pair(cuda_device, n, k, 40 + i) for i, (n, k) in enumerate([(512, 1024), (1024, 2048), (256, 512)])]
    xs = [_x(cuda_device, m, k, 50 + i) for i, (m, k) in enumerate([(2, 1024), (5, 2048), (1, 512)])]
    a = iq3_s_fp8_linear_group(xs, [p[1] for p in pairs], out_dtype=torch.float32)
    b = iq3_s_fp8_linear_group(xs, [p[0] for p in pairs], out_dtype=torch.float32)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


def test_soa_readers_refuse_packed_only_weights(cuda_device):
    _, lean = _pair(cuda_device, 256, 512, 60)
    with pytest.raises(ValueError):
        launch_dequant_iq3_s(lean)
    xq, xs = launch_quantize_fp8(_x(cuda_device, 4, 512, 61))
    sync = config_search_space(_lib.MAMBO_KERNEL_GEMV_SYNC)[0]
    launch_iq3_s_fp8_matmul(xq, xs, prepare_iq3_s_fields(torch.from_numpy(O.make_synthetic_iq3s(256, 512, 60))
                                                         .to(cuda_device)), config=sync)  # the config itself is valid
    with pytest.raises(ValueError, match="SoA"):
        launch_iq3_s_fp8_matmul(xq, xs, lean, config=sync)
    with pytest.raises(ValueError):
        prepare_iq3_s_fields(torch.from_numpy(O.make_synthetic_iq3s(12, 512, 62)).to(cuda_device), soa=False)
