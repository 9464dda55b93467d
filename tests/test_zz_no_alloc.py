"""mambo_iq3s_linear_noalloc (library-held static scratch) against mambo_iq3s_linear.

The entry point serves callers that cannot allocate device memory; it must give
the workspace entry point's results, call after call, with the split-K scratch
in the library's static device array. Collected last so that it also runs after
every other GPU test in the same process; it needs nothing from them.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from mambo_b200 import _lib
from oracle import iq3s_oracle as O
from mambo_b200.kernels.iq3_s_fp8 import _get_iq3_table, launch_iq3_s_fp8_matmul
from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields, weight_struct

pytestmark = pytest.mark.gpu

# The linear tests' bound against the float64 oracle (relative Frobenius).
FROB_TOL = 1e-4


def _noalloc(lib, xq, xs, fields, table, out, cfg=None):
    w = weight_struct(fields)
    out_dtype = _lib.MAMBO_BF16 if out.dtype == torch.bfloat16 else _lib.MAMBO_F32
    return lib.mambo_iq3s_linear_noalloc(
        xq.data_ptr(), xq.stride(0), xs.data_ptr(), xs.stride(0), xq.shape[0], ctypes.byref(w), table.data_ptr(),
        out.data_ptr(), out_dtype, out.stride(0), cfg, torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("m,n,k", [(8, 1024, 4096), (13, 520, 768), (1, 4096, 14336)])
def test_noalloc_matches_workspace_entry_twice(cuda_device, m, n, k):
    lib = _lib.load()
    raw = O.make_synthetic_iq3s(n, k, 4242 + m)
    rng = np.random.default_rng(m + n)
    xq_np, xs_np = O.quantize_mxfp8(rng.standard_normal((m, k)).astype(np.float32))
    fields = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))
    xq, xs = torch.from_numpy(xq_np).to(cuda_device), torch.from_numpy(xs_np).to(cuda_device)
    table = _get_iq3_table(cuda_device)
    oracle = O.iq3s_linear_f64(xq_np, xs_np, raw)

    expected = launch_iq3_s_fp8_matmul(xq, xs, fields).cpu().numpy().astype(np.float64)
    assert O.relative_frobenius(expected, oracle) < FROB_TOL
    for call in range(2):
        out = torch.full((m, n), float("nan"), dtype=torch.float32, device=cuda_device)
        _lib.check(_noalloc(lib, xq, xs, fields, table, out), "mambo_iq3s_linear_noalloc")
        torch.cuda.synchronize(cuda_device)
        got = out.cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all(), f"call {call}: unwritten outputs"
        assert O.relative_frobenius(got, expected) < FROB_TOL, f"call {call}"
        assert O.relative_frobenius(got, oracle) < FROB_TOL, f"call {call} against the float64 oracle"
        np.testing.assert_allclose(got, expected, rtol=5e-4, atol=5e-4 * np.abs(expected).max())
    assert _lib.device_status()[0] == _lib.MAMBO_OK


def test_noalloc_unaligned_rows_bf16_output(cuda_device):
    """Activation rows that are not 16-byte aligned go through the copies into the
    static scratch; bf16 output rows are written chunk by chunk (8 + 5 tokens)."""
    lib = _lib.load()
    m, n, k = 13, 1032, 1024
    raw = O.make_synthetic_iq3s(n, k, 777)
    xq_np, xs_np = O.quantize_mxfp8(np.random.default_rng(5).standard_normal((m, k)).astype(np.float32))
    fields = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))
    # Row strides k + 8 and k/32 + 3 bytes: rows 1.. start off a 16-byte boundary.
    xq_big = torch.zeros((m, k + 8), dtype=torch.uint8, device=cuda_device)
    xs_big = torch.zeros((m, k // 32 + 3), dtype=torch.uint8, device=cuda_device)
    xq_big[:, :k] = torch.from_numpy(xq_np).to(cuda_device)
    xs_big[:, : k // 32] = torch.from_numpy(xs_np).to(cuda_device)
    xq, xs = xq_big[:, :k], xs_big[:, : k // 32]
    assert xq.stride(0) % 16 and xs.stride(0) % 16
    oracle = O.iq3s_linear_f64(xq_np, xs_np, raw)
    table = _get_iq3_table(cuda_device)
    for call in range(2):
        out_big = torch.full((m, n + 8), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        out = out_big[:, :n]
        _lib.check(_noalloc(lib, xq, xs, fields, table, out), "mambo_iq3s_linear_noalloc")
        torch.cuda.synchronize(cuda_device)
        got = out.float().cpu().numpy().astype(np.float64)
        assert np.isfinite(got).all(), f"call {call}: unwritten outputs"
        assert torch.isnan(out_big[:, n:]).all(), f"call {call}: wrote past the row"
        # bf16 output: rounding of 2^-9 relative per element
        assert O.relative_frobenius(got, oracle) < 4e-3, f"call {call}"
        np.testing.assert_allclose(got, oracle, rtol=8e-3, atol=8e-3 * np.abs(oracle).max())
    assert _lib.device_status()[0] == _lib.MAMBO_OK


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_device):
    lib = _lib.load()
    n, blocks = 8, 385  # K = 98560 > 98304, the largest K the static scratch holds
    raw = np.zeros((n, blocks, 110), dtype=np.uint8)
    fields = prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))
    xq = torch.zeros((1, blocks * 256), dtype=torch.uint8, device=cuda_device)
    xs = torch.zeros((1, blocks * 8), dtype=torch.uint8, device=cuda_device)
    out = torch.zeros((1, n), dtype=torch.float32, device=cuda_device)
    status = _noalloc(lib, xq, xs, fields, _get_iq3_table(cuda_device), out)
    assert status == _lib.MAMBO_EINVAL
    assert "K <= 98304" in _lib.last_error()
