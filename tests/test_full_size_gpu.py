"""Full-size parity of the benchmarked workloads against the float64 oracle.

* The decode sweep exactly as bench.py times it: the 20
  Llama-3-8B linears at M in {1, 2, 4, 8}, bf16 activations, in ONE grouped
  launch (mambo_iq3s_linear_group), and the same linears one launch each.
  Every output is compared with the C float64 oracle (IQ3_S decode restated
  from gguf-py, MXFP8 quantization restated from the reference, float64
  product: the reference's own test oracle, test_iq3_s_fp8.py:192-198).
* Prefill at M = 8192 (BASELINE config 3's largest M, 1 % outlier columns
  x50): every token against a float64 product on the GPU, and one token of
  every 128-token tile against the C oracle directly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, group_linear_into, launch_dequant_iq3_s, \
    launch_iq3_s_fp8_matmul
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields
from oracle import c_oracle as C
from oracle import iq3s_oracle as O

pytestmark = pytest.mark.gpu

ORACLE_FROB_TOL = 1e-4  # FP32 accumulation against the float64 product of the same MXFP8 operands
NORTH_STAR_TOL = 1e-3   # relative Frobenius bound of the north star
PROJECTIONS = (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate", 14336, 4096), ("up", 14336, 4096),
               ("down", 4096, 14336))
M_SWEEP = (1, 2, 4, 8)


@pytest.fixture(scope="module")
def sweep(cuda_device):
    """Weights, bf16 activations and the float64 oracle output of every linear of the sweep."""
    cases = []
    for li, m in enumerate(M_SWEEP):
        for pi, (name, n, k) in enumerate(PROJECTIONS):
            raw = O.make_synthetic_iq3s(n, k, seed=0x1A3 + 7919 * li + pi)
            x = np.random.default_rng(1000 * m + pi).standard_normal((m, k)).astype(np.float32)
            xb = torch.from_numpy(x).to(torch.bfloat16)
            xq, xs = C.quantize_mxfp8(xb.float().numpy())  # round to nearest even, as the fused path
            ref = C.iq3s_linear_f64(xq, xs, raw)
            cases.append({"m": m, "name": name, "n": n, "k": k, "ref": ref, "x": xb.to(cuda_device),
                          "w": prepare_iq3_s_fields(torch.from_numpy(raw).to(cuda_device))})
    return cases


def test_grouped_decode_sweep_matches_oracle(cuda_device, sweep):
    outs = [torch.full((c["m"], c["n"]), float("nan"), dtype=torch.float32, device=cuda_device) for c in sweep]
    group_linear_into([c["x"] for c in sweep], [c["w"] for c in sweep], outs)
    torch.cuda.synchronize(cuda_device)
    for c, out in zip(sweep, outs):
        got = out.cpu().numpy().astype(np.float64)
        err = O.relative_frobenius(got, c["ref"])
        assert np.isfinite(got).all(), f"M={c['m']} {c['name']}: unwritten outputs"
        assert err < ORACLE_FROB_TOL, f"M={c['m']} {c['name']}: {err}"


def test_grouped_decode_sweep_bf16_outputs(cuda_device, sweep):
    """The bench's own output type: bf16 rounding on top of the FP32 result."""
    outs = [torch.empty((c["m"], c["n"]), dtype=torch.bfloat16, device=cuda_device) for c in sweep]
    group_linear_into([c["x"] for c in sweep], [c["w"] for c in sweep], outs)
    torch.cuda.synchronize(cuda_device)
    for c, out in zip(sweep, outs):
        err = O.relative_frobenius(out.float().cpu().numpy(), c["ref"])
        assert err < 4e-3, f"M={c['m']} {c['name']}: {err}"


@pytest.mark.parametrize("m", M_SWEEP)
def test_single_launch_decode_matches_oracle(cuda_device, sweep, m):
    """One fused launch per linear (the reference's call shape), each M's quantizer path included."""
    for c in (c for c in sweep if c["m"] == m):
        out = torch.full((m, c["n"]), float("nan"), dtype=torch.float32, device=cuda_device)
        fused_linear_into(c["x"], c["w"], out)
        torch.cuda.synchronize(cuda_device)
        err = O.relative_frobenius(out.cpu().numpy(), c["ref"])
        assert err < ORACLE_FROB_TOL, f"M={m} {c['name']}: {err}"


LLAMA3_8B_PREFILL = {"qkv": (6144, 4096), "o": (4096, 4096), "gate_up": (14336, 4096), "down": (4096, 14336)}


@pytest.mark.parametrize("proj", sorted(LLAMA3_8B_PREFILL))
def test_prefill_m8192_matches_oracle(cuda_device, proj):
    n, k = LLAMA3_8B_PREFILL[proj]
    m = 8192
    raw_np = O.make_synthetic_iq3s(n, k, seed=8192 + n + k)
    fields = prepare_iq3_s_fields(torch.from_numpy(raw_np).to(cuda_device))
    gen = torch.Generator(device=cuda_device).manual_seed(8192 + n)
    x = torch.randn((m, k), device=cuda_device, generator=gen)
    cols = torch.randperm(k, device=cuda_device, generator=gen)[: round(0.01 * k)]
    x[:, cols] *= 50.0
    xq, xs = launch_quantize_fp8(x.to(torch.bfloat16))
    out = launch_iq3_s_fp8_matmul(xq, xs, fields)
    torch.cuda.synchronize(cuda_device)
    # One token of every 128-token tile, each at a different row of its tile, against the C oracle.
    toks = np.array([128 * t + (37 * t) % 128 for t in range(m // 128)])
    ref_s = C.iq3s_linear_f64(xq[toks].cpu().numpy(), xs[toks].cpu().numpy(), raw_np)
    got_s = out[torch.from_numpy(toks).to(cuda_device)].cpu().numpy().astype(np.float64)
    err_s = O.relative_frobenius(got_s, ref_s)
    assert err_s < ORACLE_FROB_TOL, err_s
    # Every token against a float64 product of the dequantized operands.
    bits, scales = launch_dequant_iq3_s(fields)
    lut = torch.from_numpy(O.decode_e4m3(np.arange(256, dtype=np.uint8))).to(cuda_device)
    w = (lut[bits.long()] * scales.repeat_interleave(32, dim=1)).double()
    del bits, scales
    xe = lut[xq.long()].double() * torch.exp2(xs.double() - 127).repeat_interleave(32, dim=1)
    ref = xe @ w.t()
    del xe, w
    err = (torch.linalg.norm(out.double() - ref) / torch.linalg.norm(ref)).item()
    assert err < ORACLE_FROB_TOL, err
