"""The device-timed autotuner on B200 (mini_benchmark over make_benchmark_cases).

The reference tunes its cuTile kernels with an exhaustive search per case
(src/python/mambo/utils/kernel_benchmark.py:41-100, cases from
src/python/mambo/kernels/iq3_s_fp8.py:402-465). Here the search runs over the
library's configuration spaces (GEMV below 32 tokens; FP16 GEMM stages x K
split and CTA pairs from 32), records each case's winner for its (M, N, K),
and later launches of that shape use it.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from mambo_b200.kernels import iq3_s_fp8
from mambo_b200.kernels.iq3_s_fp8 import launch_iq3_s_fp8_matmul, make_benchmark_cases, select_config
from mambo_b200.utils.kernel_benchmark import mini_benchmark
from oracle import iq3s_oracle as O

pytestmark = pytest.mark.gpu

ORACLE_FROB_TOL = 1e-4


def test_autotuner_records_winners_that_match_the_oracle(cuda_device, tmp_path):
    n, k = 512, 2048
    raw = O.make_synthetic_iq3s(n, k, seed=2024)
    weight = torch.from_numpy(raw).to(cuda_device)
    saved = dict(iq3_s_fp8._TUNED)
    try:
        cases = make_benchmark_cases(weight, ms=(4, 64))
        assert cases[0].search_space[0] == select_config(4, n, k, cuda_device, tuned=False)
        path = tmp_path / "tuned.json"
        results = mini_benchmark(cases, warmup=2, iters=4, quiet=True, save_path=path)
        assert all(r["passed"] >= 1 for r in results), results
        records = json.loads(path.read_text())
        assert {(r["m"], r["n"], r["k"]) for r in records} == {(4, n, k), (64, n, k)}
        for rec in records:
            m = rec["m"]
            assert select_config(m, n, k, cuda_device) == rec["config"]  # later launches use the winner
            xq, xs = O.quantize_mxfp8(np.random.default_rng(m).standard_normal((m, k)).astype(np.float32))
            out = launch_iq3_s_fp8_matmul(torch.from_numpy(xq).to(cuda_device), torch.from_numpy(xs).to(cuda_device),
                                          iq3_s_fp8.prepare_iq3_s_fields(weight))
            err = O.relative_frobenius(out.cpu().numpy(), O.iq3s_linear_f64(xq, xs, raw))
            assert err < ORACLE_FROB_TOL, (m, rec["config"], err)
    finally:
        iq3_s_fp8._TUNED.clear()
        iq3_s_fp8._TUNED.update(saved)


def test_packaged_tuned_configs_are_valid(cuda_device):
    """Every record of the committed tuning file names a kernel of its M's class and a configuration
    that is one of the library's search-space entries (or the untuned default)."""
    from mambo_b200 import _lib

    if not iq3_s_fp8.TUNED_CONFIGS_PATH.is_file():
        pytest.skip("no packaged tuning file")
    spaces = {kind: iq3_s_fp8.config_search_space(kind) for kind in
              (_lib.MAMBO_KERNEL_GEMV, _lib.MAMBO_KERNEL_GEMM_F16, _lib.MAMBO_KERNEL_GEMM_F16_PAIR)}
    for rec in json.loads(iq3_s_fp8.TUNED_CONFIGS_PATH.read_text()):
        cfg, m = rec["config"], rec["m"]
        default = select_config(m, rec["n"], rec["k"], cuda_device, tuned=False)
        if cfg == default:
            continue
        large = m >= iq3_s_fp8.LARGE_TOKEN_THRESHOLD
        assert (cfg["kernel"] != _lib.MAMBO_KERNEL_GEMV) == large, rec
        assert cfg in spaces[cfg["kernel"]], rec
