"""CPU: host-side logic of the operator API (validation, configs, tuning registry)."""

from __future__ import annotations

import json

import pytest

from mambo_b200.kernels import iq3_s_fp8, quantize_fp8
from mambo_b200.utils import iq3_s_weight, kernel_benchmark


def test_reference_constants():
    assert iq3_s_fp8.IQ3_S_BLOCK_BYTES == 110
    assert iq3_s_fp8.IQ3_S_BLOCK_VALUES == 256
    assert iq3_s_fp8.IQ3_S_SCALE_VALUES == 32
    assert iq3_s_fp8.LARGE_TOKEN_THRESHOLD == 32
    assert set(iq3_s_fp8.BEST_CONFIGS["sm100"]) == {"medium", "large"}
    assert set(quantize_fp8.BEST_CONFIGS["sm100"]) == {"medium", "large"}


def test_codebook_tables_match_oracle():
    from oracle import iq3s_oracle as O

    assert (iq3_s_fp8.iq3_s_table() == O.iq3s_grid_u32()).all()
    assert (iq3_s_fp8.iq3_s_fp8_table() == O.iq3s_fp8_table()).all()


def test_unprepared_weight_is_a_type_error():
    with pytest.raises(TypeError):
        iq3_s_weight._weight_dimensions(object())


def test_power_of_two_checks():
    with pytest.raises(ValueError):
        iq3_s_fp8._power_of_two(3, "tile_n")
    with pytest.raises(ValueError):
        quantize_fp8._power_of_two(0, "tile_m")
    iq3_s_fp8._power_of_two(4, "tile_n")


def test_search_space_enumerates_library_configs():
    space = iq3_s_fp8.config_search_space()
    assert len(space) > 4
    assert all({"warps", "stages", "split"} <= set(c) for c in space)


def test_tuned_config_registry_roundtrip(tmp_path):
    cfg = {"kernel": 1, "warps": 4, "stages": 3, "ctas_per_sm": 1, "split": 0}
    path = tmp_path / "tuned.json"
    path.write_text(json.dumps([{"m": 4, "n": 4096, "k": 4096, "config": cfg}]))
    assert iq3_s_fp8.load_tuned_configs(path) == 1
    assert iq3_s_fp8._TUNED[(8, 4096, 4096)] == cfg
    iq3_s_fp8._TUNED.clear()


def test_benchmark_case_fields_match_reference():
    fields = set(kernel_benchmark.BenchmarkCase.__dataclass_fields__)
    assert {"name", "stream", "kernel", "search_space", "grid_fn", "args_fn", "hints_fn", "summary_keys",
            "before_launch_fn"} <= fields


def test_install_as_mambo_aliases_modules():
    import sys

    import mambo_b200

    mambo_b200.install_as_mambo()
    import mambo.kernels.iq3_s_fp8 as alias  # noqa: F401

    assert sys.modules["mambo.kernels.iq3_s_fp8"] is iq3_s_fp8


def test_m_buckets_keep_gemv_and_gemm_apart():
    b = iq3_s_fp8._m_bucket
    assert [b(m) for m in (1, 8, 9, 16, 17, 31)] == [8, 8, 16, 16, 31, 31]
    assert [b(m) for m in (32, 33, 64, 512, 513, 8192)] == [32, 64, 64, 512, 1024, 8192]


def test_gemm_search_spaces():
    from mambo_b200 import _lib

    f16 = iq3_s_fp8.config_search_space(_lib.MAMBO_KERNEL_GEMM_F16)
    assert {(c["stages"], c["split"]) for c in f16} == {(s, k) for s in (2, 3, 4) for k in (1, 2, 3, 4, 6, 8)}
    pair = iq3_s_fp8.config_search_space(_lib.MAMBO_KERNEL_GEMM_F16_PAIR)
    assert {c["stages"] for c in pair} == {2, 3, 4} and all(c["split"] == 0 for c in pair)
    gemv = iq3_s_fp8.config_search_space(_lib.MAMBO_KERNEL_GEMV)
    assert {c["split"] for c in gemv} == {0, 1, 2}


def _default(m, n, k):
    import ctypes

    from mambo_b200 import _lib

    c = _lib.MamboLinearConfig()
    _lib.check(_lib.load().mambo_default_config(m, n, k // 256, ctypes.byref(c)))
    return c.to_dict()


def test_default_gemm_k_split_follows_the_tile_count():
    """No GPU: the default for a 148-SM device. Few output tiles (Llama-3-70B O at 64 tokens:
    64 tiles) split K; many tiles (8B gate at 2048 tokens) do not; decode stays on the GEMV."""
    from mambo_b200 import _lib

    o70 = _default(64, 8192, 8192)
    assert o70["kernel"] == _lib.MAMBO_KERNEL_GEMM_F16 and o70["split"] == 2
    down70 = _default(64, 8192, 28672)
    assert down70["split"] == 2
    assert _default(2048, 14336, 4096)["split"] == 1
    assert _default(8, 4096, 4096)["kernel"] == _lib.MAMBO_KERNEL_GEMV
