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
