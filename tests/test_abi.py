"""CPU: the C-ABI library loads and exports every symbol include/mambo_b200.h declares (no compute)."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import ROOT
from mambo_b200 import _lib

HEADER = ROOT / "include" / "mambo_b200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"MAMBO_API\s+[\w\s\*]+?\b(mambo_\w+)\s*\(", text))


def test_header_declares_the_binding_table():
    assert declared_symbols() == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [name for name in sorted(declared_symbols()) if not hasattr(lib, name)]
    assert not missing, missing


def test_version_and_configs_without_gpu():
    lib = _lib.load()
    assert b"sm_100a" in lib.mambo_version()
    n = lib.mambo_num_configs(_lib.MAMBO_KERNEL_GEMV)
    assert n > 0
    seen = set()
    for i in range(n):
        c = _lib.MamboLinearConfig()
        assert lib.mambo_config_at(_lib.MAMBO_KERNEL_GEMV, i, c) == _lib.MAMBO_OK
        seen.add(tuple(c.to_dict().items()))
    assert len(seen) == n
    c = _lib.MamboLinearConfig()
    assert lib.mambo_config_at(_lib.MAMBO_KERNEL_GEMV, n, c) == _lib.MAMBO_EINVAL
    assert lib.mambo_default_config(8, 4096, 16, c) == _lib.MAMBO_OK and c.warps > 0


def test_argument_errors_are_reported_not_raised():
    lib = _lib.load()
    # null pointers and bad shapes are rejected before any device work
    st = lib.mambo_quantize_mxfp8(None, _lib.MAMBO_F32, 4, 64, 64, None, 64, None, 2, 0, None)
    assert st == _lib.MAMBO_EINVAL
    assert "null" in _lib.last_error()
    w = _lib.MamboIQ3SWeight()
    st = lib.mambo_iq3s_linear(None, 0, None, 0, 1, w, None, None, 0, 0, None, None, 0, None)
    assert st == _lib.MAMBO_EINVAL
    with pytest.raises(ValueError):
        _lib.check(st)


def test_workspace_size_is_positive_and_monotone():
    lib = _lib.load()
    small = lib.mambo_iq3s_linear_workspace_bytes(8, 4096, 16, None)
    big = lib.mambo_iq3s_linear_workspace_bytes(8, 28672, 112, None)
    assert 0 < small <= big


def test_grouped_entry_points_check_arguments_without_gpu():
    """The grouped IQ3_S and Q4_K calls reject bad groups before any device work."""
    lib = _lib.load()
    items = (_lib.MamboQ4KItem * 2)()
    for i, (m, n, b) in enumerate(((1, 4096, 16), (8, 14336, 16))):
        items[i].m, items[i].n_rows, items[i].n_blocks = m, n, b
        items[i].x_dtype, items[i].ldx = _lib.MAMBO_BF16, b * 256
        items[i].out_dtype, items[i].ldo = _lib.MAMBO_BF16, n
    assert lib.mambo_q4k_linear_group(None, 1, None, 0, None) == _lib.MAMBO_EINVAL
    assert lib.mambo_q4k_linear_group(items, 0, None, 0, None) == _lib.MAMBO_EINVAL
    assert lib.mambo_q4k_linear_group(items, 2, None, 0, None) == _lib.MAMBO_EINVAL
    assert "item 0: null pointer" in _lib.last_error()
    # Workspace: zero for an empty group, and a group needs at least what its largest item does.
    assert lib.mambo_q4k_linear_group_workspace_bytes(None, 0) == 0
    one = lib.mambo_q4k_linear_group_workspace_bytes(items, 1)
    two = lib.mambo_q4k_linear_group_workspace_bytes(items, 2)
    assert 0 < one <= two
    assert two >= lib.mambo_q4k_linear_fused_workspace_bytes(8, 14336, 16, None)
    linears = (_lib.MamboLinearItem * 1)()
    assert lib.mambo_iq3s_linear_group(None, 1, None, None, 0, None) == _lib.MAMBO_EINVAL
    assert lib.mambo_iq3s_linear_group(linears, 1, None, None, 0, None) == _lib.MAMBO_EINVAL
    assert "null" in _lib.last_error()
