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
