"""The C ABI from C++ without Python: tests/cpp/c_abi_runner.cpp, built here
against include/mambo_b200.h and linked to libmambo_b200.so (the role of the
reference's C++ loader test, tests/cpp/loadtest/loadtest.cpp:201-412).

CPU: the program compiles and links against the header and the library.
GPU: it runs the prepare / pack / quantize / linear / fused / grouped path and
checks each result against the C oracle itself (exit status 0).
"""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT
from mambo_b200 import _lib

SOURCE = ROOT / "tests" / "cpp" / "c_abi_runner.cpp"
ORACLE_LIB = ROOT / "oracle" / "_build" / "liboracle_iq3s.so"
CUDA = Path("/usr/local/cuda")


def _build(out_dir: Path) -> Path:
    if shutil.which("g++") is None:
        pytest.skip("g++ is not installed")
    if not ORACLE_LIB.is_file():
        subprocess.run(["make", "-C", str(ROOT / "oracle")], check=True, capture_output=True)
    exe = out_dir / "c_abi_runner"
    lib_dir = _lib.LIB_PATH.parent
    cmd = ["g++", "-O2", "-std=c++17", "-Wall", "-Wextra", f"-I{ROOT / 'include'}", f"-I{CUDA / 'include'}",
           str(SOURCE), "-o", str(exe),
           f"-L{lib_dir}", "-lmambo_b200", f"-Wl,-rpath,{lib_dir}",
           f"-L{ORACLE_LIB.parent}", "-loracle_iq3s", f"-Wl,-rpath,{ORACLE_LIB.parent}",
           f"-L{CUDA / 'lib64'}", "-lcudart", f"-Wl,-rpath,{CUDA / 'lib64'}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr[-4000:]
    return exe


def test_runner_builds_against_the_header_and_library(tmp_path):
    exe = _build(tmp_path)
    assert exe.is_file()


@pytest.mark.gpu
def test_runner_passes_on_the_gpu(tmp_path, cuda_device):
    from oracle import iq3s_oracle as O

    exe = _build(tmp_path)
    grid, table = tmp_path / "grid.bin", tmp_path / "fp8_table.bin"
    O.iq3s_grid_u32().astype("<u4").tofile(grid)
    np.asarray(O.iq3s_fp8_table(), dtype="<u4").tofile(table)
    res = subprocess.run([str(exe), str(grid), str(table)], capture_output=True, text=True, timeout=240)
    print(res.stdout)
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-4000:]
    assert "PASSED" in res.stdout and "FAIL " not in res.stdout
