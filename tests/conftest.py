"""pytest configuration: the `gpu` marker and shared fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU and libmambo_b200.so")


@pytest.fixture(scope="session")
def golden():
    """The committed golden vectors (see tests/golden/make_golden.py)."""
    return {name: dict(np.load(GOLDEN / f"golden_{name}.npz")) for name in ("iq3s_decode", "mxfp8", "linear")}


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"GPU tests need an sm_100 device, found sm{major}{minor}")
    return torch.device("cuda", 0)


@pytest.fixture(scope="session")
def write_gguf():
    """Writes a GGUF v3 file with gguf-py's writer: ``write_gguf(path, {name: (array, type)})``.

    ``type`` is a ``gguf.GGMLQuantizationType`` name ("IQ3_S", "F32", ...). A
    quantized tensor is given as its packed bytes ``uint8 [rows, row_bytes]``.
    """
    def write(path, tensors):
        from gguf import GGMLQuantizationType, GGUFWriter

        writer = GGUFWriter(str(path), "llama")
        for name, (array, type_name) in tensors.items():
            qtype = GGMLQuantizationType[type_name]
            if qtype in (GGMLQuantizationType.F32, GGMLQuantizationType.F16):
                writer.add_tensor(name, array)
            else:
                writer.add_tensor(name, array, raw_dtype=qtype)
        writer.write_header_to_file()
        writer.write_kv_data_to_file()
        writer.write_tensors_to_file()
        writer.close()
        return path

    return write
