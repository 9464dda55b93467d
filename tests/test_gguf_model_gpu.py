"""GPU parity on GGUF weights read from a file: GGUF tensor -> prepared fields
-> launch_quantize_fp8 -> launch_iq3_s_fp8_matmul.

After the reference's test_model_projection_matches_f32_and_fp8_references
(tests/python/test_iq3_s_fp8.py:213-269). Its two comparisons are kept:
  * against the float64 product of the ORIGINAL f32 activations and gguf-py's
    dequantized weight: NMSE < 1e-3 (the FP8 activation-quantization bound);
  * against the float64 product of the MXFP8-reconstructed activations: the
    IQ3_S decode and tensor-core arithmetic alone, rtol 5e-4, atol 5e-3.
The reference's third reference, ggml's CUDA matmul, needs the ggml tool that
its pinned llama.cpp submodule builds; it is not part of this build.

A real model is used when one is named: MAMBO_GGUF_MODEL (path), or
tests/config.json's "qwen_gguf_path" as in the reference, with the tensor
MAMBO_GGUF_WEIGHT (default blk.1.attn_qkv.weight, the reference's). Without
one, that case is skipped; the same checks always run on a GGUF file written
here with synthetic IQ3_S weights.
"""

from __future__ import annotations

import json
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import iq3s_oracle as O
from mambo_b200.kernels.iq3_s_fp8 import launch_iq3_s_fp8_matmul
from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
from mambo_b200.utils.gguf_weight import load_iq3_s_fields, read_model_weight

pytestmark = pytest.mark.gpu

WEIGHT_NAME = os.environ.get("MAMBO_GGUF_WEIGHT", "blk.1.attn_qkv.weight")
MS = [1, 4, 8, 128]


def _named_model() -> Path | None:
    value = os.environ.get("MAMBO_GGUF_MODEL")
    if not value:
        config = Path(__file__).resolve().parent / "config.json"
        if config.is_file():
            value = json.loads(config.read_text(encoding="utf-8")).get("qwen_gguf_path")
    if not value:
        return None
    path = Path(value).expanduser()
    if not path.is_file():
        raise FileNotFoundError(f"GGUF model not found: {path}")
    return path


def _gguf_py_weight(path: Path, name: str) -> np.ndarray:
    """gguf-py's own dequantization of the tensor, float64 [N, K]."""
    from gguf import GGMLQuantizationType, GGUFReader
    from gguf.quants import dequantize

    tensor = next(t for t in GGUFReader(str(path)).tensors if t.name == name)
    k, n = (int(v) for v in tensor.shape)
    return dequantize(np.asarray(tensor.data), GGMLQuantizationType.IQ3_S).reshape(n, k).astype(np.float64)


def _check_projection(path: Path, name: str, m: int, cuda_device, *, reference_allclose: bool) -> None:
    raw, n_rows, k = read_model_weight(path, name, expected_type="iq3_s")
    assert raw.shape[2] == 110
    weight = load_iq3_s_fields(path, name, device=cuda_device)
    gen = torch.Generator(device="cpu").manual_seed(20261017)
    x = torch.randn((m, k), generator=gen, dtype=torch.float32)
    xq, xs = launch_quantize_fp8(x.to(cuda_device))
    out = launch_iq3_s_fp8_matmul(xq, xs, weight).cpu().numpy()
    assert out.shape == (m, n_rows)

    w = _gguf_py_weight(path, name)
    original = x.numpy().astype(np.float64) @ w.T
    nmse = float(np.sum((out - original) ** 2) / np.sum(original ** 2))
    assert nmse < 1e-3, (m, nmse)
    if reference_allclose:  # the reference's tolerance, set on its real model weight
        np.testing.assert_allclose(out, original, rtol=0.05, atol=0.18)

    effective_x = O.decode_mxfp8(xq.cpu().numpy(), xs.cpu().numpy()).astype(np.float64)
    np.testing.assert_allclose(out, effective_x @ w.T, rtol=5e-4, atol=5e-3)


@pytest.mark.parametrize("m", MS)
def test_synthetic_gguf_projection(tmp_path, write_gguf, cuda_device, m):
    raw = O.make_synthetic_iq3s(1024, 2048, seed=77)
    path = write_gguf(tmp_path / "synthetic.gguf", {WEIGHT_NAME: (raw.reshape(1024, -1), "IQ3_S")})
    _check_projection(path, WEIGHT_NAME, m, cuda_device, reference_allclose=False)


@pytest.mark.parametrize("m", MS)
def test_model_projection_matches_f32_and_fp8_references(cuda_device, m):
    path = _named_model()
    if path is None:
        pytest.skip("name a GGUF model with MAMBO_GGUF_MODEL (or tests/config.json qwen_gguf_path)")
    _check_projection(path, WEIGHT_NAME, m, cuda_device, reference_allclose=True)
