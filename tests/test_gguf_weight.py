"""GGUF ingestion on the host: a named tensor of a GGUF file in its packed block
layout (mambo_b200.utils.gguf_weight, after the reference's test helper
read_model_weight, tests/python/utils/gguf_weight.py:16-48).

The files are written here with gguf-py's writer. The IQ3_S blocks read back
must be the bytes written, and the oracle's decode of them must equal gguf-py's
own dequantization of the same tensor in the file.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import iq3s_oracle as O
from mambo_b200.utils.gguf_weight import read_model_weight


@pytest.fixture()
def model(tmp_path, write_gguf):
    raw = O.make_synthetic_iq3s(40, 768, seed=11)
    other = O.make_synthetic_iq3s(16, 256, seed=12)
    tensors = {
        "blk.0.attn_qkv.weight": (raw.reshape(40, -1), "IQ3_S"),
        "blk.1.ffn_down.weight": (other.reshape(16, -1), "IQ3_S"),
        "blk.0.attn_norm.weight": (np.linspace(-1, 1, 24, dtype=np.float32), "F32"),
        "token_embd.weight": (np.arange(48, dtype=np.float32).reshape(6, 8), "F32"),
    }
    return write_gguf(tmp_path / "model.gguf", tensors), raw, other


def test_iq3_s_blocks_read_back_byte_exact(model):
    path, raw, other = model
    packed, n, k = read_model_weight(path, "blk.0.attn_qkv.weight", expected_type="iq3_s")
    assert (n, k) == (40, 768) and packed.shape == (40, 3, 110) and packed.dtype == np.uint8
    assert np.array_equal(packed, raw)
    packed2, n2, k2 = read_model_weight(path, "blk.1.ffn_down.weight", expected_type="IQ3_S")
    assert (n2, k2) == (16, 256) and np.array_equal(packed2, other)


def test_oracle_decode_of_loaded_blocks_equals_gguf_py(model):
    from gguf import GGMLQuantizationType, GGUFReader
    from gguf.quants import dequantize

    path, _, _ = model
    packed, n, k = read_model_weight(path, "blk.0.attn_qkv.weight", expected_type="iq3_s")
    tensor = next(t for t in GGUFReader(str(path)).tensors if t.name == "blk.0.attn_qkv.weight")
    ref = dequantize(np.asarray(tensor.data), GGMLQuantizationType.IQ3_S).reshape(n, k)
    ours = O.dequantize_iq3s(np.ascontiguousarray(packed)).reshape(n, k)
    assert np.array_equal(ours.astype(np.float32), ref.astype(np.float32))


def test_non_quantized_2d_tensor_without_a_type_check(model):
    path, _, _ = model
    packed, n, k = read_model_weight(path, "token_embd.weight")
    assert (n, k) == (6, 8) and packed.shape == (6, 8, 4)
    assert np.array_equal(packed.reshape(6, 32).view(np.float32), np.arange(48, dtype=np.float32).reshape(6, 8))


def test_errors_follow_the_reference_helper(model):
    path, _, _ = model
    with pytest.raises(KeyError):
        read_model_weight(path, "blk.9.missing.weight")
    with pytest.raises(AssertionError):
        read_model_weight(path, "token_embd.weight", expected_type="iq3_s")
    with pytest.raises(ValueError):
        read_model_weight(path, "blk.0.attn_norm.weight")
