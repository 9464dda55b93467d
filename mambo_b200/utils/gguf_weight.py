"""Real GGUF weights into the linear path: a named 2-D tensor in its packed
block layout, and from there the prepared IQ3_S fields on the device.

Follows the reference's test helper ``read_model_weight``
(tests/python/utils/gguf_weight.py:16-48), which reads tensor descriptors with
its own GGUF parser (src/python/mambo/utils/gguf_manifest.py:435-563). Here the
descriptors come from gguf-py's ``GGUFReader`` (the GGUF format's own Python
package), which memory-maps the file: no weight bytes are copied until the
caller moves them to the GPU.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np


def read_model_weight(model_path: str | Path, weight_name: str, *,
                      expected_type: str | None = None) -> tuple[np.ndarray, int, int]:
    """Packed bytes ``uint8 [N, K/block_elements, block_bytes]`` of a 2-D GGUF tensor, N and K.

    The array is a read-only view of the memory-mapped file. Errors as the
    reference helper raises them: ``KeyError`` for a missing name,
    ``AssertionError`` for another tensor type than ``expected_type`` (a type
    name such as ``"iq3_s"``, any case), ``ValueError`` for a tensor that is not
    2-D or whose byte count does not match whole blocks.
    """
    from gguf import GGML_QUANT_SIZES, GGUFReader

    reader = GGUFReader(str(model_path))
    tensor = next((t for t in reader.tensors if t.name == weight_name), None)
    if tensor is None:
        raise KeyError(f"GGUF has no tensor named {weight_name!r}")
    type_name = tensor.tensor_type.name.lower()
    if expected_type is not None and type_name != expected_type.lower():
        raise AssertionError(f"{weight_name} must use {expected_type}, got {type_name}")
    if len(tensor.shape) != 2:
        raise ValueError(f"{weight_name} must be a two-dimensional weight")
    k, n = (int(v) for v in tensor.shape)  # GGUF lists the fastest-varying dimension first
    block_elements, block_bytes = GGML_QUANT_SIZES[tensor.tensor_type]
    data = np.asarray(tensor.data)
    n_bytes = data.size * data.itemsize
    if k % block_elements or n_bytes != n * (k // block_elements) * block_bytes:
        raise ValueError(f"{weight_name} has an inconsistent GGUF block layout")
    payload = data.reshape(-1).view(np.uint8).reshape(n, k // block_elements, block_bytes)
    return payload, n, k


def load_iq3_s_fields(model_path: str | Path, weight_name: str, device="cuda"):
    """A GGUF IQ3_S weight prepared for ``launch_iq3_s_fp8_matmul`` (``IQ3SFields`` on ``device``)."""
    import torch

    from .iq3_s_weight import prepare_iq3_s_fields

    raw, _, _ = read_model_weight(model_path, weight_name, expected_type="iq3_s")
    return prepare_iq3_s_fields(torch.from_numpy(np.ascontiguousarray(raw)).to(device))
