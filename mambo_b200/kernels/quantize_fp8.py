"""Block-scaled FP8 (MXFP8) activation quantization on sm_100a.

Mirror of src/python/mambo/kernels/quantize_fp8.py (Menooker/Mambo): same
entry point, arguments, outputs and errors. Outputs E4M3 value bytes and one
UE8M0 scale byte per 32 values along K:

    e = clamp(ceil(log2(amax / 448)), -127, 127)   (amax == 0 -> e = 0)
    q = E4M3(x * 2^-e),  scale byte = e + 127

The exponent is computed exactly from the bits of amax. Values round to
nearest-even like the reference kernel's cast; ``rounding="ties_down"``
resolves exact ties toward the smaller magnitude like the reference's NumPy
test oracle (the two differ only on exact ties, which bf16 inputs hit often).
Also accepts bf16 activations (converted to f32 exactly).
"""

from __future__ import annotations

import torch

from .. import _lib, _runtime

# Launch shape of the sm_100a kernel: each warp quantizes 8 groups of 32
# (4 lanes per group, 128-bit loads); tile options of the reference are
# accepted and validated but the grid is sized by the library.
BEST_CONFIGS = {
    "sm100": {
        "medium": {"tile_m": 4, "tile_k_groups": 4},
        "large": {"tile_m": 16, "tile_k_groups": 16},
    },
}
LARGE_TOKEN_THRESHOLD = 32

_ROUNDING = {"nearest_even": _lib.MAMBO_ROUND_NEAREST_EVEN, "ties_down": _lib.MAMBO_ROUND_TIES_DOWN}


def _power_of_two(value: int, name: str) -> None:
    if value < 1 or value & (value - 1):
        raise ValueError(f"{name} must be a positive power of two")


def _activation_config(m: int, device: torch.device) -> dict:
    major, minor = torch.cuda.get_device_capability(device)
    sm = f"sm{major}{minor}"
    if sm not in BEST_CONFIGS:
        raise RuntimeError(f"FP8 activation quantizer has no tuned config for {sm}")
    return BEST_CONFIGS[sm]["large" if m >= LARGE_TOKEN_THRESHOLD else "medium"]


def launch_quantize_fp8(x, *, tile_m: int | None = None, tile_k_groups: int | None = None, stream=None,
                        rounding: str = "nearest_even", out=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Return [M,K] E4M3 bytes and [M,K/32] E8M0 scale bytes (quantize_fp8.py:67-84).

    ``out``: optional preallocated (values uint8 [M,K], scales uint8 [M,K/32]).
    """
    x = _runtime.as_cuda_tensor(x)
    if x.ndim != 2 or x.dtype not in (torch.float32, torch.bfloat16) or x.shape[1] % 32:
        raise ValueError("activation must be float32 [M,K] with K divisible by 32")
    if rounding not in _ROUNDING:
        raise ValueError(f"rounding must be one of {sorted(_ROUNDING)}")
    m, k = x.shape
    if m < 1 or k < 32:
        raise ValueError("activation must be float32 [M,K] with K divisible by 32")
    if tile_m is None or tile_k_groups is None:
        config = _activation_config(m, x.device)
        tile_m = config["tile_m"] if tile_m is None else tile_m
        tile_k_groups = config["tile_k_groups"] if tile_k_groups is None else tile_k_groups
    _power_of_two(tile_m, "tile_m")
    _power_of_two(tile_k_groups, "tile_k_groups")
    _runtime.require_device(x.device)
    if x.stride(1) != 1:
        x = x.contiguous()
    if out is None:
        values = torch.empty((m, k), dtype=torch.uint8, device=x.device)
        scales = torch.empty((m, k // 32), dtype=torch.uint8, device=x.device)
    else:
        values, scales = out
        if values.shape != (m, k) or scales.shape != (m, k // 32) or values.dtype != torch.uint8 \
                or scales.dtype != torch.uint8 or values.stride(1) != 1 or scales.stride(1) != 1:
            raise ValueError("out must be (uint8 [M,K], uint8 [M,K/32]) with unit column stride")
    dtype = _lib.MAMBO_BF16 if x.dtype == torch.bfloat16 else _lib.MAMBO_F32
    with torch.cuda.device(x.device):
        st = _runtime.stream_handle(stream, x.device)
        _lib.check(
            _lib.load().mambo_quantize_mxfp8(
                x.data_ptr(), dtype, m, k, x.stride(0), values.data_ptr(), values.stride(0),
                scales.data_ptr(), scales.stride(0), _ROUNDING[rounding], st,
            ),
            "launch_quantize_fp8",
        )
    return values, scales
