"""Device plumbing shared by the operators: tensors, streams, device checks, workspaces.

PyTorch provides device memory and streams; the compute is in libmambo_b200.
"""

from __future__ import annotations

import threading

import torch

from . import _lib

_checked_devices: dict[int, int] = {}
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_ws_lock = threading.Lock()


def as_cuda_tensor(obj) -> torch.Tensor:
    """Zero-copy view of a CUDA array (torch, DLPack or __cuda_array_interface__ object)."""
    if isinstance(obj, torch.Tensor):
        t = obj
    elif hasattr(obj, "__dlpack__"):
        t = torch.from_dlpack(obj)
    elif hasattr(obj, "__cuda_array_interface__"):
        t = torch.as_tensor(obj, device="cuda")
    else:
        raise TypeError(f"expected a CUDA tensor, got {type(obj).__name__}")
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor (this build has no CPU path)")
    return t


def stream_handle(stream, device: torch.device) -> int:
    """cudaStream_t of `stream` (None = torch's current stream on `device`)."""
    if stream is None:
        return torch.cuda.current_stream(device).cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    if isinstance(stream, int):
        return stream
    for attr in ("cuda_stream", "ptr", "handle"):
        if hasattr(stream, attr):
            return int(getattr(stream, attr))
    raise TypeError(f"unsupported stream object {type(stream).__name__}")


def require_device(device: torch.device) -> None:
    """Raise RuntimeError unless `device` is an sm_100 GPU this library runs on."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    status = _checked_devices.get(index)
    if status is None:
        lib = _lib.load()
        with torch.cuda.device(index):
            status = lib.mambo_device_check()
        _checked_devices[index] = status
    if status != _lib.MAMBO_OK:
        major, minor = torch.cuda.get_device_capability(index)
        raise RuntimeError(f"IQ3_S FP8 kernels have no build for sm{major}{minor} (this library targets sm_100a)")


def workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Zero-filled scratch for split-K partials and counters, one per (device, stream).

    The kernels leave the counter region zeroed again, so the buffer is reused
    across calls on the same stream; calls on different streams get their own.
    """
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            size = max(nbytes, 1 << 20)
            if ws is not None:
                size = max(size, 2 * ws.numel())
            dev = torch.device("cuda", index)
            # Drain pending work before swapping buffers: a kernel on `stream`
            # may still use the old one, and the zero-fill runs on torch's stream.
            torch.cuda.synchronize(dev)
            ws = torch.zeros(size, dtype=torch.uint8, device=dev)
            torch.cuda.synchronize(dev)
            _workspaces[key] = ws
        return ws
