"""Torch-side plumbing for libdwa: pointers, streams, dtypes and workspaces.

PyTorch provides device memory and streams; all arithmetic of the hot path runs
in libdwa's kernels.  Workspaces are ordinary torch allocations cached per
(device, purpose), so the library itself never allocates.
"""

from __future__ import annotations

import ctypes as C

import torch

from . import _lib

_ACT_CODES = {torch.float32: _lib.DWA_F32, torch.bfloat16: _lib.DWA_BF16}


def dtype_code(dt: torch.dtype, what: str) -> int:
    try:
        return _ACT_CODES[dt]
    except KeyError:
        raise TypeError(f"{what}: dtype {dt} not supported (float32 or bfloat16)") from None


def ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_of(device: torch.device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def require_cuda(name: str, t: torch.Tensor, device: torch.device | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be on a CUDA device (the hot path has no CPU fallback)")
    if device is not None and t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


_workspaces: dict[tuple, torch.Tensor] = {}


def workspace(device: torch.device, purpose: str, nbytes: int) -> torch.Tensor:
    """A cached uint8 device buffer of at least ``nbytes`` for one purpose.

    Buffers are reused call after call on the current stream (stream order keeps
    reuse safe); the status word in the first bytes is zeroed when a buffer is
    first made.
    """
    key = (device.index if device.index is not None else torch.cuda.current_device(), purpose)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def workspace_status(clear: bool = True) -> dict:
    """Device status word of every cached workspace (synchronises the streams)."""
    lib = _lib.load()
    out = {}
    for key, buf in _workspaces.items():
        bits = C.c_uint32()
        with torch.cuda.device(buf.device):
            lib.dwa_workspace_status(stream_of(buf.device), ptr(buf), C.byref(bits), int(clear))
        out[key] = bits.value
    return out


def raise_on_device_status() -> None:
    bad = {k: v for k, v in workspace_status(clear=True).items() if v}
    if bad:
        msg = "; ".join(f"{k[1]}@cuda:{k[0]}: {_lib.describe_status(v)}" for k, v in bad.items())
        raise _lib.DwaError(f"device status: {msg}")
