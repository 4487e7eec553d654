"""Argument checks and pointer/stream extraction shared by the Python entry points.

The reference relies on trace-time ``assert``s and otherwise launches blindly
(python/cutedsl_kernels/gemm/kernel/attempt4.py:69,80-82,121,130). Here every
entry point checks dtype, device, shape and contiguity before it launches and
raises ``TypeError`` (wrong dtype / not a tensor) or ``ValueError`` (shape,
device, layout); the C ABI re-checks sizes and alignment.
"""
from __future__ import annotations

import torch

from . import _native


def require_tensor(name: str, t, dtype: torch.dtype, ndim: int | None = None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(t).__name__}")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor, got device {t.device}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous (row-major)")
    return t


def require_shape(name: str, t: torch.Tensor, shape: tuple) -> None:
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def same_device(*ts: torch.Tensor) -> torch.device:
    dev = ts[0].device
    for t in ts[1:]:
        if t.device != dev:
            raise ValueError(f"all tensors must be on one device, got {dev} and {t.device}")
    return dev


def stream_for(dev: torch.device, stream=None) -> int:
    """cudaStream_t (as int) to launch on: explicit, else torch's current stream."""
    _native.use_device(dev.index if dev.index is not None else torch.cuda.current_device())
    if stream is None:
        return torch.cuda.current_stream(dev).cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    return int(stream)


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()
