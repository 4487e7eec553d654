"""Linear-family entry points (host side of ``csrc/skinny_gemm.cu`` / ``csrc/gemm_tc.cu``).

Reference boundary: the reference's GEMM kernels are objects built with
tuning arguments and called on caller-allocated tensors, returning ``None``:

* ``Gemm4SM90(tile_shape_mnk, ...)(a, b, c)`` — ``c = a @ b.t()``
  (python/cutedsl_kernels/gemm/kernel/attempt4.py:57-68,133-168; demo/gemm_run.py:29-41)
* ``RMSNormLinear1SM90(..., eps)(a, b, c, stream)`` — ``c = rms_norm(a) @ b.t()``
  (python/cutedsl_kernels/rmsnorm_linear/attempt1/gemm.py:52-65,136-170)
* ``Swiglu2SM90(...)(a, b, b1, c)`` — ``c = silu(a @ b.t()) * (a @ b1.t())``
  (python/cutedsl_kernels/swiglu/attempt1/gemm2.py:69-81,145-187)
* ``GemmSM90(...)(a, b, lora_xA, lora_B, c, stream)`` of the LoRA kernel —
  ``c = a @ b.t() + lora_xA @ lora_B.t()``
  (python/cutedsl_kernels/lora/attempt1/gemm.py:57-178; check :672-675)

The same class names are provided here. Their Hopper tuning arguments (tile
shapes, cluster shapes, stage counts) are accepted and ignored: the B200
kernels pick their own tiling from M. Functional forms (``skinny_gemm``,
``rmsnorm_linear``, ``swiglu_gemm``, ``linear``) take an explicit ``out``.

The stream-K kernels need a small fp32 workspace whose counters start at
zero; :func:`workspace_for` keeps one zero-initialised buffer per device and
grows it on demand. Calls on one stream may share it; calls that may overlap
on the GPU (different streams) need ``workspace=`` buffers of their own.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import _native
from ._tensors import ptr, require_tensor, same_device, stream_for

FLAG_SWIGLU = 1
_ws_lock = threading.Lock()
_ws: dict[str, torch.Tensor] = {}


def workspace_bytes(M: int, N: int, K: int, swiglu: bool = False) -> int:
    """Bytes of stream-K workspace a call with these sizes needs (on the current device)."""
    out = ctypes.c_size_t(0)
    _native.check(_native.load().fk_linear_workspace_bytes(int(M), int(N), int(K),
                                                           FLAG_SWIGLU if swiglu else 0, ctypes.byref(out)))
    return int(out.value)


def alloc_workspace(nbytes: int, device) -> torch.Tensor:
    """A zero-filled, 256-byte aligned workspace of at least ``nbytes`` bytes."""
    return torch.zeros(max(256, (nbytes + 255) // 256 * 256), dtype=torch.uint8, device=device)


def workspace_for(nbytes: int, device: torch.device) -> torch.Tensor:
    """Per-device shared workspace (zero-initialised, grown on demand)."""
    key = str(device)
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = alloc_workspace(max(nbytes, 1 << 20), device)
            _ws[key] = buf
        return buf


def _check_x_w(x, w, name_w="w"):
    require_tensor("x", x, torch.bfloat16, 2)
    require_tensor(name_w, w, torch.bfloat16, 2)
    if x.shape[1] != w.shape[1]:
        raise ValueError(f"x is [M, K={x.shape[1]}] but {name_w} is [N, K={w.shape[1]}]")
    if x.shape[1] % 8 != 0:
        raise ValueError(f"K={x.shape[1]} must be a multiple of 8")


def _check_out(out, M, N, name="out"):
    require_tensor(name, out, torch.bfloat16, 2)
    if tuple(out.shape) != (M, N):
        raise ValueError(f"{name} must have shape {(M, N)}, got {tuple(out.shape)}")


def linear(x, w, out=None, *, gamma=None, eps: float = 1e-6, w_up=None, up_row_offset: int = 0,
           residual=None, workspace=None, stream=None):
    """General fused linear: ``out = [residual +] epi(rms_norm?(x) @ w.t())``.

    ``gamma`` fuses RMSNorm (with ``eps``); ``w_up`` selects SwiGLU with up rows
    at ``w_up[up_row_offset + n]``; ``residual`` is added last. Returns ``out``.
    """
    _check_x_w(x, w)
    M, K = x.shape
    N = out.shape[1] if out is not None else (w.shape[0] - up_row_offset if (w_up is not None and w_up is w)
                                               else w.shape[0])
    if w_up is not None:
        require_tensor("w_up", w_up, torch.bfloat16, 2)
        if w_up.shape[1] != K or w_up.shape[0] < up_row_offset + N:
            raise ValueError(f"w_up must be [>= {up_row_offset + N}, {K}], got {tuple(w_up.shape)}")
    if w_up is not w and w.shape[0] != N:
        raise ValueError(f"w must have N={N} rows, got {w.shape[0]}")
    dev = x.device
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _check_out(out, M, N)
    if gamma is not None:
        require_tensor("gamma", gamma, torch.bfloat16, 1)
        if gamma.shape[0] != K:
            raise ValueError(f"gamma must be [{K}], got {tuple(gamma.shape)}")
    if residual is not None:
        _check_out(residual, M, N, "residual")
    same_device(*[t for t in (x, w, w_up, gamma, residual, out) if t is not None])
    st = stream_for(dev, stream)
    need = workspace_bytes(M, N, K, w_up is not None)
    ws = workspace if workspace is not None else workspace_for(need, dev)
    if ws.numel() * ws.element_size() < need:
        raise ValueError(f"workspace holds {ws.numel() * ws.element_size()} bytes, needs {need}")
    _native.check(_native.load().fk_linear(
        ptr(x), ptr(gamma) if gamma is not None else None, ptr(w), ptr(w_up) if w_up is not None else None,
        int(up_row_offset), ptr(residual) if residual is not None else None, ptr(out), M, N, K, float(eps),
        ptr(ws), ws.numel() * ws.element_size(), st))
    return out


def skinny_gemm(x, w, out=None, *, residual=None, workspace=None, stream=None):
    """``out = x @ w.t()`` (+ ``residual``)."""
    return linear(x, w, out, residual=residual, workspace=workspace, stream=stream)


def rmsnorm_linear(x, gamma, w, out=None, *, eps: float = 1e-6, residual=None, workspace=None, stream=None):
    """``out = rms_norm(x, gamma, eps) @ w.t()`` with the normalisation fused into the GEMM."""
    if gamma is None:
        raise ValueError("gamma is required (use ones for the reference's gain-free RMSNorm)")
    return linear(x, w, out, gamma=gamma, eps=eps, residual=residual, workspace=workspace, stream=stream)


def swiglu_gemm(x, w_gate_up, out=None, *, gamma=None, eps: float = 1e-6, workspace=None, stream=None):
    """``out = silu(x @ Wg.t()) * (x @ Wu.t())`` for ``w_gate_up = cat([Wg, Wu])`` of shape [2N, K]."""
    require_tensor("w_gate_up", w_gate_up, torch.bfloat16, 2)
    if w_gate_up.shape[0] % 2:
        raise ValueError("w_gate_up must have an even number of rows [2N, K]")
    n = w_gate_up.shape[0] // 2
    if out is None:
        out = torch.empty((x.shape[0], n), dtype=torch.bfloat16, device=x.device)
    return linear(x, w_gate_up, out, gamma=gamma, eps=eps, w_up=w_gate_up, up_row_offset=n,
                  workspace=workspace, stream=stream)


def swiglu_gemm2(x, w_gate, w_up, out=None, *, workspace=None, stream=None):
    """``out = silu(x @ w_gate.t()) * (x @ w_up.t())`` with two separate weights."""
    require_tensor("w_up", w_up, torch.bfloat16, 2)
    if tuple(w_up.shape) != tuple(w_gate.shape):
        raise ValueError("w_gate and w_up must have the same shape")
    return linear(x, w_gate, out, w_up=w_up, up_row_offset=0, workspace=workspace, stream=stream)


def lora_linear(x, w, lora_b, out=None, *, lora_a=None, lora_xa=None, residual=None, workspace=None,
                stream=None):
    """``out = x @ w.t() + (x @ lora_a.t()) @ lora_b.t()`` (+ ``residual``).

    Give either ``lora_a`` [rank, K] (``x @ lora_a.t()`` is then computed with
    :func:`linear`, as the reference computes its ``lora_xA`` operand before the
    call, lora/attempt1/gemm.py:700-704) or the precomputed ``lora_xa`` [M, rank].
    The low-rank product is accumulated in the same fp32 accumulator as the main
    product (extra k blocks of one GEMM) and rounded once.
    """
    _check_x_w(x, w)
    M, K = x.shape
    N = w.shape[0]
    require_tensor("lora_b", lora_b, torch.bfloat16, 2)
    if lora_b.shape[0] != N:
        raise ValueError(f"lora_b must be [N={N}, rank], got {tuple(lora_b.shape)}")
    r = lora_b.shape[1]
    if r < 8 or r % 8:
        raise ValueError(f"LoRA rank must be a positive multiple of 8, got {r}")
    if (lora_a is None) == (lora_xa is None):
        raise ValueError("give exactly one of lora_a and lora_xa")
    if lora_xa is None:
        require_tensor("lora_a", lora_a, torch.bfloat16, 2)
        if tuple(lora_a.shape) != (r, K):
            raise ValueError(f"lora_a must be [{r}, {K}], got {tuple(lora_a.shape)}")
        lora_xa = linear(x, lora_a, workspace=workspace, stream=stream)
    require_tensor("lora_xa", lora_xa, torch.bfloat16, 2)
    if tuple(lora_xa.shape) != (M, r):
        raise ValueError(f"lora_xa must be [{M}, {r}], got {tuple(lora_xa.shape)}")
    dev = x.device
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    _check_out(out, M, N)
    if residual is not None:
        _check_out(residual, M, N, "residual")
    same_device(*[t for t in (x, w, lora_b, lora_xa, residual, out) if t is not None])
    st = stream_for(dev, stream)
    need = workspace_bytes(M, N, K)
    ws = workspace if workspace is not None else workspace_for(need, dev)
    if ws.numel() * ws.element_size() < need:
        raise ValueError(f"workspace holds {ws.numel() * ws.element_size()} bytes, needs {need}")
    _native.check(_native.load().fk_lora_linear(
        ptr(x), ptr(w), ptr(lora_xa), ptr(lora_b), ptr(residual) if residual is not None else None, ptr(out),
        M, N, K, r, ptr(ws), ws.numel() * ws.element_size(), st))
    return out


_ones_cache: dict = {}


def _ones(k: int, device) -> torch.Tensor:
    key = (k, str(device))
    t = _ones_cache.get(key)
    if t is None:
        t = torch.ones(k, dtype=torch.bfloat16, device=device)
        _ones_cache[key] = t
    return t


class Gemm4SM90:
    """``Gemm4SM90(**tuning)(a, b, c)``: ``c = a @ b.t()`` (tuning arguments accepted, unused)."""

    def __init__(self, *args, **kwargs):
        self.tuning = (args, kwargs)

    def __call__(self, a, b, c, stream=None):
        skinny_gemm(a, b, c, stream=stream)


class RMSNormLinear1SM90:
    """``RMSNormLinear1SM90(..., eps)(a, b, c, stream)``: ``c = rms_norm(a, eps) @ b.t()``.

    As in the reference the norm has no gain unless ``gamma`` is given to the call.
    """

    def __init__(self, *args, eps: float = 1e-5, **kwargs):
        self.eps = eps
        self.tuning = (args, kwargs)

    def __call__(self, a, b, c, stream=None, gamma=None):
        g = gamma if gamma is not None else _ones(a.shape[1], a.device)
        rmsnorm_linear(a, g, b, c, eps=self.eps, stream=stream)


class Swiglu2SM90:
    """``Swiglu2SM90(**tuning)(a, b, b1, c)``: ``c = silu(a @ b.t()) * (a @ b1.t())``."""

    def __init__(self, *args, **kwargs):
        self.tuning = (args, kwargs)

    def __call__(self, a, b, b1, c, stream=None):
        swiglu_gemm2(a, b, b1, c, stream=stream)


SwigluSM90 = Swiglu2SM90


class LoraGemmSM90:
    """LoRA ``GemmSM90(**tuning)(a, b, lora_xA, lora_B, c, stream)``:
    ``c = a @ b.t() + lora_xA @ lora_B.t()`` (lora/attempt1/gemm.py:57-178;
    tuning arguments accepted, unused)."""

    def __init__(self, *args, **kwargs):
        self.tuning = (args, kwargs)

    def __call__(self, a, b, lora_xA, lora_B, c, stream=None):
        lora_linear(a, b, lora_B, c, lora_xa=lora_xA, stream=stream)
