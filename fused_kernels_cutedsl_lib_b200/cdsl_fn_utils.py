"""``compile_cutedsl`` with the reference's signature, for drop-in call sites.

The reference compiles a CuTe-DSL kernel object against sample tensors and
returns a TVM-FFI function taking torch tensors
(python/cdsl_helpers/cdsl_fn_utils.py:38-44, used as
``compiled = compile_cutedsl((a, b, c), kernel, False); compiled(a, b, c)``;
with ``include_stream=True`` the compiled function takes a trailing stream).

Here the kernels are precompiled sm_100a code. When apache-tvm-ffi is
installed and the kernel object has a TVM-FFI function with the reference's
call shape (``Gemm4SM90`` -> ``gemm(a, b, c)``, ``Swiglu2SM90`` ->
``swiglu2(a, b, b1, c)``, ``DAttn1`` -> ``dattn1(Q, K, V, O, scale)``,
``FlashSM90`` -> ``prefill_attn(mQ, mK, mV, mO, scale)``), the result IS that
``tvm_ffi.Function`` (without a stream argument), exactly as the reference
returns one; it runs on the TVM-FFI environment stream, torch's current stream.
With ``include_stream=True`` a trailing stream argument is accepted and the
call runs on that stream. Kernel objects without such a function (the
RMSNorm / LoRA / DAttn2 kernels, whose reference call shapes carry no
workspace or add keyword arguments) get a callable that forwards to the
kernel object.
"""
from __future__ import annotations

import torch

from . import _native

_TVM_NAMES = {"Gemm4SM90": "gemm", "Swiglu2SM90": "swiglu2", "DAttn1": "dattn1", "FlashSM90": "prefill_attn"}


def _tvm_function(kernel):
    name = _TVM_NAMES.get(type(kernel).__name__)
    if name is None:
        return None
    try:
        import tvm_ffi  # noqa: F401

        from . import tvm_ffi_module
    except ImportError:
        return None
    return getattr(tvm_ffi_module.load(), name)


def _as_torch_stream(stream, device):
    if isinstance(stream, torch.cuda.Stream):
        return stream
    handle = int(getattr(stream, "cuda_stream", None) or int(stream))  # cuda-python CUstream / int handle
    return torch.cuda.ExternalStream(handle, device=device)


def compile_cutedsl(tensors, kernel, include_stream: bool = True):
    """Return the compiled form of ``kernel`` for the sample ``tensors``: a
    ``tvm_ffi.Function`` where one exists with the reference's call shape, else a
    callable ``f(*tensors[, stream])`` over the kernel object."""
    _native.load()  # fail loudly here, not at the first call, if the library is missing
    dev = None
    for t in tensors:
        if isinstance(t, torch.Tensor):
            if t.device.type != "cuda":
                raise ValueError("compile_cutedsl: sample tensors must be CUDA tensors")
            dev = t.device
    fn = _tvm_function(kernel)
    if fn is not None and not include_stream:
        return fn
    if fn is not None:
        def compiled_tvm(*args):
            *rest, stream = args
            with torch.cuda.stream(_as_torch_stream(stream, dev)):
                return fn(*rest)

        compiled_tvm.kernel = kernel
        compiled_tvm.tvm_function = fn
        return compiled_tvm

    def compiled(*args):
        if include_stream and args and not isinstance(args[-1], (torch.Tensor, float, int)):
            *rest, stream = args
            return kernel(*rest, stream=stream)
        return kernel(*args)

    compiled.kernel = kernel
    return compiled
