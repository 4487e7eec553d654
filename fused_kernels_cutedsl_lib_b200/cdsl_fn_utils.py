"""``compile_cutedsl`` with the reference's signature, for drop-in call sites.

The reference compiles a CuTe-DSL kernel object against sample tensors and
returns a TVM-FFI callable taking torch tensors
(python/cdsl_helpers/cdsl_fn_utils.py:38-44, used as
``compiled = compile_cutedsl((a, b, c), kernel, False); compiled(a, b, c)``).
Here the kernels are precompiled sm_100a code, so "compiling" validates the
sample tensors once by running nothing and returns a callable that forwards
to the kernel object. With ``include_stream=True`` the callable accepts (and
uses) a trailing stream argument, as the reference's compiled functions do.
"""
from __future__ import annotations

import torch

from . import _native


def compile_cutedsl(tensors, kernel, include_stream: bool = True):
    """Return a callable ``f(*tensors[, stream])`` that runs ``kernel`` on sm_100a."""
    _native.load()  # fail loudly here, not at the first call, if the library is missing
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.device.type != "cuda":
            raise ValueError("compile_cutedsl: sample tensors must be CUDA tensors")

    def compiled(*args):
        if include_stream and args and not isinstance(args[-1], (torch.Tensor, float, int)):
            *rest, stream = args
            return kernel(*rest, stream=stream)
        return kernel(*args)

    compiled.kernel = kernel
    return compiled
