"""The TVM-FFI face of the library: ``load()`` returns a tvm_ffi Module whose
functions take torch tensors directly, as the reference's compiled kernels do
(README.md:1, python/cdsl_helpers/cdsl_fn_utils.py:38-44).

Functions: ``dec_attn_splitkv_fwd``, ``dec_attn_combine``, ``dattn1``,
``prefill_attn`` (FlashSM90's ``(mQ, mK, mV, mO, softmax_scale)``),
``dattn2`` (DAttn2's call plus ``tmp`` [3, M, H*D] and workspace),
``skinny_gemm``, ``rmsnorm_linear``, ``swiglu_gemm``, ``swiglu_gemm2``,
``lora_gemm`` (the LoRA kernel's ``(a, b, lora_xA, lora_B, c)`` plus workspace),
``linear_workspace_bytes`` (same arguments and meaning as the C ABI in
include/fk_b200.h, with tensors in place of pointer + size lists). They run
on the tensors' current stream and write caller-allocated outputs.
"""
from __future__ import annotations

from pathlib import Path

LIB = Path(__file__).resolve().parent / "_lib" / "libfk_b200_tvmffi.so"
_mod = None


def load():
    """Load libfk_b200_tvmffi.so through apache-tvm-ffi (raises if either is missing)."""
    global _mod
    if _mod is None:
        import tvm_ffi

        if not LIB.exists():
            raise ImportError(f"{LIB} is missing: run `python -m fused_kernels_cutedsl_lib_b200.build`")
        _mod = tvm_ffi.load_module(str(LIB))
    return _mod
