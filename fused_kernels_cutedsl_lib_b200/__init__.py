"""B200-native (sm_100a) decode-step kernels with the reference's torch-tensor entry points.

Host code is Python/PyTorch over the C ABI of ``_lib/libfk_b200.so``
(``include/fk_b200.h``); the kernels are hand-written CUDA for sm_100a. There is
no CPU or eager fallback: if the library is missing, calls raise.
"""
from .cdsl_fn_utils import compile_cutedsl
from .gemm import (
    Gemm4SM90,
    LoraGemmSM90,
    RMSNormLinear1SM90,
    Swiglu2SM90,
    SwigluSM90,
    alloc_workspace,
    linear,
    lora_linear,
    rmsnorm_linear,
    skinny_gemm,
    swiglu_gemm,
    swiglu_gemm2,
    workspace_bytes,
)
from .prefill_attention import FlashSM90, flash_attention
from .decoding_attention import (
    DAttn1,
    DAttn2,
    DecodeAttention,
    alloc_counters,
    alloc_partials,
    chunk_tokens,
    dec_attn_combine,
    dec_attn_splitkv_fwd,
    dec_attn_splitkv_partial,
    decode_attention,
    default_num_splits,
    fused_partial_slots,
    plan_attention,
)

__all__ = [
    "Gemm4SM90",
    "LoraGemmSM90",
    "RMSNormLinear1SM90",
    "Swiglu2SM90",
    "SwigluSM90",
    "alloc_workspace",
    "compile_cutedsl",
    "linear",
    "lora_linear",
    "rmsnorm_linear",
    "skinny_gemm",
    "swiglu_gemm",
    "swiglu_gemm2",
    "workspace_bytes",
    "FlashSM90",
    "flash_attention",
    "DAttn1",
    "DAttn2",
    "DecodeAttention",
    "alloc_counters",
    "alloc_partials",
    "chunk_tokens",
    "dec_attn_combine",
    "dec_attn_splitkv_fwd",
    "dec_attn_splitkv_partial",
    "decode_attention",
    "default_num_splits",
    "fused_partial_slots",
    "plan_attention",
]
