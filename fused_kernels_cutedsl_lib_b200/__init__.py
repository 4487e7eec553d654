"""B200-native (sm_100a) decode-step kernels with the reference's torch-tensor entry points.

Host code is Python/PyTorch over the C ABI of ``_lib/libfk_b200.so``
(``include/fk_b200.h``); the kernels are hand-written CUDA for sm_100a. There is
no CPU or eager fallback: if the library is missing, calls raise.
"""
from .decoding_attention import (
    DecodeAttention,
    alloc_partials,
    chunk_tokens,
    dec_attn_combine,
    dec_attn_splitkv_fwd,
    dec_attn_splitkv_partial,
    decode_attention,
    default_num_splits,
)

__all__ = [
    "DecodeAttention",
    "alloc_partials",
    "chunk_tokens",
    "dec_attn_combine",
    "dec_attn_splitkv_fwd",
    "dec_attn_splitkv_partial",
    "decode_attention",
    "default_num_splits",
]
