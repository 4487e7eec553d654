"""Prefill (full-sequence) attention: host side of ``csrc/prefill_attn.cu``.

Reference boundary: ``FlashSM90(qk_mn, cluster_size_m, num_stages, ...)``
(python/cutedsl_kernels/attn/attempt6_epi_pipeline/attn.py:73-117) is built
with Hopper tuning arguments and called as ``fa(mQ, mK, mV, mO, softmax_scale,
stream)`` on caller-allocated ``[b, h, seqlen, d]`` tensors (attn.py:118-175,
tests.py:75-80), writing ``mO`` in place. The same class is provided here; its
tuning arguments are accepted and ignored (the sm_100a kernel has one tiling:
128 queries x 128 keys, S and O accumulated in TMEM).

Semantics: ``softmax(q @ k.transpose(-1, -2) * softmax_scale) @ v`` without a
mask, head_dim 64 or 128; k/v may have fewer heads than q (grouped-query: q
head ``h`` reads kv head ``h // (Hq // Hkv)``), an extension of the reference's
equal-head layout.
"""
from __future__ import annotations

import math

import torch

from . import _native
from ._tensors import ptr, require_tensor, same_device, stream_for


def flash_attention(q, k, v, out=None, *, softmax_scale=None, lse=None, return_lse=False, stream=None):
    """``out = softmax(q k^T * scale) v`` for q [B, Hq, Lq, D], k/v [B, Hkv, Lkv, D] bf16.

    ``softmax_scale`` defaults to ``D ** -0.5``. With ``return_lse`` (or an
    ``lse`` tensor [B, Hq, Lq] fp32) the natural-log logsumexp of the scaled
    scores is written too. Returns ``out`` (and ``lse``).
    """
    require_tensor("q", q, torch.bfloat16, 4)
    require_tensor("k", k, torch.bfloat16, 4)
    require_tensor("v", v, torch.bfloat16, 4)
    B, Hq, Lq, D = q.shape
    if k.shape != v.shape:
        raise ValueError(f"k and v must have the same shape, got {tuple(k.shape)} and {tuple(v.shape)}")
    if k.shape[0] != B or k.shape[3] != D:
        raise ValueError(f"k/v must be [B={B}, Hkv, Lkv, D={D}], got {tuple(k.shape)}")
    Hkv, Lkv = k.shape[1], k.shape[2]
    if Hq % Hkv:
        raise ValueError(f"num_heads_q={Hq} must be a multiple of num_heads_kv={Hkv}")
    if D not in (64, 128):
        raise ValueError(f"head_dim must be 64 or 128, got {D}")
    if out is None:
        out = torch.empty_like(q)
    require_tensor("out", out, torch.bfloat16, 4)
    if tuple(out.shape) != tuple(q.shape):
        raise ValueError(f"out must have shape {tuple(q.shape)}, got {tuple(out.shape)}")
    if lse is None and return_lse:
        lse = torch.empty(B, Hq, Lq, dtype=torch.float32, device=q.device)
    if lse is not None:
        require_tensor("lse", lse, torch.float32, 3)
        if tuple(lse.shape) != (B, Hq, Lq):
            raise ValueError(f"lse must have shape {(B, Hq, Lq)}, got {tuple(lse.shape)}")
    same_device(*[t for t in (q, k, v, out, lse) if t is not None])
    scale = D ** -0.5 if softmax_scale is None else float(softmax_scale)
    if not (scale > 0 and math.isfinite(scale)):
        raise ValueError(f"softmax_scale must be positive and finite, got {softmax_scale}")
    st = stream_for(q.device, stream)
    _native.check(_native.load().fk_prefill_attn_fwd(
        ptr(q), ptr(k), ptr(v), ptr(out), ptr(lse) if lse is not None else None, B, Hq, Hkv, Lq, Lkv, D, scale,
        st))
    return (out, lse) if (return_lse or lse is not None) else out


class FlashSM90:
    """``FlashSM90(qk_mn, ...)(mQ, mK, mV, mO, softmax_scale, stream)`` (attn.py:73-175)."""

    def __init__(self, qk_mn=(128, 128), cluster_size_m=1, num_stages=2, intra_wg_overlap=False, pingpong=False,
                 mma_m_size=64, epi_n=32, epi_stages=2):
        self.tuning = dict(qk_mn=qk_mn, cluster_size_m=cluster_size_m, num_stages=num_stages,
                           intra_wg_overlap=intra_wg_overlap, pingpong=pingpong, mma_m_size=mma_m_size,
                           epi_n=epi_n, epi_stages=epi_stages)

    def __call__(self, mQ, mK, mV, mO, softmax_scale, stream=None):
        flash_attention(mQ, mK, mV, mO, softmax_scale=softmax_scale, stream=stream)
