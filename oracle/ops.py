"""fp32 CPU restatements of the reference's torch check paths — TEST INFRASTRUCTURE.

Each function cites the reference file:line whose torch formula it restates
(paths relative to the reference project root). Inputs may be bf16; every
function upcasts to fp32 (the reference's own check paths compare bf16 kernel
outputs against fp32 torch). Nothing here is on the product path.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _cpu32(t: torch.Tensor) -> torch.Tensor:
    return t.detach().to("cpu", torch.float32)


def decode_attention(q, k_cache, v_cache, cache_seqlens, softmax_scale=None):
    """Softmax decode attention with GQA over each row's first ``cache_seqlens[b]`` keys.

    Restates ``attn_reimpl`` (python/cutedsl_kernels/attn/attempt6_epi_pipeline/attn.py:778-784:
    ``p = exp2(q k^T * scale*log2e - max)``, ``pv * 1/sum``) and the SDPA check of
    attn/attempt6_epi_pipeline/tests.py:85, extended with what the decode path
    needs and the reference kernels leave implicit: query head h reads kv head
    ``h // (Hq // Hkv)``; keys past ``cache_seqlens[b]`` are masked; the LSE is the
    natural-log ``logsumexp(q k^T * scale)``; a row with no keys gives out = 0 and
    lse = -inf (the zero-row-sum guard of attn/attempt6_epi_pipeline/my_softmax.py:88-97).

    q: [B, 1, Hq, D] or [B, Hq, D]; k_cache/v_cache: [B, Lmax, Hkv, D].
    Returns (out [B, Hq, D] fp32, lse [B, Hq] fp32). Loops per row so an 8 GB
    padded cache is never upcast whole.
    """
    qf = _cpu32(q).reshape(q.shape[0], -1, q.shape[-1])
    B, Hq, D = qf.shape
    Lmax, Hkv = k_cache.shape[1], k_cache.shape[2]
    G = Hq // Hkv
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    lens = cache_seqlens.detach().to("cpu", torch.int64).clamp(0, Lmax)
    out = torch.zeros(B, Hq, D)
    lse = torch.full((B, Hq), float("-inf"))
    for b in range(B):
        L = int(lens[b])
        if L == 0:
            continue
        kb = _cpu32(k_cache[b, :L]).permute(1, 0, 2)  # [Hkv, L, D]
        vb = _cpu32(v_cache[b, :L]).permute(1, 0, 2)
        qb = qf[b].view(Hkv, G, D)
        s = torch.matmul(qb, kb.transpose(1, 2)) * scale  # [Hkv, G, L]
        lse[b] = torch.logsumexp(s, dim=-1).reshape(Hq)
        p = torch.softmax(s, dim=-1)
        out[b] = torch.matmul(p, vb).reshape(Hq, D)
    return out, lse


def prefill_attention(q, k, v, softmax_scale=None):
    """Full-sequence attention in fp32, the reference's ``attn_reimpl``
    (attn/attempt6_epi_pipeline/attn.py:778-784: ``p = q k^T * scale * log2 e``,
    ``exp2(p - rowmax)``, ``(p v) / rowsum``), with grouped kv heads
    (q head h reads kv head h // (Hq // Hkv)). Returns (out, lse) with the
    natural-log logsumexp of the scaled scores. q [B, Hq, Lq, D], k/v [B, Hkv, Lkv, D].
    """
    qf, kf, vf = _cpu32(q), _cpu32(k), _cpu32(v)
    B, Hq, Lq, D = qf.shape
    g = Hq // kf.shape[1]
    kf = kf.repeat_interleave(g, dim=1)
    vf = vf.repeat_interleave(g, dim=1)
    scale = D ** -0.5 if softmax_scale is None else float(softmax_scale)
    s = (qf @ kf.transpose(2, 3)) * scale
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp2((s - s.amax(dim=-1, keepdim=True)) * math.log2(math.e))
    out = (p @ vf) / p.sum(dim=-1, keepdim=True)
    return out, lse


def dattn1_reference(Q, K, V):
    """The reference decode kernel's own check: ``(Q @ K^T) @ Vt`` with V given transposed.

    demo/dec_attn_second_part.py:27-35 (Q [H,M,D], K [H,P,D], V [H,D,P],
    ``Vt = V.transpose(1, 2)``); no softmax and no scale, as in
    decoding_attention/attn1.py:217-236.
    """
    return torch.matmul(torch.matmul(_cpu32(Q), _cpu32(K).transpose(1, 2)), _cpu32(V).transpose(1, 2))


def linear(x, w):
    """``a @ b.t()`` in fp32 (demo/gemm_run.py:29, demo/skinny_gemm_test.py:5-6)."""
    return _cpu32(x) @ _cpu32(w).t()


def rmsnorm(x, gamma, eps=1e-6):
    """``F.rms_norm(x.float(), (K,), weight=gamma, eps)``.

    python/cutedsl_kernels/rmsnorm_linear/attempt1/gemm.py:721 normalises with
    ``rms_norm(a.float(), normalized_shape=(k,), eps)``; the decode path adds the
    learned gain ``gamma`` (the reference kernel has none).
    """
    xf = _cpu32(x)
    g = None if gamma is None else _cpu32(gamma)
    return F.rms_norm(xf, (xf.shape[-1],), weight=g, eps=eps)


def rmsnorm_linear(x, gamma, w, eps=1e-6):
    """``rms_norm(x) @ W.t()`` in fp32 (rmsnorm_linear/attempt1/gemm.py:721-722, plus gamma)."""
    return rmsnorm(x, gamma, eps) @ _cpu32(w).t()


def silu(x):
    """``x / (1 + exp(-x))`` (swiglu/attempt1/gemm2.py:63-66 computes it via exp2)."""
    return F.silu(x)


def swiglu(x, w_gate_up):
    """``o1, o2 = (a @ bb1.t()).chunk(2, 1); silu(o1) * o2`` (demo/swiglu.py:47-49).

    ``w_gate_up`` is [2N, K]: gate rows first, then up rows.
    """
    o = _cpu32(x) @ _cpu32(w_gate_up).t()
    g, u = o.chunk(2, dim=-1)
    return silu(g) * u


def swiglu_separate(x, b, b1):
    """``silu(a @ b.t()) * (a @ b1.t())`` (swiglu/attempt1/gemm2.py:714-717, two weights)."""
    xf = _cpu32(x)
    return silu(xf @ _cpu32(b).t()) * (xf @ _cpu32(b1).t())


def lora_linear(x, w, lora_a, lora_b, lora_xa=None):
    """``(a @ b.t()) + (a @ lA.t() @ lB.t())`` in fp32 (lora/attempt1/gemm.py:672-675).

    The reference kernel takes ``lora_xA = a @ lA.t()`` precomputed by torch
    (gemm.py:700-704); pass that bf16 tensor as ``lora_xa`` to check a kernel
    that was given the same operand.
    """
    xf = _cpu32(x)
    xa = _cpu32(lora_xa) if lora_xa is not None else xf @ _cpu32(lora_a).t()
    return xf @ _cpu32(w).t() + xa @ _cpu32(lora_b).t()


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def decode_layer(x, weights: dict, k_cache, v_cache, cache_seqlens, eps=1e-6,
                 num_heads_q=32, num_heads_kv=8, round_intermediates=True):
    """Unfused Llama-style decoder-layer decode step in fp32.

    Composition of the functions above (the full-layer config of the decode
    path): ``h = x + Wo·attn(rmsnorm(x)·Wqkv)``, ``y = h + Wdown·swiglu(rmsnorm(h)·Wgu)``.
    The new token's K/V are appended after the first ``cache_seqlens[b]`` keys of
    each row (the caches themselves are not modified) and attention runs over
    ``cache_seqlens[b] + 1`` keys.
    With ``round_intermediates`` every hand-off between kernels is rounded to
    bf16, as the kernels' bf16 outputs are.

    weights: ``gamma_attn [H]``, ``w_qkv [(Hq+2Hkv)·128, H]``, ``w_o [H, Hq·128]``,
    ``gamma_ffn [H]``, ``w_gate_up [2F, H]``, ``w_down [H, F]``.
    Returns (y [B, H] fp32, new_k_rows, new_v_rows, new_seqlens).
    """
    rnd = _bf16 if round_intermediates else (lambda t: t)
    xf = _cpu32(x)
    B, H = xf.shape
    D = 128
    qkv = rnd(rmsnorm_linear(xf, weights["gamma_attn"], weights["w_qkv"], eps))
    q = qkv[:, : num_heads_q * D].reshape(B, num_heads_q, D)
    k_new = qkv[:, num_heads_q * D:(num_heads_q + num_heads_kv) * D].reshape(B, num_heads_kv, D)
    v_new = qkv[:, (num_heads_q + num_heads_kv) * D:].reshape(B, num_heads_kv, D)
    lens = cache_seqlens.detach().to("cpu", torch.int64)
    attn = torch.empty(B, num_heads_q * D)
    for b in range(B):  # per row: the cached keys plus the appended one; no full-cache copy
        L = int(lens[b])
        kb = torch.cat([_cpu32(k_cache[b, :L]), k_new[b:b + 1]], 0).unsqueeze(0)
        vb = torch.cat([_cpu32(v_cache[b, :L]), v_new[b:b + 1]], 0).unsqueeze(0)
        o, _ = decode_attention(q[b:b + 1], kb, vb, torch.tensor([L + 1]))
        attn[b] = o.reshape(-1)
    new_lens = (lens + 1).to(torch.int32)
    attn = rnd(attn)
    h = rnd(xf + linear(attn, weights["w_o"]))
    gu = rnd(swiglu(rmsnorm(h, weights["gamma_ffn"], eps), weights["w_gate_up"]))
    y = h + linear(gu, weights["w_down"])
    return y, k_new, v_new, new_lens
