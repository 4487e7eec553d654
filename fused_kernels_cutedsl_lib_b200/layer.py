"""Llama-style decoder-layer decode step built from this library's kernels.

One step for a batch of B sequences, each generating one token:

1. ``qkv = rms_norm(x, gamma_attn) @ W_qkv^T``      fused RMSNorm->QKV GEMM, whose epilogue also
2. appends the new K/V rows to the cache at ``cache_seqlens[b]`` (lengths += 1, published by attention)
3. ``attn = softmax(q K^T / sqrt(d)) V``             split-KV attention, q read in place from qkv
4. ``h = x + attn @ W_o^T``                          GEMM with residual epilogue
5. ``gu = silu(g) * u`` for ``[g; u] = rms_norm(h, gamma_ffn) @ W_gu^T``   fused RMSNorm->gate/up->SwiGLU
6. ``y = h + gu @ W_down^T``                         GEMM with residual epilogue

Eleven kernel launches (tcgen05 path: RMSNorm prologue, GEMM and split-row-block
reduction per RMSNorm GEMM, GEMM and reduction per plain GEMM, one single-launch
attention), no host synchronisation and no torch compute on the path.
The reference has no layer composition; this follows the decode path's full
layer configuration (hidden 4096, 32 q / 8 kv heads of 128, FFN 14336).

:class:`TPDecodeLayer` runs the same step on P GPUs (one process each):
GEMMs are column-parallel (each rank holds 1/P of every weight's output
features) with an NCCL all-gather of each GEMM's output, and attention is
batch-parallel (each rank holds the KV cache of B/P rows), its output
all-gathered over rows. :class:`PeerTPDecodeLayer` computes the same step with
the all-gathers done by the kernels themselves: each GEMM epilogue and
attention's merge store their output blocks into every rank's buffer over
peer memory, with a stage barrier kernel between stages.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _native
from ._tensors import ptr, stream_for
from .decoding_attention import (alloc_counters, alloc_partials, attn_fused_launch, plan_attention,
                                 shared_counters)
from .gemm import alloc_workspace, linear, workspace_bytes, workspace_for
from .sharding import column_range, shard_gate_up

HEAD_DIM = 128


@dataclass
class LayerWeights:
    gamma_attn: torch.Tensor  # [H]
    w_qkv: torch.Tensor       # [(Hq + 2 Hkv) * 128, H]
    w_o: torch.Tensor         # [H, Hq * 128]
    gamma_ffn: torch.Tensor   # [H]
    w_gate_up: torch.Tensor   # [2F, H], gate rows then up rows
    w_down: torch.Tensor      # [H, F]

    def as_dict(self) -> dict:
        return dict(gamma_attn=self.gamma_attn, w_qkv=self.w_qkv, w_o=self.w_o, gamma_ffn=self.gamma_ffn,
                    w_gate_up=self.w_gate_up, w_down=self.w_down)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.as_dict().values())


def random_layer_weights(hidden=4096, ffn=14336, num_heads_q=32, num_heads_kv=8, seed=4, device="cuda",
                         std=0.02) -> LayerWeights:
    """bf16 weights N(0, std) and gains 1 + N(0, 0.1), drawn from ``seed``."""
    g = torch.Generator(device=device).manual_seed(seed)

    def w(*shape):
        return (torch.randn(*shape, generator=g, device=device) * std).to(torch.bfloat16)

    def gain(n):
        return (1 + 0.1 * torch.randn(n, generator=g, device=device)).to(torch.bfloat16)

    qkv = (num_heads_q + 2 * num_heads_kv) * HEAD_DIM
    return LayerWeights(gamma_attn=gain(hidden), w_qkv=w(qkv, hidden), w_o=w(hidden, num_heads_q * HEAD_DIM),
                        gamma_ffn=gain(hidden), w_gate_up=w(2 * ffn, hidden), w_down=w(hidden, ffn))


def kv_append(qkv, k_cache, v_cache, cache_seqlens, num_heads_q, num_heads_kv, seqlens_out=None, stream=None):
    """Write the new K/V rows held in ``qkv`` into the caches; lengths updated in ``seqlens_out``."""
    B, L = k_cache.shape[0], k_cache.shape[1]
    st = stream_for(qkv.device, stream)
    out = cache_seqlens if seqlens_out is None else seqlens_out
    _native.check(_native.load().fk_kv_append(
        ptr(qkv), qkv.stride(0), num_heads_q * HEAD_DIM, (num_heads_q + num_heads_kv) * HEAD_DIM,
        ptr(k_cache), ptr(v_cache), ptr(cache_seqlens), ptr(out), B, L, num_heads_kv, HEAD_DIM, st))


def kv_append_paged(qkv, k_pool, v_pool, block_table, cache_seqlens, num_heads_q, num_heads_kv, seqlens_out=None,
                    stream=None):
    """Paged form of :func:`kv_append`: row len of b goes to block ``block_table[b, len // bs]``."""
    B, MB = block_table.shape
    bs = k_pool.shape[1]
    st = stream_for(qkv.device, stream)
    out = cache_seqlens if seqlens_out is None else seqlens_out
    _native.check(_native.load().fk_kv_append_paged(
        ptr(qkv), qkv.stride(0), num_heads_q * HEAD_DIM, (num_heads_q + num_heads_kv) * HEAD_DIM,
        ptr(k_pool), ptr(v_pool), ptr(block_table), ptr(cache_seqlens), ptr(out), B, MB, bs, num_heads_kv,
        HEAD_DIM, st))


def attention_from_qkv(qkv, k_cache, v_cache, cache_seqlens, out, lse, o_partial, lse_partial, num_splits,
                       num_heads_q, num_heads_kv, softmax_scale=None, stream=None, counters=None,
                       single_launch=True):
    """Split-KV attention reading q from the first ``Hq*128`` columns of each ``qkv`` row."""
    B, L = k_cache.shape[0], k_cache.shape[1]
    scale = 1.0 / math.sqrt(HEAD_DIM) if softmax_scale is None else float(softmax_scale)
    st = stream_for(qkv.device, stream)
    if not single_launch:
        _native.check(_native.load().fk_dec_attn_fwd_ex(
            ptr(qkv), qkv.stride(0), ptr(k_cache), ptr(v_cache), ptr(cache_seqlens), ptr(out), ptr(lse),
            ptr(o_partial), ptr(lse_partial), B, L, num_heads_q, num_heads_kv, HEAD_DIM, num_splits, scale, st))
        return
    if counters is None:
        counters = shared_counters(B * num_heads_kv, qkv.device, st)
    attn_fused_launch(ptr(qkv), qkv.stride(0), k_cache, v_cache, cache_seqlens, ptr(out), lse, o_partial,
                      lse_partial, counters, batch=B, max_seqlen=L, num_heads_q=num_heads_q,
                      num_heads_kv=num_heads_kv, num_splits=num_splits, softmax_scale=scale, stream_handle=st)


def linear_kv_append(x, w, out, k_cache, v_cache, cache_seqlens, seqlens_next, num_heads_q, num_heads_kv, *,
                     gamma=None, eps=1e-6, block_table=None, workspace=None, stream=None):
    """QKV projection (RMSNorm-fused when ``gamma`` is given) whose epilogue also
    writes the new K/V rows into the caches at ``cache_seqlens[b]`` and the
    advanced lengths into ``seqlens_next`` (a different tensor). With
    ``block_table`` the caches are block pools ``[num_blocks, block_size, Hkv, D]``."""
    M, K = x.shape
    N = w.shape[0]
    if seqlens_next is not None and seqlens_next.data_ptr() == cache_seqlens.data_ptr():
        raise ValueError("seqlens_next must not alias cache_seqlens")
    if block_table is not None:
        cap = block_table.shape[1] * k_cache.shape[1]
        bs = k_cache.shape[1]
    else:
        cap, bs = k_cache.shape[1], 0
    dev = x.device
    st = stream_for(dev, stream)
    need = workspace_bytes(M, N, K)
    ws = workspace if workspace is not None else workspace_for(need, dev)
    _native.check(_native.load().fk_linear_kv_append(
        ptr(x), ptr(gamma) if gamma is not None else None, ptr(w), ptr(out), M, N, K, float(eps),
        ptr(k_cache), ptr(v_cache), ptr(block_table) if block_table is not None else None, ptr(cache_seqlens),
        ptr(seqlens_next) if seqlens_next is not None else None, num_heads_q * HEAD_DIM,
        (num_heads_q + num_heads_kv) * HEAD_DIM, num_heads_kv, HEAD_DIM, cap, bs, ptr(ws),
        ws.numel() * ws.element_size(), st))
    return out


def attention_commit(qkv, k_cache, v_cache, cache_seqlens, seqlens_commit, out, lse, o_partial, lse_partial,
                     num_splits, num_heads_q, num_heads_kv, *, block_table=None, softmax_scale=None, stream=None,
                     counters=None, single_launch=True):
    """:func:`attention_from_qkv` that also copies the lengths it used into
    ``seqlens_commit`` (a different tensor from ``cache_seqlens``), written by
    the unit that finishes each row (``single_launch``) or by pass 2."""
    B = qkv.shape[0]
    if block_table is not None:
        bs = k_cache.shape[1]
        L, nblk = block_table.shape[1] * bs, k_cache.shape[0]
    else:
        L, bs, nblk = k_cache.shape[1], 0, 0
    scale = 1.0 / math.sqrt(HEAD_DIM) if softmax_scale is None else float(softmax_scale)
    st = stream_for(qkv.device, stream)
    if not single_launch:
        _native.check(_native.load().fk_dec_attn_fwd_commit(
            ptr(qkv), qkv.stride(0), ptr(k_cache), ptr(v_cache),
            ptr(block_table) if block_table is not None else None, ptr(cache_seqlens), ptr(seqlens_commit),
            ptr(out), ptr(lse), ptr(o_partial), ptr(lse_partial), B, L, bs, nblk, num_heads_q, num_heads_kv,
            HEAD_DIM, num_splits, scale, st))
        return
    if counters is None:
        counters = shared_counters(B * num_heads_kv, qkv.device, st)
    attn_fused_launch(ptr(qkv), qkv.stride(0), k_cache, v_cache, cache_seqlens, ptr(out), lse, o_partial,
                      lse_partial, counters, batch=B, max_seqlen=L, num_heads_q=num_heads_q,
                      num_heads_kv=num_heads_kv, num_splits=num_splits, softmax_scale=scale, stream_handle=st,
                      block_table=block_table, block_size=bs, num_blocks=nblk, seqlens_commit=seqlens_commit)


class DecodeLayer:
    """Single-GPU decode step. ``layer(x, k_cache, v_cache, cache_seqlens) -> y``.

    Appends the new token's K/V in place and advances ``cache_seqlens`` by one
    (rows whose cache is full keep their length). Intermediate buffers are
    allocated once per batch size and reused, so steady-state calls allocate
    nothing and the step can be replayed inside a CUDA graph.
    """

    def __init__(self, weights: LayerWeights, num_heads_q=32, num_heads_kv=8, eps=1e-6, num_splits=None,
                 fuse_append=True):
        self.fuse_append = fuse_append  # KV append in the QKV epilogue (else a separate append kernel)
        self.w = weights
        self.hq, self.hkv, self.eps = num_heads_q, num_heads_kv, eps
        self.num_splits = num_splits
        self.hidden = weights.w_qkv.shape[1]
        self.ffn = weights.w_gate_up.shape[0] // 2
        self.qkv_dim = weights.w_qkv.shape[0]
        self._bufs: dict = {}

    def buffers(self, B: int, L: int, device) -> dict:
        key = (B, L, str(device))
        b = self._bufs.get(key)
        if b is None:
            single, S = plan_attention(B, self.hkv, L)
            if self.num_splits:
                S = self.num_splits
                single = single and S >= 2
            o_p, l_p = alloc_partials(B, self.hq, S, device)
            ws = max(workspace_bytes(B, n, k, sw) for n, k, sw in [
                (self.qkv_dim, self.hidden, False), (self.hidden, self.hq * HEAD_DIM, False),
                (self.ffn, self.hidden, True), (self.hidden, self.ffn, False)])
            bf = dict(dtype=torch.bfloat16, device=device)
            b = dict(S=S, single=single, o_p=o_p, l_p=l_p, ws=alloc_workspace(ws, device),
                     ctr=alloc_counters(B, self.hkv, device),
                     qkv=torch.empty(B, self.qkv_dim, **bf), attn=torch.empty(B, self.hq * HEAD_DIM, **bf),
                     lse=torch.empty(B, self.hq, dtype=torch.float32, device=device),
                     h=torch.empty(B, self.hidden, **bf), gu=torch.empty(B, self.ffn, **bf),
                     y=torch.empty(B, self.hidden, **bf),
                     lens_next=torch.empty(B, dtype=torch.int32, device=device))
            self._bufs[key] = b
        return b

    def __call__(self, x, k_cache, v_cache, cache_seqlens, out=None, stream=None):
        B, L = x.shape[0], k_cache.shape[1]
        b = self.buffers(B, L, x.device)
        w, ws = self.w, b["ws"]
        if self.fuse_append:
            # QKV epilogue appends K/V and writes the advanced lengths to lens_next;
            # attention reads lens_next and publishes it back to cache_seqlens.
            linear_kv_append(x, w.w_qkv, b["qkv"], k_cache, v_cache, cache_seqlens, b["lens_next"], self.hq,
                             self.hkv, gamma=w.gamma_attn, eps=self.eps, workspace=ws, stream=stream)
            attention_commit(b["qkv"], k_cache, v_cache, b["lens_next"], cache_seqlens, b["attn"], b["lse"],
                             b["o_p"], b["l_p"], b["S"], self.hq, self.hkv, stream=stream, counters=b["ctr"],
                             single_launch=b["single"])
        else:
            linear(x, w.w_qkv, b["qkv"], gamma=w.gamma_attn, eps=self.eps, workspace=ws, stream=stream)
            kv_append(b["qkv"], k_cache, v_cache, cache_seqlens, self.hq, self.hkv, stream=stream)
            attention_from_qkv(b["qkv"], k_cache, v_cache, cache_seqlens, b["attn"], b["lse"], b["o_p"], b["l_p"],
                               b["S"], self.hq, self.hkv, stream=stream, counters=b["ctr"],
                               single_launch=b["single"])
        linear(b["attn"], w.w_o, b["h"], residual=x, workspace=ws, stream=stream)
        linear(b["h"], w.w_gate_up, b["gu"], gamma=w.gamma_ffn, eps=self.eps, w_up=w.w_gate_up,
               up_row_offset=self.ffn, workspace=ws, stream=stream)
        y = b["y"] if out is None else out
        linear(b["gu"], w.w_down, y, residual=b["h"], workspace=ws, stream=stream)
        return y


def shard_layer_weights(full: LayerWeights, rank: int, world: int, num_heads_q=32, num_heads_kv=8) -> LayerWeights:
    """Column (output-feature) shard of every weight for tensor-parallel rank ``rank``."""
    qkv_lo, qkv_hi = column_range(full.w_qkv.shape[0], rank, world)
    h_lo, h_hi = column_range(full.w_o.shape[0], rank, world)
    return LayerWeights(
        gamma_attn=full.gamma_attn, gamma_ffn=full.gamma_ffn,
        w_qkv=full.w_qkv[qkv_lo:qkv_hi].contiguous(),
        w_o=full.w_o[h_lo:h_hi].contiguous(),
        w_gate_up=shard_gate_up(full.w_gate_up, rank, world),
        w_down=full.w_down[h_lo:h_hi].contiguous())


class KernelOps:
    """The compute steps of the TP layer, on this library's kernels (the product path)."""

    def __init__(self, num_heads_q, num_heads_kv, eps):
        self.hq, self.hkv, self.eps = num_heads_q, num_heads_kv, eps

    def _wsp(self, x):
        return None  # the per-device shared workspace of gemm.linear, grown on demand

    def rms_linear(self, x, gamma, w, out):
        return linear(x, w, out, gamma=gamma, eps=self.eps, workspace=self._wsp(x))

    def linear(self, x, w, out, residual=None):
        return linear(x, w, out, residual=residual, workspace=self._wsp(x))

    def rms_swiglu(self, x, gamma, w_gate_up, out):
        n = w_gate_up.shape[0] // 2
        return linear(x, w_gate_up, out, gamma=gamma, eps=self.eps, w_up=w_gate_up, up_row_offset=n,
                      workspace=self._wsp(x))

    def append_and_attend(self, qkv, k_cache, v_cache, cache_seqlens, out):
        B, L = k_cache.shape[0], k_cache.shape[1]
        single, S = plan_attention(B, self.hkv, L)
        o_p, l_p = alloc_partials(B, self.hq, S, qkv.device)
        lse = torch.empty(B, self.hq, dtype=torch.float32, device=qkv.device)
        kv_append(qkv, k_cache, v_cache, cache_seqlens, self.hq, self.hkv)
        attention_from_qkv(qkv, k_cache, v_cache, cache_seqlens, out, lse, o_p, l_p, S, self.hq, self.hkv,
                           single_launch=single)
        return out


class TPDecodeLayer:
    """Decode step on P ranks: column-parallel GEMMs + batch-parallel attention.

    ``weights`` is this rank's :func:`shard_layer_weights` shard; ``rows`` the
    contiguous block of batch rows whose KV cache this rank holds (equal blocks
    on every rank). Activations entering a GEMM are replicated; each GEMM's
    output shard is all-gathered (``all_gather_into_tensor``) and re-laid out
    from [P, B, n/P] to [B, n]. Attention output rows are gathered the same way
    (already row-contiguous). ``ops`` defaults to the CUDA kernels.
    """

    def __init__(self, weights: LayerWeights, group=None, num_heads_q=32, num_heads_kv=8, eps=1e-6, ops=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.w = weights
        self.hq, self.hkv = num_heads_q, num_heads_kv
        self.ops = ops if ops is not None else KernelOps(num_heads_q, num_heads_kv, eps)
        for name, n in (("w_qkv", weights.w_qkv.shape[0] * self.world), ("w_o", weights.w_o.shape[0] * self.world),
                        ("w_down", weights.w_down.shape[0] * self.world)):
            if n % (128 * self.world):
                raise ValueError(f"{name}: {n} output features do not split into equal 128-column blocks "
                                 f"over {self.world} ranks")

    def _gather_cols(self, part: torch.Tensor) -> torch.Tensor:
        """[B, n/P] on every rank -> [B, n] (rank-major column blocks)."""
        B, c = part.shape
        buf = torch.empty(self.world * B, c, dtype=part.dtype, device=part.device)
        self.dist.all_gather_into_tensor(buf, part.contiguous(), group=self.group)
        return buf.view(self.world, B, c).permute(1, 0, 2).reshape(B, self.world * c)

    def _gather_rows(self, part: torch.Tensor) -> torch.Tensor:
        buf = torch.empty(self.world * part.shape[0], *part.shape[1:], dtype=part.dtype, device=part.device)
        self.dist.all_gather_into_tensor(buf, part.contiguous(), group=self.group)
        return buf

    def __call__(self, x, k_cache, v_cache, cache_seqlens):
        """x [B, H] replicated; k/v caches and lengths hold this rank's B/P rows. Returns y [B, H]."""
        B = x.shape[0]
        Bl = k_cache.shape[0]
        if Bl * self.world != B:
            raise ValueError(f"batch {B} must split evenly: {Bl} rows per rank x {self.world} ranks")
        w, ops = self.w, self.ops
        dt = dict(dtype=x.dtype, device=x.device)
        qkv = self._gather_cols(ops.rms_linear(x, w.gamma_attn, w.w_qkv, torch.empty(B, w.w_qkv.shape[0], **dt)))
        r0 = self.rank * Bl
        my_qkv = qkv[r0:r0 + Bl].contiguous()
        attn_local = ops.append_and_attend(my_qkv, k_cache, v_cache, cache_seqlens,
                                           torch.empty(Bl, self.hq * HEAD_DIM, **dt))
        attn = self._gather_rows(attn_local)
        c_lo, c_hi = column_range(x.shape[1], self.rank, self.world)
        # residual added in the GEMM epilogue on this rank's column block
        h = self._gather_cols(ops.linear(attn, w.w_o, torch.empty(B, c_hi - c_lo, **dt),
                                         residual=x[:, c_lo:c_hi].contiguous()))
        gu = self._gather_cols(ops.rms_swiglu(h, w.gamma_ffn, w.w_gate_up,
                                              torch.empty(B, w.w_gate_up.shape[0] // 2, **dt)))
        return self._gather_cols(ops.linear(gu, w.w_down, torch.empty(B, c_hi - c_lo, **dt),
                                            residual=h[:, c_lo:c_hi].contiguous()))


def _vp(ptrs):
    arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
    return arr, len(ptrs)


class PeerTPDecodeLayer:
    """Tensor-parallel decode step whose all-gathers are done by the kernels.

    Same sharding and results as :class:`TPDecodeLayer`, but each column-parallel
    GEMM stores its output block straight into the full ``[B, n]`` activation
    buffer of every rank (``fk_linear_ex`` with peer outputs: CUDA IPC mappings
    of a :class:`~fused_kernels_cutedsl_lib_b200.peer.PeerArena`), and attention's
    pass 2 stores this rank's batch rows into every rank's buffer
    (``fk_dec_attn_fwd_peers``). A one-thread stage barrier (``fk_peer_barrier``)
    separates the stages. Per step: no NCCL call, no re-layout copy; 5 barriers.
    Buffers are allocated once per batch size; steady-state calls allocate
    nothing and can be captured in a CUDA graph.
    """

    def __init__(self, weights: LayerWeights, group=None, num_heads_q=32, num_heads_kv=8, eps=1e-6,
                 fold_barriers=True):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.fold_barriers = fold_barriers
        self.w = weights
        self.hq, self.hkv, self.eps = num_heads_q, num_heads_kv, eps
        self.hidden = weights.w_qkv.shape[1]
        self.n_qkv = weights.w_qkv.shape[0] * self.world
        self.ffn = weights.w_gate_up.shape[0] // 2 * self.world
        self.qkv_lo = column_range(self.n_qkv, self.rank, self.world)[0]
        self.c_lo = column_range(self.hidden, self.rank, self.world)[0]
        self.f_lo = column_range(self.ffn, self.rank, self.world)[0]
        self.arena = None
        self._bufs: dict = {}

    def _setup(self, B: int, Bl: int, L: int, device):
        from .peer import PeerArena

        key = (B, Bl, L)
        if key in self._bufs:
            return self._bufs[key]
        H, F = self.hidden, self.ffn
        if self.arena is None:
            self.arena = PeerArena(2 * B * (self.n_qkv + self.hq * HEAD_DIM + 2 * H + F) + (1 << 16), self.group)
        a = self.arena
        single, S = plan_attention(Bl, self.hkv, L)
        o_p, l_p = alloc_partials(Bl, self.hq, S, device)
        ws_need = max(workspace_bytes(B, n, k, sw) for n, k, sw in [
            (self.w.w_qkv.shape[0], H, False), (self.w.w_o.shape[0], self.hq * HEAD_DIM, False),
            (self.w.w_gate_up.shape[0] // 2, H, True), (self.w.w_down.shape[0], F, False)])
        b = dict(qkv=a.region(f"qkv{B}", (B, self.n_qkv)), attn=a.region(f"attn{B}", (B, self.hq * HEAD_DIM)),
                 h=a.region(f"h{B}", (B, H)), gu=a.region(f"gu{B}", (B, F)), y=a.region(f"y{B}", (B, H)),
                 S=S, single=single, o_p=o_p, l_p=l_p,
                 lse=torch.empty(Bl, self.hq, dtype=torch.float32, device=device),
                 ctr=alloc_counters(Bl, self.hkv, device),
                 ws=alloc_workspace(ws_need, device))
        self._bufs[key] = b
        return b

    def _linear(self, x, w, out_region, name, col_lo, n_total, b, *, gamma=None, w_up=None, up_row_offset=0,
                residual=None, ldr=0, wait=False):
        M, K = x.shape
        N = w.shape[0] - up_row_offset if w_up is not None else w.shape[0]
        peers, n = _vp(self.arena.peer_ptrs(name, col_lo))
        ws = b["ws"]
        st = torch.cuda.current_stream(x.device).cuda_stream
        args = (ptr(x), ptr(gamma) if gamma is not None else None, ptr(w), ptr(w_up) if w_up is not None else None,
                up_row_offset, residual, ldr, out_region.data_ptr() + 2 * col_lo, n_total, peers, n, M, N, K,
                float(self.eps), ptr(ws), ws.numel())
        if wait:
            _native.check(_native.load().fk_linear_ex_wait(*args, *self.arena.wait_args(), ctypes.c_void_p(st)))
        else:
            _native.check(_native.load().fk_linear_ex(*args, ctypes.c_void_p(st)))

    def _stage_end(self):
        """Between stages: signal only (the next stage's first kernel waits) when
        folding barriers, else the full barrier kernel."""
        if self.fold_barriers:
            self.arena.signal()
        else:
            self.arena.barrier()

    def __call__(self, x, k_cache, v_cache, cache_seqlens):
        """x [B, H] replicated; k/v caches and lengths hold this rank's B/P rows. Returns y [B, H] (arena view)."""
        B, Bl, L = x.shape[0], k_cache.shape[0], k_cache.shape[1]
        if Bl * self.world != B:
            raise ValueError(f"batch {B} must split evenly: {Bl} rows per rank x {self.world} ranks")
        b = self._setup(B, Bl, L, x.device)
        w, a, H, F = self.w, self.arena, self.hidden, self.ffn
        B_ = str(B)
        st = torch.cuda.current_stream(x.device).cuda_stream
        # QKV: this rank's column block of every row, pushed to all ranks
        self._linear(x, w.w_qkv, b["qkv"], "qkv" + B_, self.qkv_lo, self.n_qkv, b, gamma=w.gamma_attn)
        self._stage_end()
        # attention on this rank's batch rows (q read in place), rows pushed to all ranks
        r0 = self.rank * Bl
        my_qkv = b["qkv"][r0:r0 + Bl]
        if self.fold_barriers:
            _native.check(_native.load().fk_kv_append_wait(
                ptr(my_qkv), my_qkv.stride(0), self.hq * HEAD_DIM, (self.hq + self.hkv) * HEAD_DIM, ptr(k_cache),
                ptr(v_cache), ptr(cache_seqlens), ptr(cache_seqlens), Bl, k_cache.shape[1], self.hkv, HEAD_DIM,
                *a.wait_args(), ctypes.c_void_p(st)))
        else:
            kv_append(my_qkv, k_cache, v_cache, cache_seqlens, self.hq, self.hkv)
        hd = self.hq * HEAD_DIM
        if b["single"]:
            attn_fused_launch(ptr(my_qkv), my_qkv.stride(0), k_cache, v_cache, cache_seqlens,
                              b["attn"].data_ptr() + 2 * r0 * hd, b["lse"], b["o_p"], b["l_p"], b["ctr"], batch=Bl,
                              max_seqlen=L, num_heads_q=self.hq, num_heads_kv=self.hkv, num_splits=b["S"],
                              softmax_scale=1.0 / math.sqrt(HEAD_DIM), stream_handle=st,
                              peer_out=a.peer_ptrs("attn" + B_, r0 * hd))
        else:
            peers, n = _vp(a.peer_ptrs("attn" + B_, r0 * hd))
            _native.check(_native.load().fk_dec_attn_fwd_peers(
                ptr(my_qkv), my_qkv.stride(0), ptr(k_cache), ptr(v_cache), ptr(cache_seqlens),
                b["attn"].data_ptr() + 2 * r0 * hd, peers, n, ptr(b["lse"]), ptr(b["o_p"]), ptr(b["l_p"]), Bl, L,
                self.hq, self.hkv, HEAD_DIM, b["S"], 1.0 / math.sqrt(HEAD_DIM), ctypes.c_void_p(st)))
        self._stage_end()
        fold = self.fold_barriers
        # O-projection + residual x
        self._linear(b["attn"], w.w_o, b["h"], "h" + B_, self.c_lo, H, b, residual=x.data_ptr() + 2 * self.c_lo,
                     ldr=H, wait=fold)
        self._stage_end()
        # RMSNorm -> gate/up -> SwiGLU
        fl = w.w_gate_up.shape[0] // 2
        self._linear(b["h"], w.w_gate_up, b["gu"], "gu" + B_, self.f_lo, F, b, gamma=w.gamma_ffn,
                     w_up=w.w_gate_up, up_row_offset=fl, wait=fold)
        self._stage_end()
        # down-projection + residual h
        self._linear(b["gu"], w.w_down, b["y"], "y" + B_, self.c_lo, H, b,
                     residual=b["h"].data_ptr() + 2 * self.c_lo, ldr=H, wait=fold)
        a.barrier()  # full barrier: y is complete on every rank when the call returns
        return b["y"]

    def close(self):
        if self.arena is not None:
            self.arena.close()
            self.arena = None
            self._bufs.clear()


class HybridDecodeLayer:
    """Decode step on P GPUs: the attention block batch-parallel, the FFN tensor-parallel.

    Each rank holds the attention-side weights whole (W_qkv, W_o, 84 MB at config
    5) and a column shard of the FFN weights (W_gate_up, W_down: 352 MB / P).
    Per step, with ``x`` the full [B, H] input (replicated):

    1. RMSNorm -> QKV for this rank's B/P rows, KV append in the epilogue, attention
       over the rows' own cache, O-projection + residual: all local, no exchange;
       the O-projection's epilogue stores its rows into every rank's ``h`` buffer;
    2. RMSNorm -> gate/up -> SwiGLU on all B rows for this rank's FFN columns,
       stored into every rank's ``gu`` buffer at its column offset;
    3. down-projection + residual for this rank's columns, stored into every
       rank's ``y`` buffer.

    A stage barrier separates the stages: 3 per step instead of the 5 of
    :class:`PeerTPDecodeLayer`, and the attention-side GEMMs run on B/P rows of
    whole weights (the weight-streaming path at B/P <= 16) instead of on N/P
    columns of all rows. The exchanges are plain stores into CUDA IPC mappings
    of the peers' buffers (no NCCL on the data path). Returns ``y`` [B, H], a
    view into the shared arena valid until the next call.
    """

    def __init__(self, full: LayerWeights, group=None, num_heads_q=32, num_heads_kv=8, eps=1e-6,
                 fold_barriers=True):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.fold_barriers = fold_barriers
        self.hq, self.hkv, self.eps = num_heads_q, num_heads_kv, eps
        self.hidden = full.w_qkv.shape[1]
        self.ffn = full.w_gate_up.shape[0] // 2
        shard = shard_layer_weights(full, self.rank, self.world, num_heads_q, num_heads_kv)
        self.w_attn = full  # gammas, W_qkv and W_o are used whole
        self.w_gate_up, self.w_down = shard.w_gate_up, shard.w_down
        self.c_lo = column_range(self.hidden, self.rank, self.world)[0]
        self.f_lo = column_range(self.ffn, self.rank, self.world)[0]
        self.arena = None
        self._bufs: dict = {}

    def _setup(self, B: int, Bl: int, L: int, device):
        from .peer import PeerArena

        key = (B, Bl, L)
        if key in self._bufs:
            return self._bufs[key]
        H, F = self.hidden, self.ffn
        if self.arena is None:
            self.arena = PeerArena(2 * B * (2 * H + F) + (1 << 16), self.group)
        a = self.arena
        single, S = plan_attention(Bl, self.hkv, L)
        o_p, l_p = alloc_partials(Bl, self.hq, S, device)
        qkv_dim = self.w_attn.w_qkv.shape[0]
        ws_need = max(workspace_bytes(m, n, k, sw) for m, n, k, sw in [
            (Bl, qkv_dim, H, False), (Bl, H, self.hq * HEAD_DIM, False),
            (B, self.w_gate_up.shape[0] // 2, H, True), (B, self.w_down.shape[0], F, False)])
        bf = dict(dtype=torch.bfloat16, device=device)
        b = dict(h=a.region(f"h{B}", (B, H)), gu=a.region(f"gu{B}", (B, F)), y=a.region(f"y{B}", (B, H)),
                 qkv=torch.empty(Bl, qkv_dim, **bf), attn=torch.empty(Bl, self.hq * HEAD_DIM, **bf),
                 lse=torch.empty(Bl, self.hq, dtype=torch.float32, device=device),
                 lens_next=torch.empty(Bl, dtype=torch.int32, device=device),
                 S=S, single=single, o_p=o_p, l_p=l_p, ctr=alloc_counters(Bl, self.hkv, device),
                 ws=alloc_workspace(ws_need, device))
        self._bufs[key] = b
        return b

    def _linear(self, x, w, y_ptr, ldy, peers, M, N, K, b, *, gamma=None, w_up=None, up_row_offset=0,
                residual=None, ldr=0, wait=False):
        pp, n = _vp(peers)
        ws = b["ws"]
        st = torch.cuda.current_stream(x.device).cuda_stream
        args = (ptr(x), ptr(gamma) if gamma is not None else None, ptr(w), ptr(w_up) if w_up is not None else None,
                up_row_offset, residual, ldr, y_ptr, ldy, pp, n, M, N, K, float(self.eps), ptr(ws), ws.numel())
        if wait:
            _native.check(_native.load().fk_linear_ex_wait(*args, *self.arena.wait_args(), ctypes.c_void_p(st)))
        else:
            _native.check(_native.load().fk_linear_ex(*args, ctypes.c_void_p(st)))

    def _stage_end(self):
        if self.fold_barriers:
            self.arena.signal()
        else:
            self.arena.barrier()

    def __call__(self, x, k_cache, v_cache, cache_seqlens):
        """x [B, H] replicated; k/v caches and lengths hold this rank's B/P rows. Returns y [B, H] (arena view)."""
        B, Bl, L = x.shape[0], k_cache.shape[0], k_cache.shape[1]
        if Bl * self.world != B:
            raise ValueError(f"batch {B} must split evenly: {Bl} rows per rank x {self.world} ranks")
        b = self._setup(B, Bl, L, x.device)
        w, a, H, F = self.w_attn, self.arena, self.hidden, self.ffn
        B_ = str(B)
        r0 = self.rank * Bl
        x_loc = x[r0:r0 + Bl]
        # 1. attention block on this rank's rows: QKV (+ KV append), attention, O-proj + residual
        linear_kv_append(x_loc, w.w_qkv, b["qkv"], k_cache, v_cache, cache_seqlens, b["lens_next"], self.hq,
                         self.hkv, gamma=w.gamma_attn, eps=self.eps, workspace=b["ws"])
        attention_commit(b["qkv"], k_cache, v_cache, b["lens_next"], cache_seqlens, b["attn"], b["lse"], b["o_p"],
                         b["l_p"], b["S"], self.hq, self.hkv, counters=b["ctr"], single_launch=b["single"])
        self._linear(b["attn"], w.w_o, b["h"].data_ptr() + 2 * r0 * H, H, a.peer_ptrs("h" + B_, r0 * H), Bl, H,
                     self.hq * HEAD_DIM, b, residual=x_loc.data_ptr(), ldr=x.stride(0))
        self._stage_end()
        fold = self.fold_barriers
        # 2. RMSNorm -> gate/up -> SwiGLU, this rank's FFN columns of all rows
        fl = self.w_gate_up.shape[0] // 2
        self._linear(b["h"], self.w_gate_up, b["gu"].data_ptr() + 2 * self.f_lo, F, a.peer_ptrs("gu" + B_, self.f_lo),
                     B, fl, H, b, gamma=w.gamma_ffn, w_up=self.w_gate_up, up_row_offset=fl, wait=fold)
        self._stage_end()
        # 3. down-projection + residual h, this rank's columns of all rows
        self._linear(b["gu"], self.w_down, b["y"].data_ptr() + 2 * self.c_lo, H, a.peer_ptrs("y" + B_, self.c_lo),
                     B, self.w_down.shape[0], F, b, residual=b["h"].data_ptr() + 2 * self.c_lo, ldr=H, wait=fold)
        a.barrier()  # full barrier: y is complete on every rank when the call returns
        return b["y"]

    def close(self):
        if self.arena is not None:
            self.arena.close()
            self.arena = None
            self._bufs.clear()
