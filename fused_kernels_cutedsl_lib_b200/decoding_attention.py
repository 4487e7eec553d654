"""Split-KV decode attention (host side of ``csrc/dec_attn.cu``).

Reference boundary: the reference exports its decode attention as a kernel
object, ``DAttn1(qk_mnk, stages, p_stages, is_persistent)``, compiled by
``compile_cutedsl`` into a callable over torch tensors
(python/cutedsl_kernels/decoding_attention/attn1.py:70-90,
python/cdsl_helpers/cdsl_fn_utils.py:38-44). The callable writes the
caller-allocated output in place and returns ``None``. This module keeps that
ownership and calling style for the split-KV decode path:

* :func:`dec_attn_splitkv_fwd` — the whole attention, either in ONE launch
  (the C ABI ``fk_dec_attn_fwd_fused``: stream-K ranges of tiles, the last
  piece of each (row, kv head) to finish merges the pair) or as two launches
  (``fk_dec_attn_fwd``: fixed chunks, then pass 2); :func:`plan_attention`
  picks the form by the batch's size;
* :func:`dec_attn_splitkv_partial` / :func:`dec_attn_combine` — pass 1 / pass 2;
* :class:`DecodeAttention` — a kernel object in the reference's style whose
  ``__call__(q, k_cache, v_cache, cache_seqlens, out, lse, softmax_scale)``
  allocates the split partials itself (once, cached per shape).

Semantics (softmax, GQA, natural-log LSE, empty rows) follow the reference's
attention references ``attn_reimpl`` (attn/attempt6_epi_pipeline/attn.py:778-784)
and SDPA (attn/attempt6_epi_pipeline/tests.py:85), with the zero-row-sum guard of
attn/attempt6_epi_pipeline/my_softmax.py:88-97 (a row with no keys yields 0).
"""
from __future__ import annotations

import ctypes
import math
import threading

import torch

from . import _native
from ._tensors import ptr, require_shape, require_tensor, same_device, stream_for

HEAD_DIM = 128
TILE_TOKENS = 64


def chunk_tokens(max_seqlen: int, num_splits: int) -> int:
    """Tokens per split: ceil(max_seqlen / num_splits) rounded up to 64."""
    c = -(-max_seqlen // num_splits)
    return -(-c // TILE_TOKENS) * TILE_TOKENS


def default_num_splits(batch: int, num_heads_kv: int, max_seqlen: int,
                       total_tokens: int | None = None, num_sms: int = 148) -> int:
    """Pick num_splits: the largest chunk of {1024, 512, 256, 128, 64} tokens
    that still gives work units (row, kv head, split) for at least three
    quarters of the SMs.

    Large chunks amortise each unit's setup (q load, pipeline fill) and keep
    the merge of the splits short; at config 2's ~1.1 M tokens 1024-token
    chunks still give ~8700 units, dealt round-robin. At config 1 (B = 4,
    L = 4096) the rule gives 4 splits = 128 units, one per SM on 128 of the 148
    SMs, each streaming 512 KB. Measured there in one call (two-launch form):
    4 splits 21.5 us isolated / 16.8 us back to back, 8 splits (256 units,
    the earlier one-unit-per-SM rule) 21.5 / 17.5 us, 16 splits 25.6 / 20.1 us,
    64 splits (an older "4 units per resident CTA" rule) 36.5 us back to back;
    configs 1 and 2 are the measured shapes.

    ``total_tokens`` (sum of the true lengths) sharpens the count for ragged
    batches. Callers whose lengths live on the GPU (the decode layer) leave it
    out: reading them would synchronise the host with the device every step,
    so the padded count ``batch * max_seqlen`` stands in and can pick a larger
    chunk than the true work supports.
    """
    total = total_tokens if total_tokens is not None else batch * max_seqlen
    chunk = TILE_TOKENS
    for c in (1024, 512, 256, 128, 64):
        units = num_heads_kv * max(1, -(-total // c))
        if 4 * units >= 3 * num_sms:
            chunk = c
            break
    return max(1, -(-max_seqlen // chunk))


def fused_partial_slots(batch: int, num_heads_kv: int, max_seqlen: int, num_sms: int = 148) -> int:
    """Partial slots per (row, kv head) for the single-launch form.

    That form cuts the batch's (row, kv head, 64-token tile) sequence into one
    equal range per resident CTA (two per SM) and merges the pieces of each pair
    in-kernel; a pair cut into n pieces uses n partial slots. The kernel picks
    ranges long enough that no pair needs more slots than the buffer holds, so
    more slots let it keep every CTA busy on shorter (ragged) batches. This
    sizes the buffer for a batch whose true tokens are down to a quarter of the
    padded ``batch * max_seqlen``: ceil(tiles per row * CTAs * 4 / padded
    tiles) + 1, within [2, tiles per row + 1].
    """
    ntmax = -(-max_seqlen // TILE_TOKENS)
    grid = 2 * num_sms
    padded = max(1, batch * num_heads_kv * ntmax)
    slots = -(-(ntmax * grid * 4) // padded) + 1
    return max(2, min(slots, ntmax + 1))


# Padded tiles per resident CTA from which the single launch pays off. Below it
# (config 1: B = 4, L = 4096 gives 7) the in-kernel merge's atomic and L2 round
# trips at the end of the kernel cost more than pass 2 launched as a programmatic
# dependent: measured 23.3 vs 21.5 us per call at config 1, while at config 2
# (885 per CTA) the single launch is faster (674 vs 684-687 us).
SINGLE_LAUNCH_MIN_TILES_PER_CTA = 32


def plan_attention(batch: int, num_heads_kv: int, max_seqlen: int, num_sms: int = 148) -> tuple[bool, int]:
    """(single_launch, num_splits) for a batch shape: the single-launch form with
    :func:`fused_partial_slots` slots when the batch gives every resident CTA (two
    per SM) at least ``SINGLE_LAUNCH_MIN_TILES_PER_CTA`` padded 64-token tiles,
    else the two-launch form with :func:`default_num_splits` chunks."""
    ntmax = -(-max_seqlen // TILE_TOKENS)
    per_cta = batch * num_heads_kv * ntmax / (2 * num_sms)
    if per_cta >= SINGLE_LAUNCH_MIN_TILES_PER_CTA:
        return True, fused_partial_slots(batch, num_heads_kv, max_seqlen, num_sms)
    return False, default_num_splits(batch, num_heads_kv, max_seqlen, num_sms=num_sms)


def _check_attn(q, k_cache, v_cache, cache_seqlens):
    require_tensor("q", q, torch.bfloat16)
    require_tensor("k_cache", k_cache, torch.bfloat16, 4)
    require_tensor("v_cache", v_cache, torch.bfloat16, 4)
    require_tensor("cache_seqlens", cache_seqlens, torch.int32, 1)
    B, L, Hkv, D = k_cache.shape
    require_shape("v_cache", v_cache, (B, L, Hkv, D))
    if D != HEAD_DIM:
        raise ValueError(f"head_dim must be {HEAD_DIM}, got {D}")
    if q.dim() == 4:
        if q.shape[1] != 1:
            raise ValueError("decode attention takes one query token per row (q.shape[1] == 1)")
        Hq = q.shape[2]
    elif q.dim() == 3:
        Hq = q.shape[1]
    else:
        raise ValueError(f"q must be [B, 1, Hq, D] or [B, Hq, D], got {tuple(q.shape)}")
    if q.shape[0] != B or q.shape[-1] != D:
        raise ValueError(f"q shape {tuple(q.shape)} does not match k_cache {tuple(k_cache.shape)}")
    if Hq % Hkv != 0 or Hq // Hkv > 8:
        raise ValueError(f"num_heads_q ({Hq}) must be a multiple of num_heads_kv ({Hkv}), ratio <= 8")
    require_shape("cache_seqlens", cache_seqlens, (B,))
    dev = same_device(q, k_cache, v_cache, cache_seqlens)
    return B, L, Hq, Hkv, D, dev


def alloc_partials(batch: int, num_heads_q: int, num_splits: int, device) -> tuple[torch.Tensor, torch.Tensor]:
    o_partial = torch.empty((num_splits, batch, num_heads_q, HEAD_DIM), dtype=torch.float32, device=device)
    lse_partial = torch.empty((num_splits, batch, num_heads_q), dtype=torch.float32, device=device)
    return o_partial, lse_partial


def _check_partials(o_partial, lse_partial, num_splits, B, Hq):
    require_tensor("o_partial", o_partial, torch.float32, 4)
    require_tensor("lse_partial", lse_partial, torch.float32, 3)
    if o_partial.shape[0] < num_splits or tuple(o_partial.shape[1:]) != (B, Hq, HEAD_DIM):
        raise ValueError(f"o_partial must be [>= {num_splits}, {B}, {Hq}, {HEAD_DIM}], got {tuple(o_partial.shape)}")
    if lse_partial.shape[0] < num_splits or tuple(lse_partial.shape[1:]) != (B, Hq):
        raise ValueError(f"lse_partial must be [>= {num_splits}, {B}, {Hq}], got {tuple(lse_partial.shape)}")
    if o_partial.shape[0] != num_splits or lse_partial.shape[0] != num_splits:
        raise ValueError("o_partial / lse_partial leading dim must equal num_splits")


def dec_attn_splitkv_partial(q, k_cache, v_cache, cache_seqlens, o_partial, lse_partial,
                             num_splits: int, softmax_scale: float | None = None, stream=None) -> None:
    """Pass 1: write per-split normalised O (fp32) and natural-log LSE."""
    B, L, Hq, Hkv, D, dev = _check_attn(q, k_cache, v_cache, cache_seqlens)
    _check_partials(o_partial, lse_partial, num_splits, B, Hq)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    st = stream_for(dev, stream)
    _native.check(_native.load().fk_dec_attn_splitkv_fwd(
        ptr(q), ptr(k_cache), ptr(v_cache), ptr(cache_seqlens), ptr(o_partial), ptr(lse_partial),
        B, L, Hq, Hkv, D, num_splits, scale, st))


def dec_attn_combine(o_partial, lse_partial, cache_seqlens, out, lse, max_seqlen: int,
                     stream=None) -> None:
    """Pass 2: merge the splits of every (row, q head) into bf16 ``out`` and fp32 ``lse``."""
    require_tensor("o_partial", o_partial, torch.float32, 4)
    require_tensor("lse_partial", lse_partial, torch.float32, 3)
    require_tensor("cache_seqlens", cache_seqlens, torch.int32, 1)
    require_tensor("out", out, torch.bfloat16)
    require_tensor("lse", lse, torch.float32, 2)
    S, B, Hq, D = o_partial.shape
    require_shape("lse_partial", lse_partial, (S, B, Hq))
    if out.numel() != B * Hq * D:
        raise ValueError(f"out must hold {B}x{Hq}x{D} elements, got shape {tuple(out.shape)}")
    require_shape("lse", lse, (B, Hq))
    dev = same_device(o_partial, lse_partial, cache_seqlens, out, lse)
    st = stream_for(dev, stream)
    _native.check(_native.load().fk_dec_attn_combine(
        ptr(o_partial), ptr(lse_partial), ptr(cache_seqlens), ptr(out), ptr(lse),
        B, int(max_seqlen), Hq, D, S, st))


def alloc_counters(batch: int, num_heads_kv: int, device) -> torch.Tensor:
    """Zeroed arrival counters of the single-launch form: one int32 per (row, kv head).
    Every call leaves them zero again, so one buffer serves any number of calls
    that are ordered on the GPU."""
    return torch.zeros(batch * num_heads_kv, dtype=torch.int32, device=device)


_ctr_lock = threading.Lock()
_ctr_cache: dict = {}


def shared_counters(n: int, device, stream_handle: int) -> torch.Tensor:
    """Counters for callers that pass none: one zeroed buffer per (device, stream),
    grown on demand. Calls on one stream are ordered, so they can share it; a
    different stream gets its own buffer."""
    key = (str(device), int(stream_handle))
    with _ctr_lock:
        buf = _ctr_cache.get(key)
        if buf is None or buf.numel() < n:
            buf = torch.zeros(max(n, 1024), dtype=torch.int32, device=device)
            _ctr_cache[key] = buf
        return buf


def _vptrs(ptrs):
    arr = (ctypes.c_void_p * max(1, len(ptrs)))(*ptrs)
    return arr, len(ptrs)


def attn_fused_launch(q_ptr: int, q_batch_stride: int, k_cache, v_cache, cache_seqlens, out_ptr: int, lse,
                      o_partial, lse_partial, counters, *, batch: int, max_seqlen: int, num_heads_q: int,
                      num_heads_kv: int, num_splits: int, softmax_scale: float, stream_handle: int,
                      block_table=None, block_size: int = 0, num_blocks: int = 0, seqlens_commit=None,
                      peer_out=()) -> None:
    """Raw call of ``fk_dec_attn_fwd_fused`` (pointers and sizes already checked by the caller)."""
    peers, npeers = _vptrs(list(peer_out))
    _native.check(_native.load().fk_dec_attn_fwd_fused(
        q_ptr, q_batch_stride, ptr(k_cache), ptr(v_cache),
        ptr(block_table) if block_table is not None else None, ptr(cache_seqlens),
        ptr(seqlens_commit) if seqlens_commit is not None else None, out_ptr, peers, npeers, ptr(lse),
        ptr(o_partial), ptr(lse_partial), ptr(counters), batch, max_seqlen, block_size, num_blocks,
        num_heads_q, num_heads_kv, HEAD_DIM, num_splits, float(softmax_scale), stream_handle))


def dec_attn_splitkv_fwd(q, k_cache, v_cache, cache_seqlens, out, lse, o_partial, lse_partial,
                         num_splits: int, softmax_scale: float | None = None, stream=None, *,
                         counters=None, single_launch: bool | None = None) -> None:
    """``out = softmax(q K^T * scale) V`` per row over its first ``cache_seqlens[b]`` keys.

    ``single_launch`` (default): one kernel. Each CTA takes an equal range of
    the batch's (row, kv head, 64-token tile) sequence; the last piece of each
    (row, kv head) to finish merges the pair, through ``counters`` (int32
    ``[B * Hkv]``, zero; :func:`alloc_counters`; default: a buffer shared per
    device and stream). ``num_splits`` is then the number of partial slots per
    pair the buffers hold (>= 2, see :func:`fused_partial_slots`).
    ``single_launch=False``: pass 1 over ``num_splits`` fixed chunks, then pass 2.
    ``single_launch=None`` (default): the form :func:`plan_attention` picks for
    this shape (single launch needs ``num_splits >= 2``).
    """
    B, L, Hq, Hkv, D, dev = _check_attn(q, k_cache, v_cache, cache_seqlens)
    _check_partials(o_partial, lse_partial, num_splits, B, Hq)
    require_tensor("out", out, torch.bfloat16)
    require_tensor("lse", lse, torch.float32, 2)
    if out.numel() != B * Hq * D:
        raise ValueError(f"out must hold {B}x{Hq}x{D} elements, got shape {tuple(out.shape)}")
    require_shape("lse", lse, (B, Hq))
    same_device(q, out, lse, o_partial, lse_partial)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    st = stream_for(dev, stream)
    if single_launch is None:
        single_launch = num_splits >= 2 and plan_attention(B, Hkv, L)[0]
    if not single_launch:
        _native.check(_native.load().fk_dec_attn_fwd(
            ptr(q), ptr(k_cache), ptr(v_cache), ptr(cache_seqlens), ptr(out), ptr(lse),
            ptr(o_partial), ptr(lse_partial), B, L, Hq, Hkv, D, num_splits, scale, st))
        return
    if counters is None:
        counters = shared_counters(B * Hkv, dev, st)
    else:
        require_tensor("counters", counters, torch.int32, 1)
        if counters.numel() < B * Hkv:
            raise ValueError(f"counters must hold >= {B * Hkv} entries, got {counters.numel()}")
        same_device(q, counters)
    attn_fused_launch(ptr(q), Hq * D, k_cache, v_cache, cache_seqlens, ptr(out), lse, o_partial, lse_partial,
                      counters, batch=B, max_seqlen=L, num_heads_q=Hq, num_heads_kv=Hkv, num_splits=num_splits,
                      softmax_scale=scale, stream_handle=st)


class DecodeAttention:
    """Kernel object in the reference's style (cf. ``DAttn1(...)`` then a call).

    ``DecodeAttention(num_splits=None)(q, k_cache, v_cache, cache_seqlens, out, lse,
    softmax_scale)`` runs decode attention in the form :func:`plan_attention`
    picks for the shape, writing ``out``/``lse`` in place and returning ``None``.
    Partials and counters are allocated once per (shape, device) and reused;
    ``num_splits`` pins the split count (two-launch) or partial slots (single launch).
    """

    def __init__(self, num_splits: int | None = None):
        self.num_splits = num_splits
        self._ws: dict = {}

    def plan(self, batch: int, num_heads_kv: int, max_seqlen: int) -> tuple[bool, int]:
        single, S = plan_attention(batch, num_heads_kv, max_seqlen)
        if self.num_splits is not None:
            S = int(self.num_splits)
            single = single and S >= 2
        return single, S

    def workspace(self, batch, num_heads_q, num_heads_kv, num_splits, device):
        key = (batch, num_heads_q, num_heads_kv, num_splits, str(device))
        ws = self._ws.get(key)
        if ws is None:
            ws = alloc_partials(batch, num_heads_q, num_splits, device) + (
                alloc_counters(batch, num_heads_kv, device),)
            self._ws[key] = ws
        return ws

    def __call__(self, q, k_cache, v_cache, cache_seqlens, out, lse, softmax_scale=None,
                 stream=None) -> None:
        B, L, Hq, Hkv, D, dev = _check_attn(q, k_cache, v_cache, cache_seqlens)
        single, S = self.plan(B, Hkv, L)
        o_p, l_p, ctr = self.workspace(B, Hq, Hkv, S, dev)
        dec_attn_splitkv_fwd(q, k_cache, v_cache, cache_seqlens, out, lse, o_p, l_p, S,
                             softmax_scale, stream, counters=ctr, single_launch=single)


def decode_attention(q, k_cache, v_cache, cache_seqlens, softmax_scale=None, num_splits=None):
    """Functional convenience: allocates ``out``/``lse``/partials, returns ``(out, lse)``."""
    B, L, Hq, Hkv, D, dev = _check_attn(q, k_cache, v_cache, cache_seqlens)
    single, S = plan_attention(B, Hkv, L)
    if num_splits is not None:
        S = num_splits
        single = single and S >= 2
    out = torch.empty((B, 1, Hq, D), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((B, Hq), dtype=torch.float32, device=dev)
    o_p, l_p = alloc_partials(B, Hq, S, dev)
    dec_attn_splitkv_fwd(q, k_cache, v_cache, cache_seqlens, out, lse, o_p, l_p, S, softmax_scale,
                         single_launch=single)
    return out, lse


class DAttn1:
    """The reference's decode-attention kernel object, same constructor and call.

    ``DAttn1(qk_mnk=(16, 128, 128), stages=2, p_stages=1, is_persistent=True)(Q, K, V, O, softmax_scale)``
    computes ``O[h] = (Q[h] @ K[h]^T) @ V[h]`` with the scores rounded to bf16
    and no softmax, exactly as python/cutedsl_kernels/decoding_attention/attn1.py:204-251
    does (and as its check demo/dec_attn_second_part.py:33-34 expects). Q is
    [H, M<=16, 128], K [H, P, 128], V is given transposed as [H, 128, P], O is
    [H, M, 128]; all bf16. ``softmax_scale`` is accepted and, as in the
    reference, not applied. The tuning arguments describe Hopper tiles and are
    ignored. For softmax decode attention over a KV cache use
    :class:`DecodeAttention`.
    """

    def __init__(self, qk_mnk=(16, 128, 128), stages: int = 2, p_stages: int = 1, is_persistent: bool = True):
        self.qk_mnk = tuple(qk_mnk)

    def __call__(self, Q, K, V, O, softmax_scale=1.0, stream=None):
        require_tensor("Q", Q, torch.bfloat16, 3)
        require_tensor("K", K, torch.bfloat16, 3)
        require_tensor("V", V, torch.bfloat16, 3)
        require_tensor("O", O, torch.bfloat16, 3)
        H, M, D = Q.shape
        P = K.shape[1]
        require_shape("K", K, (H, P, D))
        require_shape("V", V, (H, D, P))
        require_shape("O", O, (H, M, D))
        dev = same_device(Q, K, V, O)
        st = stream_for(dev, stream)
        _native.check(_native.load().fk_dattn1(ptr(Q), ptr(K), ptr(V), ptr(O), H, M, P, D, st))


class DAttn2:
    """The reference's fused QKV projection + KV-cache write, same constructor and call.

    ``DAttn2(qkw_mnk, stg1_stages, persistent)(X, Wq, Wk, Wv, Q_out, K_cache, V_cache)``
    (python/cutedsl_kernels/decoding_attention/attempt2.py:77-99): with X [M, H*D]
    and W* [H*D, H*D] (row = output feature), writes ``Q_out[h] = (X Wq^T)[:, h]``
    as [H, M, D] and the new K/V rows into ``K_cache/V_cache[h, P-M:P]`` of the
    [H, P, D] caches, the layout of its check demo/dec_attn_run.py:51-63. Runs as
    three weight-streaming GEMMs (x is M <= 16 tokens) and one head-major
    scatter; the Hopper tuning arguments are ignored.
    """

    def __init__(self, qkw_mnk=(16, 128, 64), stg1_stages: int = 2, persistent: bool = False):
        self.qkw_mnk = tuple(qkw_mnk)
        self._tmp: dict = {}

    def __call__(self, X, Wq, Wk, Wv, Q_out, K_cache, V_cache, stream=None):
        from .gemm import linear

        require_tensor("X", X, torch.bfloat16, 2)
        require_tensor("Q_out", Q_out, torch.bfloat16, 3)
        require_tensor("K_cache", K_cache, torch.bfloat16, 3)
        require_tensor("V_cache", V_cache, torch.bfloat16, 3)
        M, HD = X.shape
        H, _, D = Q_out.shape
        P = K_cache.shape[1]
        require_shape("Q_out", Q_out, (H, M, D))
        require_shape("K_cache", K_cache, (H, P, D))
        require_shape("V_cache", V_cache, (H, P, D))
        if H * D != HD:
            raise ValueError(f"X has {HD} features but Q_out is [{H}, {M}, {D}]")
        if P < M:
            raise ValueError("cache length must be >= M")
        dev = same_device(X, Wq, Wk, Wv, Q_out, K_cache, V_cache)
        key = (M, HD, str(dev))
        tmp = self._tmp.get(key)
        if tmp is None:
            tmp = torch.empty(3, M, HD, dtype=torch.bfloat16, device=dev)
            self._tmp[key] = tmp
        for i, w in enumerate((Wq, Wk, Wv)):
            linear(X, w, tmp[i], stream=stream)
        st = stream_for(dev, stream)
        _native.check(_native.load().fk_qkv_head_scatter(
            ptr(tmp[0]), ptr(tmp[1]), ptr(tmp[2]), ptr(Q_out), ptr(K_cache), ptr(V_cache), M, H, D, P, st))


def dec_attn_paged_fwd(q, k_pool, v_pool, block_table, cache_seqlens, out, lse, o_partial, lse_partial,
                       num_splits: int, softmax_scale: float | None = None, stream=None, *,
                       single_launch: bool | None = None) -> None:
    """Split-KV decode attention over a paged KV cache (both passes).

    ``k_pool``/``v_pool``: [num_blocks, block_size, Hkv, 128] bf16 with
    ``block_size % 64 == 0``; ``block_table``: [B, max_blocks] int32, logical
    block j of row b at physical block ``block_table[b, j]``. Splits follow
    ``max_seqlen = max_blocks * block_size`` (``chunk_tokens``). Same outputs
    as :func:`dec_attn_splitkv_fwd` on the equivalent contiguous cache.
    """
    require_tensor("q", q, torch.bfloat16)
    require_tensor("k_pool", k_pool, torch.bfloat16, 4)
    require_tensor("v_pool", v_pool, torch.bfloat16, 4)
    require_tensor("block_table", block_table, torch.int32, 2)
    require_tensor("cache_seqlens", cache_seqlens, torch.int32, 1)
    NB, BS, Hkv, D = k_pool.shape
    require_shape("v_pool", v_pool, (NB, BS, Hkv, D))
    B, MB = block_table.shape
    Hq = q.shape[-2]
    if q.numel() != B * Hq * D or D != HEAD_DIM:
        raise ValueError(f"q must be [B, 1, Hq, {HEAD_DIM}] with B={B}")
    require_shape("cache_seqlens", cache_seqlens, (B,))
    _check_partials(o_partial, lse_partial, num_splits, B, Hq)
    require_tensor("out", out, torch.bfloat16)
    require_tensor("lse", lse, torch.float32, 2)
    dev = same_device(q, k_pool, v_pool, block_table, cache_seqlens, out, lse, o_partial, lse_partial)
    scale = 1.0 / math.sqrt(D) if softmax_scale is None else float(softmax_scale)
    st = stream_for(dev, stream)
    if single_launch is None:
        single_launch = num_splits >= 2 and plan_attention(B, Hkv, MB * BS)[0]
    if not single_launch:
        _native.check(_native.load().fk_dec_attn_fwd_paged(
            ptr(q), ptr(k_pool), ptr(v_pool), ptr(block_table), ptr(cache_seqlens), ptr(out), ptr(lse),
            ptr(o_partial), ptr(lse_partial), B, MB, BS, NB, Hq, Hkv, D, num_splits, scale, st))
        return
    counters = shared_counters(B * Hkv, dev, st)
    attn_fused_launch(ptr(q), Hq * D, k_pool, v_pool, cache_seqlens, ptr(out), lse, o_partial, lse_partial,
                      counters, batch=B, max_seqlen=MB * BS, num_heads_q=Hq, num_heads_kv=Hkv,
                      num_splits=num_splits, softmax_scale=scale, stream_handle=st, block_table=block_table,
                      block_size=BS, num_blocks=NB)
