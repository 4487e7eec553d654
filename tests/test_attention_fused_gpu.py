"""Single-launch decode attention (the split merge folded into the one kernel) on the GPU.

The single-launch form must give the oracle's values within the decode
tolerances and agree with the two-launch form within them, give the same bits
on repeated calls and across the contiguous and paged caches, leave its arrival
counters at zero, and honour the commit / paged / strided-q variants. A starved
pipeline must end every consumer warp with a device error instead of a hang.
"""
import math

import pytest
import torch

import oracle
from fused_kernels_cutedsl_lib_b200 import (
    _native,
    alloc_counters,
    alloc_partials,
    configs,
    dec_attn_splitkv_fwd,
    default_num_splits,
    fused_partial_slots,
)
from fused_kernels_cutedsl_lib_b200.decoding_attention import attn_fused_launch, dec_attn_paged_fwd

from test_attention_gpu import assert_attn_close

pytestmark = pytest.mark.gpu


def _run(q, k, v, lens, S, single, ctr=None, scale=None):
    B, L, Hkv, D = k.shape
    Hq = q.shape[2]
    out = torch.full((B, 1, Hq, D), float("nan"), dtype=torch.bfloat16, device=q.device)
    lse = torch.full((B, Hq), float("nan"), dtype=torch.float32, device=q.device)
    o_p, l_p = alloc_partials(B, Hq, S, q.device)
    o_p.fill_(float("nan"))
    l_p.fill_(float("nan"))
    dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S, scale, single_launch=single, counters=ctr)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    return out, lse


def _both(q, k, v, lens, S_two, S_one=None, scale=None):
    """(two-launch out, lse), (single-launch out, lse), counters after the call."""
    B, L, Hkv, D = k.shape
    S_one = S_one if S_one is not None else fused_partial_slots(B, Hkv, L)
    ctr = alloc_counters(B, Hkv, q.device)
    two = _run(q, k, v, lens, S_two, False, scale=scale)
    one = _run(q, k, v, lens, S_one, True, ctr=ctr, scale=scale)
    return two, one, ctr


def _same(a, b):
    assert torch.equal(a[0], b[0]), (a[0].float() - b[0].float()).abs().max()
    # bitwise, -inf included
    assert torch.equal(a[1].view(torch.int32), b[1].view(torch.int32))


def _close(a, b):
    """Two kernel results that merge different split boundaries: bf16 rounding apart."""
    assert (a[0].float() - b[0].float()).abs().max().item() <= 1e-2
    fin = torch.isfinite(a[1])
    assert torch.equal(fin, torch.isfinite(b[1]))
    if fin.any():
        assert (a[1][fin] - b[1][fin]).abs().max().item() <= 1e-4


@pytest.mark.parametrize("name", ["attn_gqa4_ragged", "attn_gqa8", "attn_mha"])
@pytest.mark.parametrize("num_splits", [1, 2, 3, 8, 40])
def test_single_launch_equals_two_launch_golden(golden, name, num_splits):
    g = golden(name)
    q, k, v, lens = (g[x].cuda() for x in ("q", "k_cache", "v_cache", "cache_seqlens"))
    B, L, Hkv = k.shape[0], k.shape[1], k.shape[2]
    two, one, ctr = _both(q, k, v, lens, num_splits, S_one=max(2, num_splits))
    _close(two, one)
    assert_attn_close(one[0], one[1], g["out"], g["lse"])
    assert int(ctr.abs().sum()) == 0
    again = _run(q, k, v, lens, max(2, num_splits), True, ctr=ctr)
    _same(one, again)


def test_single_launch_config1_splits_and_counters_reused():
    cfg = configs.ATTN_CONFIG1
    q, k, v, lens = configs.attn_inputs(cfg)
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    for S in (2, 4, 8, 16, 65):  # partial slots: fewer slots -> longer ranges, fewer CTAs
        two, one, ctr = _both(q, k, v, lens, 8, S_one=S)
        _close(two, one)
        assert_attn_close(one[0], one[1], ref_out, ref_lse)
        assert int(ctr.abs().sum()) == 0
    # the same counters through many calls in a row stay consistent
    B, Hq = cfg.batch, cfg.num_heads_q
    ctr = alloc_counters(B, cfg.num_heads_kv, "cuda")
    S = fused_partial_slots(B, cfg.num_heads_kv, cfg.max_seqlen)
    o_p, l_p = alloc_partials(B, Hq, S, "cuda")
    outs = []
    for _ in range(5):
        out = torch.empty(B, 1, Hq, 128, dtype=torch.bfloat16, device="cuda")
        lse = torch.empty(B, Hq, device="cuda")
        dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S, counters=ctr)
        outs.append(out)
    torch.cuda.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])
    assert int(ctr.abs().sum()) == 0


def test_single_launch_nan_padding_edge_lengths_and_clamp():
    torch.manual_seed(7)
    B, L, Hq, Hkv = 14, 1000, 16, 4
    lens = torch.tensor([0, 1, 63, 64, 65, 127, 128, 129, 511, 999, 1000, 333, 0, 1500], dtype=torch.int32)
    q = torch.randn(B, 1, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    for b in range(B):
        k[b, min(int(lens[b]), L):] = float("nan")
        v[b, min(int(lens[b]), L):] = float("nan")
    lens = lens.cuda()
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    for S in (2, 4, 16):
        two, one, _ = _both(q, k, v, lens, S, S_one=S)
        _close(two, one)
        assert torch.isfinite(one[0].float()).all()
        assert_attn_close(one[0], one[1], ref_out, ref_lse)
        assert torch.all(one[0][0] == 0) and torch.all(torch.isneginf(one[1][0]))


def test_single_launch_commit_strided_q_and_paged():
    """The layer's variants: q read at a row stride out of a QKV buffer, lengths
    published to a second array, and a paged cache; all equal to the two-launch entries."""
    from fused_kernels_cutedsl_lib_b200.layer import attention_commit

    torch.manual_seed(9)
    B, Hq, Hkv, bs, MB = 6, 32, 8, 64, 9
    L = bs * MB
    qkv = torch.randn(B, (Hq + 2 * Hkv) * 128, device="cuda").bfloat16()
    NB = B * MB + 3
    perm = torch.randperm(NB)[: B * MB].view(B, MB).to(torch.int32).cuda()
    k_pool = torch.randn(NB, bs, Hkv, 128, device="cuda").bfloat16()
    v_pool = torch.randn(NB, bs, Hkv, 128, device="cuda").bfloat16()
    lens = torch.tensor([L, 1, 0, 65, L - 7, 300], dtype=torch.int32, device="cuda")
    results = []
    for single in (False, True):
        for paged in (False, True):
            S = 4
            out = torch.full((B, Hq * 128), float("nan"), dtype=torch.bfloat16, device="cuda")
            lse = torch.empty(B, Hq, device="cuda")
            o_p, l_p = alloc_partials(B, Hq, S, "cuda")
            commit = torch.full((B,), -7, dtype=torch.int32, device="cuda")
            if paged:
                kc, vc, bt = k_pool, v_pool, perm
            else:
                flat = perm.long().view(-1)
                kc = k_pool[flat].view(B, L, Hkv, 128).contiguous()
                vc = v_pool[flat].view(B, L, Hkv, 128).contiguous()
                bt = None
            attention_commit(qkv, kc, vc, lens, commit, out, lse, o_p, l_p, S, Hq, Hkv, block_table=bt,
                             single_launch=single)
            torch.cuda.synchronize()
            assert _native.device_error() == 0
            assert torch.equal(commit, lens)
            results.append((out, lse))
    _same(results[0], results[1])  # two-launch: contiguous == paged
    _same(results[2], results[3])  # single-launch: contiguous == paged
    _close(results[0], results[2])
    flat = perm.long().view(-1)
    k = k_pool[flat].view(B, L, Hkv, 128)
    v = v_pool[flat].view(B, L, Hkv, 128)
    ref_out, ref_lse = oracle.decode_attention(qkv[:, :Hq * 128].reshape(B, 1, Hq, 128), k, v, lens)
    assert_attn_close(results[-1][0], results[-1][1], ref_out, ref_lse)
    # the paged Python entry point has the single-launch form too
    out = torch.empty(B, 1, Hq, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, device="cuda")
    o_p, l_p = alloc_partials(B, Hq, 4, "cuda")
    dec_attn_paged_fwd(qkv[:, :Hq * 128].contiguous().view(B, 1, Hq, 128), k_pool, v_pool, perm, lens, out, lse,
                       o_p, l_p, 4, single_launch=True)
    torch.cuda.synchronize()
    assert torch.equal(out.view(B, -1), results[-1][0])


def test_config2_every_row_against_oracle():
    """Full BASELINE config 2 (B=64, Lmax=32768, ragged): every row vs the oracle,
    single-launch form, and within bf16 rounding of the two-launch form."""
    cfg = configs.ATTN_CONFIG2
    q, k, v, lens = configs.attn_inputs(cfg)
    S = default_num_splits(cfg.batch, cfg.num_heads_kv, cfg.max_seqlen, int(lens.sum()))
    two, one, ctr = _both(q, k, v, lens, S)
    _close(two, one)
    assert int(ctr.abs().sum()) == 0
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    assert_attn_close(one[0], one[1], ref_out, ref_lse)
    del k, v
    torch.cuda.empty_cache()


def test_starved_pipeline_times_out_in_every_consumer_warp():
    """CTA 0's producer withholds one stage. Every consumer warp of that CTA must
    leave its wait (one by its own bound, the others through the shared abort
    flag), meet at the merge barrier and return: the launch completes with the
    device error word set, and the context stays usable."""
    lib = _native.load()
    torch.manual_seed(1)
    B, L, Hq, Hkv = 2, 2048, 32, 8
    q = torch.randn(B, 1, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    S = 4
    out = torch.empty(B, 1, Hq, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, device="cuda")
    o_p, l_p = alloc_partials(B, Hq, S, "cuda")
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    ctr = alloc_counters(B, Hkv, "cuda")
    _native.check(lib.fk_set_wait_limit_ns(2_000_000))  # 2 ms
    try:
        for single in (False, True):
            _native.check(lib.fk_debug_attn_withhold_tile(1))
            try:
                dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S, single_launch=single, counters=ctr)
                torch.cuda.synchronize()  # returns: no warp is left blocked at a barrier
            finally:
                _native.check(lib.fk_debug_attn_withhold_tile(-1))
            code = _native.device_error(clear=True)
            assert code in (1, 2), code  # a stage wait ran out (consumer: 1, producer: 2)
    finally:
        _native.check(lib.fk_set_wait_limit_ns(0))
    # the context is still usable and the next call is correct (an aborted
    # single-launch call leaves its counters mid-count: they are zeroed again)
    ctr.zero_()
    dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S, counters=ctr)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    assert_attn_close(out, lse, ref_out, ref_lse)


def test_tvm_ffi_single_launch_entries_match_python():
    pytest.importorskip("tvm_ffi")
    from fused_kernels_cutedsl_lib_b200 import tvm_ffi_module

    mod = tvm_ffi_module.load()
    torch.manual_seed(4)
    B, L, Hq, Hkv, bs = 3, 512, 32, 8, 64
    q = torch.randn(B, 1, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    lens = torch.tensor([512, 100, 0], dtype=torch.int32, device="cuda")
    S = 5
    ref = _run(q, k, v, lens, S, True, ctr=alloc_counters(B, Hkv, "cuda"))
    out = torch.empty(B, 1, Hq, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, device="cuda")
    o_p, l_p = alloc_partials(B, Hq, S, "cuda")
    ctr = alloc_counters(B, Hkv, "cuda")
    mod.dec_attn_fused(q, k, v, lens, out, lse, o_p, l_p, ctr, 0.0)
    torch.cuda.synchronize()
    _same(ref, (out, lse))
    # paged: identity block table over the same cache
    table = torch.arange(B * (L // bs), dtype=torch.int32, device="cuda").view(B, L // bs)
    kp, vp = k.view(-1, bs, Hkv, 128), v.view(-1, bs, Hkv, 128)
    out2 = torch.empty_like(out)
    mod.dec_attn_paged(q, kp, vp, table, lens, out2, lse, o_p, l_p, ctr, 0.0)
    torch.cuda.synchronize()
    assert torch.equal(out2, out)
    assert int(ctr.abs().sum()) == 0
