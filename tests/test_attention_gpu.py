"""Parity of the split-KV decode attention kernels against the CPU oracle (GPU)."""
import math

import pytest
import torch

import oracle
from fused_kernels_cutedsl_lib_b200 import (
    DecodeAttention,
    _native,
    alloc_partials,
    chunk_tokens,
    dec_attn_combine,
    dec_attn_splitkv_fwd,
    dec_attn_splitkv_partial,
    decode_attention,
)
from fused_kernels_cutedsl_lib_b200 import configs

pytestmark = pytest.mark.gpu

# Tolerances of the decode path: bf16 outputs vs an fp32 reference.
MAX_ABS = 2e-2
MEAN_ABS = 2e-3
LSE_ABS = 1e-3


def assert_attn_close(out, lse, ref_out, ref_lse, rows=None):
    out = out.float().cpu().reshape(ref_out.shape[0] if rows is None else len(rows), -1, 128)
    lse = lse.float().cpu()
    if rows is not None:
        out, lse = out, lse
    err = (out - ref_out).abs()
    assert err.max().item() <= MAX_ABS, f"max abs {err.max().item()}"
    assert err.mean().item() <= MEAN_ABS, f"mean abs {err.mean().item()}"
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), fin)
    assert torch.all(torch.isneginf(lse[~fin]))
    if fin.any():
        lerr = (lse[fin] - ref_lse[fin]).abs().max().item()
        assert lerr <= LSE_ABS, f"lse abs {lerr}"


def run(q, k, v, lens, num_splits, scale=None):
    B, L, Hkv, D = k.shape
    Hq = q.shape[2]
    out = torch.full((B, 1, Hq, D), float("nan"), dtype=torch.bfloat16, device=q.device)
    lse = torch.full((B, Hq), float("nan"), dtype=torch.float32, device=q.device)
    o_p, l_p = alloc_partials(B, Hq, num_splits, q.device)
    o_p.fill_(float("nan"))
    l_p.fill_(float("nan"))
    # the two-launch form: pass 1 over num_splits fixed chunks, pass 2
    dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, num_splits, scale, single_launch=False)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    return out, lse


@pytest.mark.parametrize("name", ["attn_gqa4_ragged", "attn_gqa8", "attn_mha"])
@pytest.mark.parametrize("num_splits", [1, 2, 3, 8])
def test_golden(golden, name, num_splits):
    g = golden(name)
    q, k, v, lens = (g[x].cuda() for x in ("q", "k_cache", "v_cache", "cache_seqlens"))
    out, lse = run(q, k, v, lens, num_splits)
    assert_attn_close(out, lse, g["out"], g["lse"])


def test_config1_contiguous():
    cfg = configs.ATTN_CONFIG1
    q, k, v, lens = configs.attn_inputs(cfg)
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    for s in (1, 16, 64):
        out, lse = run(q, k, v, lens, s)
        assert_attn_close(out, lse, ref_out, ref_lse)


def test_ragged_with_nan_padding_and_edge_lengths():
    torch.manual_seed(7)
    B, L, Hq, Hkv = 12, 1000, 16, 4
    lens = torch.tensor([0, 1, 63, 64, 65, 127, 128, 129, 511, 999, 1000, 333], dtype=torch.int32)
    q = torch.randn(B, 1, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    for b in range(B):  # padding past each row's length is NaN: it must never leak
        k[b, lens[b]:] = float("nan")
        v[b, lens[b]:] = float("nan")
    lens = lens.cuda()
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    for s in (1, 4, 16):
        out, lse = run(q, k, v, lens, s)
        assert torch.isfinite(out.float()).all()
        assert_attn_close(out, lse, ref_out, ref_lse)
    assert torch.all(out[0] == 0)


def test_lengths_beyond_cache_are_clamped():
    torch.manual_seed(3)
    B, L = 3, 200
    q = torch.randn(B, 1, 8, 128, device="cuda").bfloat16()
    k = torch.randn(B, L, 2, 128, device="cuda").bfloat16()
    v = torch.randn(B, L, 2, 128, device="cuda").bfloat16()
    lens = torch.tensor([500, -4, 150], dtype=torch.int32, device="cuda")
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    out, lse = run(q, k, v, lens, 3)
    assert_attn_close(out, lse, ref_out, ref_lse)


def test_two_pass_api_and_custom_scale():
    torch.manual_seed(11)
    B, L, Hq, Hkv = 5, 700, 32, 8
    q = torch.randn(B, 1, Hq, 128, device="cuda").bfloat16()
    k = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    v = torch.randn(B, L, Hkv, 128, device="cuda").bfloat16()
    lens = torch.tensor([700, 10, 300, 650, 64], dtype=torch.int32, device="cuda")
    S = 6
    o_p, l_p = alloc_partials(B, Hq, S, "cuda")
    out = torch.empty(B, 1, Hq, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, device="cuda")
    dec_attn_splitkv_partial(q, k, v, lens, o_p, l_p, S, softmax_scale=0.05)
    dec_attn_combine(o_p, l_p, lens, out, lse, max_seqlen=L)
    torch.cuda.synchronize()
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens, softmax_scale=0.05)
    assert_attn_close(out, lse, ref_out, ref_lse)
    # the per-split partials are themselves attention over each split's tokens
    c = chunk_tokens(L, S)
    b, s = 3, 2
    lo, hi = s * c, min((s + 1) * c, int(lens[b]))
    kk = k[b:b + 1].clone()
    po, plse = oracle.decode_attention(q[b:b + 1], k[b:b + 1, lo:hi], v[b:b + 1, lo:hi],
                                       torch.tensor([hi - lo], dtype=torch.int32), softmax_scale=0.05)
    assert (o_p[s, b].cpu() - po[0]).abs().max().item() < 1e-2
    assert (l_p[s, b].cpu() - plse[0]).abs().max().item() < LSE_ABS
    del kk


def test_kernel_object_and_stream():
    torch.manual_seed(5)
    q = torch.randn(2, 1, 32, 128, device="cuda").bfloat16()
    k = torch.randn(2, 4096, 8, 128, device="cuda").bfloat16()
    v = torch.randn(2, 4096, 8, 128, device="cuda").bfloat16()
    lens = torch.tensor([4096, 1234], dtype=torch.int32, device="cuda")
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    attn = DecodeAttention()
    out = torch.empty(2, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(2, 32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        attn(q, k, v, lens, out, lse)
    s.synchronize()
    assert_attn_close(out, lse, ref_out, ref_lse)
    out2, lse2 = decode_attention(q, k, v, lens)
    torch.cuda.synchronize()
    assert torch.equal(out2, out) or (out2.float() - out.float()).abs().max() < 1e-2


def test_deterministic():
    cfg = configs.ATTN_CONFIG1
    q, k, v, lens = configs.attn_inputs(cfg)
    a = run(q, k, v, lens, 16)
    b = run(q, k, v, lens, 16)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_config2_ragged_full_size():
    """Full BASELINE size: every row checked against the oracle on a sample of rows."""
    cfg = configs.ATTN_CONFIG2
    q, k, v, lens = configs.attn_inputs(cfg)
    from fused_kernels_cutedsl_lib_b200 import default_num_splits

    S = default_num_splits(cfg.batch, cfg.num_heads_kv, cfg.max_seqlen, int(lens.sum()))
    out, lse = run(q, k, v, lens, S)
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()
    rows = [0, 7, 31, 63] + [int(torch.argmin(lens)), int(torch.argmax(lens))]
    for r in rows:
        ro, rl = oracle.decode_attention(q[r:r + 1], k[r:r + 1], v[r:r + 1], lens[r:r + 1])
        assert_attn_close(out[r:r + 1], lse[r:r + 1], ro, rl)
    del k, v
    torch.cuda.empty_cache()


def _normwise(out, ref):
    out, ref = out.float().cpu(), ref.float().cpu()
    return ((out - ref).abs().max() / ref.abs().max()).item()


def test_dattn1_reference_semantics(golden):
    """DAttn1's (Q K^T) V^T with bf16 scores: golden fixture from the reference's check, and the demo shape.

    Scores reach ~|11| and sums over P tokens reach hundreds, so the bound is
    normwise: max |out - ref| / max |ref| <= 1e-2 (bf16 scores and output).
    """
    from fused_kernels_cutedsl_lib_b200 import DAttn1, compile_cutedsl

    g = golden("dattn1")
    Q, K, V = g["Q"].cuda(), g["K"].cuda(), g["V"].cuda()
    O = torch.empty_like(Q)
    DAttn1(qk_mnk=(16, 128, 128), stages=2, p_stages=1, is_persistent=True)(Q, K, V, O, 1.0)
    torch.cuda.synchronize()
    assert _normwise(O, g["O"]) <= 1e-2
    torch.manual_seed(42)  # the reference demo's shape: H=128 heads, M=16, P=1024
    Q = torch.randn(128, 16, 128, device="cuda").bfloat16()
    K = torch.randn(128, 1024, 128, device="cuda").bfloat16()
    V = torch.randn(128, 128, 1024, device="cuda").bfloat16()
    O = torch.empty(128, 16, 128, dtype=torch.bfloat16, device="cuda")
    f = compile_cutedsl((Q, K, V, O, 1.0), DAttn1((16, 128, 128), 2, 1, True), False)
    f(Q, K, V, O, 1.0)
    torch.cuda.synchronize()
    assert _normwise(O, oracle.dattn1_reference(Q, K, V)) <= 1e-2
    # ragged P (multiple of 8, not of 16) and fewer query rows
    Q2, K2, V2 = Q[:3, :5].contiguous(), K[:3, :200].contiguous(), V[:3, :, :200].contiguous()
    O2 = torch.empty(3, 5, 128, dtype=torch.bfloat16, device="cuda")
    DAttn1()(Q2, K2, V2, O2)
    torch.cuda.synchronize()
    assert _normwise(O2, oracle.dattn1_reference(Q2, K2, V2)) <= 1e-2


def test_dattn2_qkv_projection_and_cache_write():
    """DAttn2 against the layout of its reference check: X @ [WQ^T WK^T WV^T], chunk, view, transpose."""
    from fused_kernels_cutedsl_lib_b200 import DAttn2

    torch.manual_seed(42)
    M, H, D, P = 16, 32, 128, 1024
    X = torch.randn(M, H * D, device="cuda").bfloat16()
    Ws = [(torch.randn(H * D, H * D, device="cuda") * 0.02).bfloat16() for _ in range(3)]
    Q_out = torch.zeros(H, M, D, dtype=torch.bfloat16, device="cuda")
    Kc = torch.zeros(H, P, D, dtype=torch.bfloat16, device="cuda")
    Vc = torch.zeros(H, P, D, dtype=torch.bfloat16, device="cuda")
    DAttn2((16, 128, 64), 2, False)(X, *Ws, Q_out, Kc, Vc)
    torch.cuda.synchronize()
    qkv = torch.cat([oracle.linear(X, w) for w in Ws], dim=1)  # [M, 3*H*D]
    q, k, v = (t.view(M, H, D).transpose(0, 1) for t in qkv.chunk(3, dim=-1))
    for got, ref in ((Q_out, q), (Kc[:, P - M:], k), (Vc[:, P - M:], v)):
        e = (got.float().cpu() - ref).abs() / ref.abs().clamp_min(1.0)
        assert e.max().item() <= 2e-2 and e.mean().item() <= 2e-3
    assert torch.all(Kc[:, :P - M] == 0) and torch.all(Vc[:, :P - M] == 0)


@pytest.mark.parametrize("block_size", [64, 256])
def test_paged_kv_cache_matches_contiguous(block_size):
    """Paged attention over a shuffled block pool equals contiguous attention on the gathered cache."""
    from fused_kernels_cutedsl_lib_b200.decoding_attention import dec_attn_paged_fwd
    from fused_kernels_cutedsl_lib_b200.layer import kv_append_paged

    torch.manual_seed(21)
    B, Hq, Hkv, MB = 6, 32, 8, 12
    L = MB * block_size
    lens = torch.tensor([L, 1, 0, 65, L - 7, 300], dtype=torch.int32)
    NB = B * MB + 5
    perm = torch.randperm(NB)[: B * MB].view(B, MB).to(torch.int32)
    k_pool = torch.randn(NB, block_size, Hkv, 128, device="cuda").bfloat16()
    v_pool = torch.randn(NB, block_size, Hkv, 128, device="cuda").bfloat16()
    q = torch.randn(B, 1, Hq, 128, device="cuda").bfloat16()
    table = perm.cuda()
    flat = perm.long().view(-1)
    k = k_pool[flat].view(B, MB * block_size, Hkv, 128).contiguous()
    v = v_pool[flat].view(B, MB * block_size, Hkv, 128).contiguous()
    S = 5
    outs = []
    for paged in (False, True):
        out = torch.full((B, 1, Hq, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
        lse = torch.empty(B, Hq, device="cuda")
        o_p, l_p = alloc_partials(B, Hq, S, "cuda")
        if paged:
            dec_attn_paged_fwd(q, k_pool, v_pool, table, lens.cuda(), out, lse, o_p, l_p, S)
        else:
            dec_attn_splitkv_fwd(q, k, v, lens.cuda(), out, lse, o_p, l_p, S)
        torch.cuda.synchronize()
        outs.append((out, lse))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    ref_out, ref_lse = oracle.decode_attention(q, k, v, lens)
    assert_attn_close(outs[1][0], outs[1][1], ref_out, ref_lse)
    # paged append: the new rows land at (block_table[b][len // bs], len % bs)
    qkv = torch.randn(B, (Hq + 2 * Hkv) * 128, device="cuda").bfloat16()
    lens_d = torch.tensor([5, 0, 64, block_size, 17, L - 1], dtype=torch.int32, device="cuda")
    before = lens_d.clone().cpu()
    kv_append_paged(qkv, k_pool, v_pool, table, lens_d, Hq, Hkv)
    torch.cuda.synchronize()
    for b in range(B):
        pos = int(before[b])
        blk = int(perm[b, pos // block_size])
        got = k_pool[blk, pos % block_size].reshape(-1)
        assert torch.equal(got, qkv[b, Hq * 128:(Hq + Hkv) * 128])
        assert torch.equal(v_pool[blk, pos % block_size].reshape(-1), qkv[b, (Hq + Hkv) * 128:])
    assert lens_d.cpu().tolist() == (before + 1).tolist()


def test_tvm_ffi_dattn2_matches_python_class():
    """The TVM-FFI ``dattn2`` export (DAttn2's call plus scratch) equals the Python DAttn2 bit for bit."""
    pytest.importorskip("tvm_ffi")
    from fused_kernels_cutedsl_lib_b200 import DAttn2, alloc_workspace, tvm_ffi_module, workspace_bytes

    mod = tvm_ffi_module.load()
    torch.manual_seed(7)
    M, H, D, P = 8, 8, 128, 96
    X = torch.randn(M, H * D, device="cuda").bfloat16()
    Ws = [(torch.randn(H * D, H * D, device="cuda") * 0.02).bfloat16() for _ in range(3)]
    outs = []
    for use_tvm in (False, True):
        Q_out = torch.zeros(H, M, D, dtype=torch.bfloat16, device="cuda")
        Kc = torch.zeros(H, P, D, dtype=torch.bfloat16, device="cuda")
        Vc = torch.zeros(H, P, D, dtype=torch.bfloat16, device="cuda")
        if use_tvm:
            tmp = torch.empty(3, M, H * D, dtype=torch.bfloat16, device="cuda")
            ws = alloc_workspace(workspace_bytes(M, H * D, H * D), "cuda")
            mod.dattn2(X, *Ws, Q_out, Kc, Vc, tmp, ws)
        else:
            DAttn2()(X, *Ws, Q_out, Kc, Vc)
        torch.cuda.synchronize()
        outs.append((Q_out, Kc, Vc))
    for a, b in zip(*outs):
        assert torch.equal(a, b)
