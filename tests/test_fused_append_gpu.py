"""KV append fused into the QKV projection epilogue, and attention that publishes the advanced lengths.

The fused path must be bit-identical to the unfused one (projection, then the
standalone append kernel, then attention), for the skinny (M <= 16) and the
tcgen05 (M > 16, several RMSNorm token tiles) GEMMs, contiguous and paged caches.
"""
import pytest
import torch

from fused_kernels_cutedsl_lib_b200 import _native, alloc_partials, default_num_splits, linear
from fused_kernels_cutedsl_lib_b200.layer import (
    DecodeLayer,
    attention_commit,
    attention_from_qkv,
    kv_append,
    kv_append_paged,
    linear_kv_append,
    random_layer_weights,
)

pytestmark = pytest.mark.gpu

HQ, HKV, H = 8, 2, 512


def _inputs(B, L, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(B, H, generator=g, device="cuda").bfloat16()
    w = (0.02 * torch.randn((HQ + 2 * HKV) * 128, H, generator=g, device="cuda")).bfloat16()
    gamma = (1 + 0.1 * torch.randn(H, generator=g, device="cuda")).bfloat16()
    k = torch.randn(B, L, HKV, 128, generator=g, device="cuda").bfloat16()
    v = torch.randn(B, L, HKV, 128, generator=g, device="cuda").bfloat16()
    lens = torch.randint(0, L, (B,), generator=g, device="cuda", dtype=torch.int32)
    lens[0] = L  # a full row: not written, length kept
    if B > 1:
        lens[1] = L - 1  # the last free slot
    return x, w, gamma, k, v, lens


@pytest.mark.parametrize("B", [1, 5, 16, 40, 200])
@pytest.mark.parametrize("norm", [True, False])
def test_contiguous_matches_unfused(B, norm):
    L = 96
    x, w, gamma, k, v, lens = _inputs(B, L, seed=B)
    g = gamma if norm else None
    qkv_ref = linear(x, w, gamma=g)
    k_ref, v_ref, lens_ref = k.clone(), v.clone(), lens.clone()
    kv_append(qkv_ref, k_ref, v_ref, lens_ref, HQ, HKV)
    qkv = torch.empty_like(qkv_ref)
    nxt = torch.full_like(lens, -7)
    linear_kv_append(x, w, qkv, k, v, lens, nxt, HQ, HKV, gamma=g)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert torch.equal(qkv, qkv_ref)
    assert torch.equal(k, k_ref) and torch.equal(v, v_ref)
    assert torch.equal(nxt, lens_ref)


@pytest.mark.parametrize("B", [3, 33])
def test_paged_matches_unfused(B):
    bs, nb = 64, 3
    x, w, gamma, _, _, _ = _inputs(B, 8, seed=100 + B)
    g = torch.Generator(device="cuda").manual_seed(B)
    pool_blocks = B * nb + 2
    kp = torch.randn(pool_blocks, bs, HKV, 128, generator=g, device="cuda").bfloat16()
    vp = torch.randn(pool_blocks, bs, HKV, 128, generator=g, device="cuda").bfloat16()
    table = torch.randperm(pool_blocks, generator=g, device="cuda")[:B * nb].reshape(B, nb).int().contiguous()
    lens = torch.randint(0, nb * bs + 1, (B,), generator=g, device="cuda", dtype=torch.int32)
    qkv_ref = linear(x, w, gamma=gamma)
    kr, vr, lr = kp.clone(), vp.clone(), lens.clone()
    kv_append_paged(qkv_ref, kr, vr, table, lr, HQ, HKV)
    qkv = torch.empty_like(qkv_ref)
    nxt = torch.empty_like(lens)
    linear_kv_append(x, w, qkv, kp, vp, lens, nxt, HQ, HKV, gamma=gamma, block_table=table)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert torch.equal(qkv, qkv_ref) and torch.equal(kp, kr) and torch.equal(vp, vr) and torch.equal(nxt, lr)


def test_attention_commit_publishes_lengths():
    B, L = 6, 200
    x, w, gamma, k, v, lens = _inputs(B, L, seed=7)
    qkv = linear(x, w, gamma=gamma)
    nxt = (lens + 1).clamp_max(L).int()
    S = default_num_splits(B, HKV, L)
    o_p, l_p = alloc_partials(B, HQ, S, x.device)
    out_ref = torch.empty(B, HQ * 128, dtype=torch.bfloat16, device="cuda")
    lse_ref = torch.empty(B, HQ, dtype=torch.float32, device="cuda")
    attention_from_qkv(qkv, k, v, nxt, out_ref, lse_ref, o_p, l_p, S, HQ, HKV)
    out = torch.empty_like(out_ref)
    lse = torch.empty_like(lse_ref)
    commit = torch.full_like(lens, -1)
    attention_commit(qkv, k, v, nxt, commit, out, lse, o_p, l_p, S, HQ, HKV)
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref) and torch.equal(lse, lse_ref)
    assert torch.equal(commit, nxt)
    with pytest.raises(ValueError):
        attention_commit(qkv, k, v, nxt, nxt, out, lse, o_p, l_p, S, HQ, HKV)


def test_aliasing_lengths_rejected():
    x, w, gamma, k, v, lens = _inputs(4, 64, seed=3)
    qkv = torch.empty(4, w.shape[0], dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        linear_kv_append(x, w, qkv, k, v, lens, lens, HQ, HKV, gamma=gamma)


@pytest.mark.parametrize("B", [4, 150])
def test_layer_fused_equals_unfused(B):
    L = 160
    w = random_layer_weights(H, 1024, HQ, HKV, seed=5)
    x, _, _, k, v, lens = _inputs(B, L, seed=11)
    outs = []
    for fuse in (False, True):
        kk, vv, ll = k.clone(), v.clone(), lens.clone()
        layer = DecodeLayer(w, HQ, HKV, fuse_append=fuse)
        y = layer(x, kk, vv, ll).clone()
        y2 = layer(y, kk, vv, ll).clone()  # a second step reads the first step's rows
        torch.cuda.synchronize()
        outs.append((y, y2, kk, vv, ll))
    assert _native.device_error() == 0
    for a, b in zip(*outs):
        assert torch.equal(a, b)
