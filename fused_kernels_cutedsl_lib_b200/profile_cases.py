"""Small, fixed workloads for Nsight Compute captures of single kernels.

Each case builds its inputs (larger than the 126 MB L2 so DRAM counters are
meaningful, a few GB at most), runs a few warm-up launches and then
``--launches`` launches of one kernel, and exits. The profiles/ summaries name
the exact command, e.g.

    ncu --set full --clock-control none -k regex:splitkv_kernel -s 2 -c 1 \
        python -m fused_kernels_cutedsl_lib_b200.profile_cases attn_fused_small
"""
from __future__ import annotations

import argparse

import torch


def _attn_case(launches: int, single: bool, B=16, L=8192):
    from . import alloc_counters, alloc_partials, dec_attn_splitkv_fwd, default_num_splits, fused_partial_slots

    Hq, Hkv = 32, 8
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, 1, Hq, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, L, Hkv, 128, device="cuda", generator=g, dtype=torch.bfloat16)
    v = torch.randn(B, L, Hkv, 128, device="cuda", generator=g, dtype=torch.bfloat16)
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    S = fused_partial_slots(B, Hkv, L) if single else default_num_splits(B, Hkv, L)
    out = torch.empty(B, 1, Hq, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, Hq, device="cuda")
    o_p, l_p = alloc_partials(B, Hq, S, "cuda")
    ctr = alloc_counters(B, Hkv, "cuda")
    for _ in range(2 + launches):
        dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S, single_launch=single, counters=ctr)
    torch.cuda.synchronize()
    print(f"attn: B={B} L={L} single_launch={single} splits={S} kv_bytes={B * L * Hkv * 128 * 4}")


def case_attn_small(launches: int):
    """Decode attention, two-launch form (pass 1 + combine_kernel): B=16, 32q/8kv,
    every row at 8192 tokens, 537 MB of KV per launch."""
    _attn_case(launches, single=False)


def case_attn_fused_small(launches: int):
    """Decode attention, single-launch form (stream-K + in-kernel merge), same 537 MB case."""
    _attn_case(launches, single=True)


def case_dattn1(launches: int):
    """Reference-semantics DAttn1 at the reference demo's shape scaled to exceed L2:
    H=512 heads, M=16, P=1024 (K and V^T 512 MB together)."""
    from .decoding_attention import DAttn1

    g = torch.Generator(device="cuda").manual_seed(0)
    H, M, P = 512, 16, 1024
    Q = torch.randn(H, M, 128, device="cuda", generator=g).bfloat16()
    K = torch.randn(H, P, 128, device="cuda", generator=g).bfloat16()
    V = torch.randn(H, 128, P, device="cuda", generator=g).bfloat16()
    O = torch.empty(H, M, 128, dtype=torch.bfloat16, device="cuda")
    k = DAttn1()
    for _ in range(2 + launches):
        k(Q, K, V, O)
    torch.cuda.synchronize()
    print(f"dattn1: H={H} M={M} P={P}")


def case_kv_append(launches: int):
    """KV-cache append of 128 rows (config 5's batch) from a QKV output."""
    from .layer import kv_append

    B, L = 128, 8192 + 64
    k = torch.zeros(B, L, 8, 128, dtype=torch.bfloat16, device="cuda")
    v = torch.zeros_like(k)
    qkv = torch.randn(B, 6144, device="cuda").bfloat16()
    for _ in range(2 + launches):
        lens = torch.full((B,), 8192, dtype=torch.int32, device="cuda")
        kv_append(qkv, k, v, lens, 32, 8)
    torch.cuda.synchronize()
    print("kv_append: B=128")


def case_peer_barrier1(launches: int):
    """The stage barrier kernel with one rank (no peer to wait for): its launch and fence cost."""
    from . import _native

    lib = _native.load()
    buf = torch.zeros(16, dtype=torch.int32, device="cuda")
    import ctypes

    peers = (ctypes.c_void_p * 1)(buf.data_ptr() + 8)
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2 + launches):
        _native.check(lib.fk_peer_barrier(buf.data_ptr(), buf.data_ptr() + 8, peers, 0, 1, st))
    torch.cuda.synchronize()
    print("peer barrier, 1 rank")


def _gemm_case(M, N, K, launches, kind="plain"):
    from . import configs
    from .gemm import alloc_workspace, linear, workspace_bytes

    rows = 2 * N if kind in ("swiglu", "rms_swiglu") else N
    x, w = configs.gemm_inputs(M, rows, K, 2)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gamma = torch.ones(K, dtype=torch.bfloat16, device="cuda") if kind in ("rms", "rms_swiglu") else None
    ws = alloc_workspace(workspace_bytes(M, N, K, kind in ("swiglu", "rms_swiglu")), "cuda")
    flush = torch.empty(256 << 18, dtype=torch.int32, device="cuda")  # 256 MB L2 flush
    for _ in range(2 + launches):
        flush.fill_(0)
        if kind in ("swiglu", "rms_swiglu"):
            linear(x, w, y, gamma=gamma, w_up=w, up_row_offset=N, workspace=ws)
        else:
            linear(x, w, y, gamma=gamma, workspace=ws)
    torch.cuda.synchronize()
    print(f"gemm {kind}: M={M} N={N} K={K} weight_bytes={rows * K * 2}")


def case_skinny_m16(launches: int):
    """Skinny stream-K GEMM, config 3 at M=16: W [14336, 4096] = 117 MB."""
    _gemm_case(16, 14336, 4096, launches)


def case_skinny_m1(launches: int):
    """Skinny stream-K GEMM, config 3 at M=1."""
    _gemm_case(1, 14336, 4096, launches)


def case_tc_m256(launches: int):
    """tcgen05 GEMM, config 3 at M=256."""
    _gemm_case(256, 14336, 4096, launches)


def case_tc_m128_swiglu(launches: int):
    """tcgen05 SwiGLU gate/up GEMM, config 4 at M=128: W [28672, 4096] = 235 MB."""
    _gemm_case(128, 14336, 4096, launches, "swiglu")


def case_tc_m128_rms_swiglu(launches: int):
    """tcgen05 RMSNorm->gate/up->SwiGLU GEMM (the layer's FFN input), M=128: 256 token columns (hi/lo)."""
    _gemm_case(128, 14336, 4096, launches, "rms_swiglu")


def case_tc_m64(launches: int):
    """tcgen05 GEMM, config 3 at M=64."""
    _gemm_case(64, 14336, 4096, launches)


def case_tc_m128_rms_qkv(launches: int):
    """tcgen05 RMSNorm->QKV GEMM, config 4 at M=128: W [6144, 4096] = 50 MB."""
    _gemm_case(128, 6144, 4096, launches, "rms")


def _prefill_case(D, launches):
    from .prefill_attention import flash_attention

    B, H, L = 2, 16, 4096
    g = torch.Generator(device="cuda").manual_seed(D)
    q, k, v = [(torch.randn(B, H, L, D, device="cuda", generator=g) + 0.5).bfloat16() for _ in range(3)]
    o = torch.empty_like(q)
    for _ in range(2 + launches):
        flash_attention(q, k, v, o)
    torch.cuda.synchronize()
    print(f"prefill D={D}: B={B} H={H} L={L} flops={4 * B * H * L * L * D}")


def case_prefill_d64(launches: int):
    """Prefill attention, the reference test shape at 2 of 16 batches: [2, 16, 4096, 64]."""
    _prefill_case(64, launches)


def case_prefill_d128(launches: int):
    """Prefill attention [2, 16, 4096, 128]."""
    _prefill_case(128, launches)


def case_tp4_rank_step(launches: int):
    """One rank's kernels of the 4-way tensor-parallel layer step at config 5 on one GPU
    (M = 128 tokens; QKV 1536, O 1024, gate/up 2 x 3584, down 1024 columns; attention
    over the rank's 32 batch rows at context 8192). Peer copies and barriers omitted."""
    from .decoding_attention import alloc_partials, default_num_splits
    from .gemm import alloc_workspace, linear, workspace_bytes
    from .layer import attention_from_qkv, kv_append, random_layer_weights, shard_layer_weights

    world, rank, B, ctx = 4, 0, 128, 8192
    w = shard_layer_weights(random_layer_weights(seed=4), rank, world)
    Bl = B // world
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(B, 4096, device="cuda", generator=g).bfloat16()
    k = torch.randn(Bl, ctx + 64, 8, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn_like(k)
    ws = alloc_workspace(workspace_bytes(B, 14336, 4096, True), "cuda")
    bf = dict(dtype=torch.bfloat16, device="cuda")
    qkv_loc = torch.empty(B, w.w_qkv.shape[0], **bf)             # this rank's column blocks
    qkv_rows = torch.randn(Bl, 6144, device="cuda", generator=g).bfloat16()  # the rank's rows, all columns
    attn_full, h_full = torch.randn(B, 4096, **bf), torch.randn(B, 4096, **bf)
    gu_full = torch.randn(B, 14336, **bf)
    attn_loc = torch.empty(Bl, 4096, **bf)
    h_loc, y_loc = torch.empty(B, w.w_o.shape[0], **bf), torch.empty(B, w.w_down.shape[0], **bf)
    fl = w.w_gate_up.shape[0] // 2
    gu_loc = torch.empty(B, fl, **bf)
    res_x, res_h = x[:, :h_loc.shape[1]].contiguous(), h_full[:, :h_loc.shape[1]].contiguous()
    S = default_num_splits(Bl, 8, ctx + 64)
    o_p, l_p = alloc_partials(Bl, 32, S, "cuda")
    lse = torch.empty(Bl, 32, device="cuda")
    for _ in range(2 + launches):
        lens = torch.full((Bl,), ctx, dtype=torch.int32, device="cuda")
        linear(x, w.w_qkv, qkv_loc, gamma=w.gamma_attn, workspace=ws)
        kv_append(qkv_rows, k, v, lens, 32, 8)
        attention_from_qkv(qkv_rows, k, v, lens, attn_loc, lse, o_p, l_p, S, 32, 8)
        linear(attn_full, w.w_o, h_loc, residual=res_x, workspace=ws)
        linear(h_full, w.w_gate_up, gu_loc, gamma=w.gamma_ffn, w_up=w.w_gate_up, up_row_offset=fl, workspace=ws)
        linear(gu_full, w.w_down, y_loc, residual=res_h, workspace=ws)
    torch.cuda.synchronize()
    print("tp4 rank step: 12 kernels per step")


CASES = {
    "attn_fused_small": case_attn_fused_small,
    "dattn1": case_dattn1,
    "kv_append": case_kv_append,
    "peer_barrier1": case_peer_barrier1,
    "tp4_rank_step": case_tp4_rank_step,
    "prefill_d64": case_prefill_d64,
    "prefill_d128": case_prefill_d128,
    "tc_m64": case_tc_m64,
    "tc_m128_rms_qkv": case_tc_m128_rms_qkv,
    "attn_small": case_attn_small,
    "skinny_m16": case_skinny_m16,
    "skinny_m1": case_skinny_m1,
    "tc_m256": case_tc_m256,
    "tc_m128_swiglu": case_tc_m128_swiglu,
    "tc_m128_rms_swiglu": case_tc_m128_rms_swiglu,
}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--launches", type=int, default=3)
    args = ap.parse_args()
    CASES[args.case](args.launches)


if __name__ == "__main__":
    main()
