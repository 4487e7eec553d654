"""Timing helpers and the GEMM-family sweep (configs 3 and 4).

Every single-kernel number is the median of CUDA-event timings of individual
launches on the launching stream. The weights of these configs (50-235 MB)
would otherwise sit partly in the 126 MB L2 between iterations, so each case
keeps several copies of its weight (together > 300 MB) and launch i reads copy
i mod n: every launch streams its weight from HBM. (A flush by writing a large
buffer would leave L2 full of dirty lines whose write-back lands inside the
next timed launch.) Algorithmic bytes per call =
weights + x + y (+ gamma); FLOPs = 2·M·N·K (x2 for SwiGLU's two products).
"""
from __future__ import annotations

import json
import statistics
from pathlib import Path

import torch

from . import configs
from .gemm import linear, workspace_bytes, alloc_workspace

ROOT = Path(__file__).resolve().parent.parent


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]), "kind": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "kind": "fallback"}


class L2Flusher:
    def __init__(self, nbytes: int = 512 << 20, device="cuda"):
        self.buf = torch.empty(nbytes // 4, dtype=torch.int32, device=device)

    def __call__(self):
        self.buf.fill_(0)


def time_launches(fn, iters: int = 30, warmup: int = 3, flush: L2Flusher | None = None,
                  busy_cycles: int = 400_000) -> list[float]:
    """Per-launch device times (ms) from CUDA events on the current stream; ``fn(i)``.

    A ~0.2 ms device spin is queued ahead of each timed launch so the host's
    enqueue work (argument checks, TMA descriptor encoding) happens while the
    GPU is busy and never shows up between the two events.
    """
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    times = []
    for i in range(iters):
        if flush is not None:
            flush()
        torch.cuda._sleep(busy_cycles)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        fn(i)
        b.record(stream)
        b.synchronize()
        times.append(a.elapsed_time(b))
    return times


def time_back_to_back(fn, n: int = 24, busy_cycles: int = 2_000_000) -> float:
    """Average device time (ms) per call of ``n`` calls issued back to back.

    This is the steady state of a decode step, where each GEMM follows another
    kernel on the stream and its weight stream may start while that kernel
    drains (programmatic dependent launch). A ~1 ms device spin queued first
    lets the host enqueue every call before the first one starts.
    """
    stream = torch.cuda.current_stream()
    fn(0)
    torch.cuda.synchronize()
    torch.cuda._sleep(busy_cycles)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(n):
        fn(i)
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b) / n


def weight_copies(w: torch.Tensor, min_total: int = 320 << 20) -> list[torch.Tensor]:
    """``w`` plus clones so that the copies together exceed ``min_total`` bytes (>= 2 copies)."""
    nb = w.numel() * w.element_size()
    n = max(2, -(-min_total // nb) + 1)
    return [w] + [w.clone() for _ in range(n - 1)]


def gemm_sweep(iters: int = 30, include_cublas: bool = True) -> list[dict]:
    """Config 3 (skinny GEMM, M sweep) and config 4 (RMSNorm->QKV, SwiGLU) on this GPU."""
    peaks = measured_peaks()
    rows = []
    cases = [("skinny_gemm", m, 14336, 4096, 2) for m in (1, 4, 8, 16, 64, 256)]
    cases += [("rmsnorm_qkv", m, 6144, 4096, 3) for m in (1, 16, 128)]
    cases += [("swiglu_gate_up", m, 14336, 4096, 3) for m in (1, 16, 128)]
    for kind, M, N, K, seed in cases:
        rows_w = 2 * N if kind == "swiglu_gate_up" else N
        x, w = configs.gemm_inputs(M, rows_w, K, seed)
        y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        gamma = None
        if kind == "rmsnorm_qkv":
            g = torch.Generator(device="cuda").manual_seed(seed)
            gamma = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).bfloat16()
        sw = kind == "swiglu_gate_up"
        ws = alloc_workspace(workspace_bytes(M, N, K, sw), "cuda")

        ws_list = weight_copies(w)
        nw = len(ws_list)

        def ours(i):
            wi = ws_list[i % nw]
            if sw:
                linear(x, wi, y, w_up=wi, up_row_offset=N, workspace=ws)
            else:
                linear(x, wi, y, gamma=gamma, eps=1e-6, workspace=ws)

        t = statistics.median(time_launches(ours, iters))
        tb = time_back_to_back(ours)
        nbytes = rows_w * K * 2 + M * K * 2 + M * N * 2 + (K * 2 if gamma is not None else 0)
        flops = 2 * M * rows_w * K
        row = {"kernel": kind, "M": M, "N": N, "K": K, "us": round(t * 1e3, 2),
               "TBps": round(nbytes / (t * 1e-3) / 1e12, 3),
               "hbm_frac": round(nbytes / (t * 1e-3) / 1e9 / peaks["hbm_gbs"], 3),
               "TFLOPs": round(flops / (t * 1e-3) / 1e12, 1),
               "path": "stream-K mma.sync" if M <= 16 else "tcgen05/TMEM",
               "us_back_to_back": round(tb * 1e3, 2),
               "hbm_frac_back_to_back": round(nbytes / (tb * 1e-3) / 1e9 / peaks["hbm_gbs"], 3)}
        if include_cublas:
            if sw:
                def ref(i):
                    o = x @ ws_list[i % nw].t()
                    torch.nn.functional.silu(o[:, :N]) * o[:, N:]
            elif gamma is not None:
                def ref(i):
                    torch.nn.functional.rms_norm(x, (K,), weight=gamma, eps=1e-6) @ ws_list[i % nw].t()
            else:
                def ref(i):
                    x @ ws_list[i % nw].t()
            tr = statistics.median(time_launches(ref, iters))
            row["torch_us_back_to_back"] = round(time_back_to_back(ref) * 1e3, 2)
            row["torch_us"] = round(tr * 1e3, 2)
            row["speedup_vs_torch"] = round(tr / t, 2)
        row["weight_copies"] = nw
        rows.append(row)
        del x, w, y, ws, ws_list
    return rows


def attention_sweep(iters: int = 30, splits_sweep: bool = True) -> list[dict]:
    """Decode attention at configs 1 and 2, single-launch and two-launch forms: µs
    per call isolated and back to back, KV-read TB/s and the fraction of the
    measured copy peak.
    Config 1's 67 MB cache fits in L2, so it rotates over copies (> 300 MB) and
    every call reads HBM; config 2's 17 GB padded cache needs none."""
    from .decoding_attention import (alloc_counters, alloc_partials, dec_attn_splitkv_fwd, default_num_splits,
                                     fused_partial_slots)

    peak = measured_peaks()
    rows = []
    for cfg in (configs.ATTN_CONFIG1, configs.ATTN_CONFIG2):
        q, k, v, lens = configs.attn_inputs(cfg)
        B, L = cfg.batch, cfg.max_seqlen
        kv_bytes = cfg.kv_bytes(lens.cpu())
        copies = [(k, v)]
        while len(copies) * kv_bytes < (300 << 20):
            copies.append((k.clone(), v.clone()))
        S0 = default_num_splits(B, cfg.num_heads_kv, L)
        ctr = alloc_counters(B, cfg.num_heads_kv, "cuda")
        variants = [(fused_partial_slots(B, cfg.num_heads_kv, L), True), (S0, False)]
        if cfg is configs.ATTN_CONFIG1 and splits_sweep:
            variants += [(s, True) for s in (5, 9, 17)] + [(s, False) for s in (4, 16) if s != S0]
        for S, single in variants:
            out = torch.empty(B, 1, cfg.num_heads_q, 128, dtype=torch.bfloat16, device="cuda")
            lse = torch.empty(B, cfg.num_heads_q, device="cuda")
            o_p, l_p = alloc_partials(B, cfg.num_heads_q, S, "cuda")

            def call(i):
                kk, vv = copies[i % len(copies)]
                dec_attn_splitkv_fwd(q, kk, vv, lens, out, lse, o_p, l_p, S, single_launch=single, counters=ctr)

            t = statistics.median(time_launches(call, iters=iters))
            tb = time_back_to_back(call)
            rows.append({"kernel": "decode_attention", "config": cfg.name, "batch": B, "max_seqlen": L,
                         "num_splits": S, "launches": 1 if single else 2, "kv_bytes": kv_bytes,
                         "kv_copies": len(copies),
                         "us_per_call": round(t * 1e3, 2), "TBps": round(kv_bytes / (t * 1e-3) / 1e12, 3),
                         "hbm_frac": round(kv_bytes / (t * 1e-3) / 1e9 / peak["hbm_gbs"], 3),
                         "us_back_to_back": round(tb * 1e3, 2),
                         "hbm_frac_back_to_back": round(kv_bytes / (tb * 1e-3) / 1e9 / peak["hbm_gbs"], 3)})
        del q, k, v, copies
        torch.cuda.empty_cache()
    return rows


def prefill_sweep(iters: int = 20) -> list[dict]:
    """Prefill attention at the reference's FlashSM90 test size ([16, 16, 4096, D],
    attn/attempt6_epi_pipeline/tests.py:138-154), D = 64 and 128, against torch
    SDPA's cuDNN and flash backends. Compute-bound: FLOPs = 4·B·H·Lq·Lkv·D;
    the median of back-to-back launches (inputs stay in L2 as they would in a model)."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from .prefill_attention import flash_attention

    peak = measured_peaks()
    rows = []
    for D in (64, 128):
        B, H, L = 16, 16, 4096
        g = torch.Generator(device="cuda").manual_seed(D)
        q, k, v = [(torch.randn(B, H, L, D, device="cuda", generator=g) + 0.5).bfloat16() for _ in range(3)]
        o = torch.empty_like(q)
        flops = 4 * B * H * L * L * D
        t = statistics.median(time_launches(lambda i: flash_attention(q, k, v, o), iters=iters))
        row = {"kernel": "fmha_fwd", "B": B, "H": H, "L": L, "D": D, "ms": round(t, 4),
               "TFLOPs": round(flops / t / 1e9, 1), "tensor_frac": round(flops / t / 1e9 / peak["bf16_tflops"], 3)}
        for name, be in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
            try:
                with sdpa_kernel([be]):
                    tr = statistics.median(time_launches(
                        lambda i: torch.nn.functional.scaled_dot_product_attention(q, k, v), iters=iters))
                row[f"sdpa_{name}_ms"] = round(tr, 4)
                row[f"sdpa_{name}_TFLOPs"] = round(flops / tr / 1e9, 1)
            except RuntimeError as e:  # backend unavailable for this shape
                row[f"sdpa_{name}"] = str(e).splitlines()[0][:80]
        rows.append(row)
    return rows


def main():
    import argparse

    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--only", choices=["gemm", "prefill", "attention"], default=None)
    args = ap.parse_args()
    if args.only in (None, "gemm"):
        for r in gemm_sweep(args.iters):
            print(json.dumps(r), flush=True)
    if args.only in (None, "attention"):
        for r in attention_sweep(args.iters):
            print(json.dumps(r), flush=True)
    if args.only in (None, "prefill"):
        for r in prefill_sweep():
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()


# ---------------------------------------------------------------------------
# Sub-benchmarks of bench.py's JSON line (the reference project's benchmark list
# beyond the headline): each returns plain numbers; bench.py adds the roofline
# denominators and the CPU baselines.
# ---------------------------------------------------------------------------

def launch_floor(iters: int = 30) -> dict:
    """Device time of a one-element torch kernel timed like every number here:
    what any single launch costs on this pool before it moves a byte."""
    x = torch.zeros(1, device="cuda")
    t = statistics.median(time_launches(lambda i: x.add_(1), iters=iters))
    tb = time_back_to_back(lambda i: x.add_(1))
    return {"us_isolated": round(t * 1e3, 2), "us_back_to_back": round(tb * 1e3, 2)}


def bench_attention_config1(iters: int = 30) -> dict:
    """Config 1 (B=4, L=4096, 32q/8kv, 67 MB of KV) through the default entry point
    (the form plan_attention picks). The cache rotates over copies (> 300 MB) so
    every call reads HBM."""
    from .decoding_attention import alloc_counters, alloc_partials, dec_attn_splitkv_fwd, plan_attention

    cfg = configs.ATTN_CONFIG1
    q, k, v, lens = configs.attn_inputs(cfg)
    B, L = cfg.batch, cfg.max_seqlen
    kv_bytes = cfg.kv_bytes(lens.cpu())
    copies = [(k, v)]
    while len(copies) * kv_bytes < (300 << 20):
        copies.append((k.clone(), v.clone()))
    single, S = plan_attention(B, cfg.num_heads_kv, L)
    out = torch.empty(B, 1, cfg.num_heads_q, 128, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, cfg.num_heads_q, device="cuda")
    o_p, l_p = alloc_partials(B, cfg.num_heads_q, S, "cuda")
    ctr = alloc_counters(B, cfg.num_heads_kv, "cuda")

    def call(i):
        kk, vv = copies[i % len(copies)]
        dec_attn_splitkv_fwd(q, kk, vv, lens, out, lse, o_p, l_p, S, single_launch=single, counters=ctr)

    t = statistics.median(time_launches(call, iters=iters))
    tb = time_back_to_back(call)
    return {"kv_bytes": kv_bytes, "algorithmic_bytes": kv_bytes + cfg.io_bytes(),
            "form": "single launch" if single else "two launches (pass 2 as a programmatic dependent)",
            "num_splits": S, "kv_copies": len(copies), "launches_per_call": 1 if single else 2,
            "us_isolated": round(t * 1e3, 2), "us_back_to_back": round(tb * 1e3, 2)}


def bench_linear_shard(kind: str, M: int, N: int, K: int, seed: int, rank: int = 0, world: int = 1,
                       iters: int = 30, include_cublas: bool = True) -> dict:
    """One rank's column shard of a config-3 / config-4 GEMM (``world`` = 1: the whole GEMM).

    kind: "plain" (y = x W^T, config 3), "rmsnorm" (RMSNorm -> W_qkv, config 4a) or
    "swiglu" (RMSNorm-free gate/up + SwiGLU on W [2N, K], config 4b: gate and up
    rows of the same columns stay on one rank). Weights rotate over copies so
    every launch streams HBM. Returns µs per launch isolated and back to back and
    the shard's algorithmic bytes."""
    from .sharding import column_range, shard_gate_up

    sw = kind == "swiglu"
    x, w = configs.gemm_inputs(M, 2 * N if sw else N, K, seed)
    if world > 1:
        if sw:
            w = shard_gate_up(w, rank, world)
        else:
            lo, hi = column_range(N, rank, world)
            w = w[lo:hi].contiguous()
    n_local = w.shape[0] // 2 if sw else w.shape[0]
    gamma = None
    if kind == "rmsnorm":
        g = torch.Generator(device="cuda").manual_seed(seed)
        gamma = (1 + 0.1 * torch.randn(K, generator=g, device="cuda")).bfloat16()
    y = torch.empty(M, n_local, dtype=torch.bfloat16, device="cuda")
    ws = alloc_workspace(workspace_bytes(M, n_local, K, sw), "cuda")
    wl = weight_copies(w)
    nw = len(wl)

    def ours(i):
        wi = wl[i % nw]
        if sw:
            linear(x, wi, y, w_up=wi, up_row_offset=n_local, workspace=ws)
        else:
            linear(x, wi, y, gamma=gamma, eps=1e-6, workspace=ws)

    t = statistics.median(time_launches(ours, iters))
    tb = time_back_to_back(ours)
    nbytes = w.numel() * 2 + M * K * 2 + M * n_local * 2 + (K * 2 if gamma is not None else 0)
    row = {"M": M, "N": N, "K": K, "N_local": n_local, "bytes_local": nbytes,
           "flops_local": 2 * M * w.shape[0] * K,
           "path": "stream-K mma.sync (M <= 16)" if M <= 16 else "tcgen05 / TMEM",
           "us_isolated": round(t * 1e3, 2), "us_back_to_back": round(tb * 1e3, 2), "weight_copies": nw}
    if include_cublas:
        if sw:
            def ref(i):
                o = x @ wl[i % nw].t()
                torch.nn.functional.silu(o[:, :n_local]) * o[:, n_local:]
        elif gamma is not None:
            def ref(i):
                torch.nn.functional.rms_norm(x, (K,), weight=gamma, eps=1e-6) @ wl[i % nw].t()
        else:
            def ref(i):
                x @ wl[i % nw].t()
        row["torch_us_isolated"] = round(statistics.median(time_launches(ref, iters)) * 1e3, 2)
        row["torch_us_back_to_back"] = round(time_back_to_back(ref) * 1e3, 2)
    del wl, w, x, y, ws
    torch.cuda.empty_cache()
    return row
