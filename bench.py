#!/usr/bin/env python
"""Benchmark of the decode-step hot path (one JSON line on rank 0).

Headline workload: split-KV decode attention with ragged lengths (config 2:
B=64, Hq=32, Hkv=8, D=128, cache padded to 32768, lengths ~U[512, 32768] from
seed 1), one step = pass 1 + pass 2 over the whole batch. Metric: KV-read
TB/s = algorithmic KV bytes (4096 B x sum of true lengths) / step time.
The KV cache (4.4 GB of true KV, 17 GB padded) is larger than L2, so no flush
is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun: rows are balanced across ranks by length (no
collective on the data path); the step time is the max over ranks.
``--impl reference`` times the reference's torch formulas on the host CPU
(the oracle port; the reference's own kernels are sm_90a-only) on a bounded
sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# DRAM bytes (read + write) per launch of splitkv_fwd_kernel, from the ncu
# capture summarised in profiles/splitkv_fwd_kernel_config2.md (small case scaled by KV bytes).
NCU_TRAFFIC_BYTES_PER_LAUNCH = 4_615_000_000  # 542.3 MB at 537 MB of KV, scaled x8.51


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms around the timed region.

    A reader thread timestamps every sample; ``mark_start``/``mark_end`` bracket
    the timed region and only samples inside it are summarised (the sample
    nearest the region is used if the region is shorter than the period).
    """

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, device_index: int):
        import threading

        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        self.t0 = self.t1 = None
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", bus, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        except Exception as e:  # no nvidia-smi: report no clocks
            self.error = repr(e)
            return
        self.error = None
        self.first = threading.Event()

        def reader():
            for line in self.proc.stdout:
                self.samples.append((time.perf_counter(), [x.strip() for x in line.split(",")]))
                self.first.set()

        self.thread = threading.Thread(target=reader, daemon=True)
        self.thread.start()
        self.first.wait(timeout=5)

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_end(self):
        self.t1 = time.perf_counter()
        if self.proc is not None:
            time.sleep(0.15)  # let the sample covering the end arrive

    def stop(self) -> dict | None:
        if self.proc is None:
            return {"error": self.error}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        good = [(t, f) for t, f in self.samples if len(f) >= 8]
        if not good:
            return {"error": "no samples: " + " | ".join(",".join(f) for _, f in self.samples[:2])}
        inside = [f for t, f in good if self.t0 is not None and self.t0 <= t <= (self.t1 or t) + 0.1]
        if not inside and self.t0 is not None:
            inside = [min(good, key=lambda tf: abs(tf[0] - self.t0))[1]]
        sms, maxes, reasons = [], [], set()
        for f in inside:
            try:
                sms.append(float(f[0]))
                maxes.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(self.NAMES, f[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return {"error": "unparsable samples"}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def run_ours(args):
    import torch.distributed as dist

    from fused_kernels_cutedsl_lib_b200 import (alloc_partials, chunk_tokens, configs,
                                                dec_attn_splitkv_fwd, default_num_splits, _native)
    from fused_kernels_cutedsl_lib_b200.sharding import balance_rows

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    cfg = configs.ATTN_CONFIG2
    all_lens = configs.attn_seqlens(cfg)
    rows = balance_rows(all_lens, world)[rank]
    q, k, v, lens = configs.attn_inputs(cfg, device=dev, batch_rows=rows)
    B = len(rows)
    total_kv_bytes = cfg.kv_bytes(all_lens)
    S = default_num_splits(B, cfg.num_heads_kv, cfg.max_seqlen, int(lens.sum()),
                           num_sms=torch.cuda.get_device_properties(dev).multi_processor_count)
    out = torch.empty(B, 1, cfg.num_heads_q, 128, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, cfg.num_heads_q, dtype=torch.float32, device=dev)
    o_p, l_p = alloc_partials(B, cfg.num_heads_q, S, dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S)

    def pass1_pass2_events(n):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
                torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        return evs

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps, events per pass on the launching stream ----
    evs = pass1_pass2_events(args.steps)
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    from fused_kernels_cutedsl_lib_b200.decoding_attention import dec_attn_combine, dec_attn_splitkv_partial
    clocks.mark_start()
    # Timed region: K steps, each pass 1 + pass 2 back to back (pass 2 is a
    # programmatic dependent of pass 1, so no event sits between them here).
    t_start.record(stream)
    for i in range(args.steps):
        dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S)
    t_end.record(stream)
    torch.cuda.synchronize()
    # Per-pass kernel durations for the roofline: a second pass over the same K
    # steps with events around each pass (this ordering forgoes the overlap).
    for i in range(args.steps):
        e0, e1, e2 = evs[i]
        e0.record(stream)
        dec_attn_splitkv_partial(q, k, v, lens, o_p, l_p, S)
        e1.record(stream)
        dec_attn_combine(o_p, l_p, lens, out, lse, cfg.max_seqlen)
        e2.record(stream)
    torch.cuda.synchronize()
    clocks.mark_end()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    p1 = [a.elapsed_time(b) for a, b, _ in evs]
    p2 = [b.elapsed_time(c) for _, b, c in evs]
    local_ms = total_ms / args.steps
    if _native.device_error() != 0:
        raise RuntimeError("device error word set during the bench")

    # ---- e2e: public API with pinned host buffers, copies inside the timed region ----
    # A serving loop: every step copies its q and lengths from pinned host memory
    # and its out and lse back; the copies of the neighbouring steps run on two
    # copy streams (double-buffered device buffers, ordered by events) while this
    # step's kernels run on the compute stream.
    q_h = q.cpu().pin_memory()
    lens_h = lens.cpu().pin_memory()
    out_h = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    lse_h = [torch.empty(lse.shape, dtype=lse.dtype).pin_memory() for _ in range(2)]
    q_d = [torch.empty_like(q) for _ in range(2)]
    lens_d = [torch.empty_like(lens) for _ in range(2)]
    out_d = [torch.empty_like(out) for _ in range(2)]
    lse_d = [torch.empty_like(lse) for _ in range(2)]
    from fused_kernels_cutedsl_lib_b200 import DecodeAttention
    attn = DecodeAttention(num_splits=S)
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]     # inputs of buffer b landed
    ev_done = [torch.cuda.Event() for _ in range(2)]   # kernels of buffer b finished
    ev_out = [torch.cuda.Event() for _ in range(2)]    # results of buffer b copied out

    def e2e_run(n):
        for i in range(n):
            bi = i & 1
            with torch.cuda.stream(h2d_s):
                if i >= 2:
                    h2d_s.wait_event(ev_done[bi])      # step i-2 no longer reads these inputs
                q_d[bi].copy_(q_h, non_blocking=True)
                lens_d[bi].copy_(lens_h, non_blocking=True)
                ev_in[bi].record(h2d_s)
            stream.wait_event(ev_in[bi])
            if i >= 2:
                stream.wait_event(ev_out[bi])          # step i-2's results are out of out_d / lse_d
            attn(q_d[bi], k, v, lens_d[bi], out_d[bi], lse_d[bi])
            ev_done[bi].record(stream)
            with torch.cuda.stream(d2h_s):
                d2h_s.wait_event(ev_done[bi])
                out_h[bi].copy_(out_d[bi], non_blocking=True)
                lse_h[bi].copy_(lse_d[bi], non_blocking=True)
                ev_out[bi].record(d2h_s)
        for bi in range(min(n, 2)):
            stream.wait_event(ev_out[bi])              # the timed region ends after the last copy out

    e2e_run(max(3, args.warmup))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    h2d_s.wait_event(a)
    d2h_s.wait_event(a)
    e2e_run(args.steps)
    b.record(stream)
    torch.cuda.synchronize()
    e2e_local_ms = a.elapsed_time(b) / args.steps
    if not torch.equal(out_h[(args.steps - 1) & 1], out.cpu()):
        raise RuntimeError("e2e result differs from the device-timed step's output")
    h2d = q_h.numel() * q_h.element_size() + lens_h.numel() * 4
    d2h = out_h[0].numel() * 2 + lse_h[0].numel() * 4

    # ---- max over ranks ----
    vals = torch.tensor([local_ms, e2e_local_ms, statistics.mean(p1), statistics.mean(p2)],
                        dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        hb = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
        dist.all_reduce(hb, op=dist.ReduceOp.SUM)
        h2d, d2h = int(hb[0]), int(hb[1])
    step_ms, e2e_ms, p1_ms, p2_ms = vals.tolist()

    if rank == 0:
        peak, peak_kind = _peaks()
        tbps = total_kv_bytes / (step_ms * 1e-3) / 1e12
        # Dominant kernel (pass 1) on one GPU: algorithmic bytes per launch / mean launch time.
        local_kv = cfg.kv_bytes(lens.cpu()) + B * cfg.num_heads_q * 256
        achieved_gbs = local_kv / (statistics.mean(p1) * 1e-3) / 1e9
        line = {
            "metric": "decode-attn KV-read TB/s (split-KV ragged, B=64, Lmax=32768, 32q/8kv, d128)",
            "value": round(tbps, 4),
            "unit": "TB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(step_ms, 5),
            "us_per_call": round(step_ms * 1e3, 2),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) q/k/v, lengths U[512,32768] seed 1)",
            "config": {"workload": "splitkv_decode_attention_config2", "batch": cfg.batch,
                       "max_seqlen": cfg.max_seqlen, "num_heads_q": cfg.num_heads_q,
                       "num_heads_kv": cfg.num_heads_kv, "head_dim": 128, "num_splits": S,
                       "chunk_tokens": chunk_tokens(cfg.max_seqlen, S),
                       "sum_seqlens": int(all_lens.sum()), "kv_bytes": total_kv_bytes,
                       "parallelism": f"batch-sharded x{world} (length-balanced, no collective)",
                       "l2": "inputs (17 GB padded KV) larger than L2; no flush",
                       "pass_timing": "per-pass events in a second loop of K steps"},
            "pass_ms": {"splitkv_fwd": round(p1_ms, 5), "combine": round(p2_ms, 5)},
            "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved_gbs / peak, 4), "peak_kind": peak_kind,
                         "frac_of_nominal_8000": round(achieved_gbs / 8000.0, 4),
                         "kernel": "splitkv_fwd_kernel",
                         "traffic": NCU_TRAFFIC_BYTES_PER_LAUNCH},
            "e2e": {"value": round(total_kv_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "per step: q + cache_seqlens H2D from pinned host, out + lse D2H, through "
                            "DecodeAttention; copies of neighbouring steps overlap the kernels on two copy "
                            "streams (double-buffered); KV cache resident"},
            "gpu_launches": 2 * args.steps,
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(cfg, q, k, v, lens, budget_s=args.cpu_seconds)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline(cfg, q, k, v, lens, budget_s=15.0):
    """Time the reference's torch formulas (oracle port) on the host over a bounded sample of rows."""
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = list(range(q.shape[0]))
    done_bytes, t_used, n = 0, 0.0, 0
    for r in rows:
        qr, kr, vr, lr = q[r:r + 1].cpu(), k[r:r + 1, :int(lens[r])].cpu(), v[r:r + 1, :int(lens[r])].cpu(), lens[r:r + 1].cpu()
        t0 = time.perf_counter()
        oracle.decode_attention(qr, kr, vr, lr)
        t_used += time.perf_counter() - t0
        done_bytes += int(lr[0]) * cfg.num_heads_kv * 128 * 4
        n += 1
        if t_used >= budget_s:
            break
    return {"value": round(done_bytes / t_used / 1e12, 6), "unit": "TB/s", "cores": threads,
            "kind": "port", "sample": f"{n} of {cfg.batch} rows of config 2 ({done_bytes} KV bytes), "
                                      f"fp32 torch on CPU, {t_used:.1f} s"}


def run_reference(args):
    """CPU arm: the reference's torch check formulas (oracle port) on the host cores."""
    world, rank, _ = _dist()
    if rank != 0:
        return
    import oracle
    from fused_kernels_cutedsl_lib_b200 import configs

    cfg = configs.ATTN_CONFIG2
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    all_lens = configs.attn_seqlens(cfg)
    # Bounded sample per step: two full rows (drawn on the CPU with the same per-row seeds).
    rows = [0, 1]
    q, k, v, lens = configs.attn_inputs(cfg, device="cpu", batch_rows=rows)
    sample_bytes = cfg.kv_bytes(lens)

    def step():
        oracle.decode_attention(q, k, v, lens)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    sec = statistics.mean(times)
    tbps = sample_bytes / sec / 1e12
    print(json.dumps({
        "impl": "reference",
        "metric": "decode-attn KV-read TB/s (split-KV ragged, B=64, Lmax=32768, 32q/8kv, d128)",
        "value": round(tbps, 6), "unit": "TB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic (same seeded rows as the GPU arm)",
        "config": {"workload": "splitkv_decode_attention_config2", "sample_rows": rows,
                   "sample_kv_bytes": sample_bytes, "sum_seqlens_full": int(all_lens.sum())},
        "cpu_baseline": {"value": round(tbps, 6), "unit": "TB/s", "cores": threads, "kind": "port",
                         "sample": f"rows {rows} of config 2 per step, fp32 torch on CPU"},
        "e2e": {"value": round(tbps, 6), "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }), flush=True)


def run_layer(args):
    """Config 5: full decoder-layer decode step, B=128 at context 8192 (tensor-parallel for N > 1)."""
    import torch.distributed as dist

    from fused_kernels_cutedsl_lib_b200 import _native
    from fused_kernels_cutedsl_lib_b200.layer import (DecodeLayer, PeerTPDecodeLayer, TPDecodeLayer,
                                                      random_layer_weights, shard_layer_weights)

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    B, ctx, H, F, HQ, HKV = 128, 8192, 4096, 14336, 32, 8
    Lmax = ctx + args.warmup + 2 * args.steps + 32
    full = random_layer_weights(H, F, HQ, HKV, seed=4, device=dev)
    Bl = B // world
    g = torch.Generator(device=dev).manual_seed(4 * 1000 + rank)
    k = torch.empty(Bl, Lmax, HKV, 128, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    v = torch.empty_like(k).normal_(generator=g)
    lens = torch.full((Bl,), ctx, dtype=torch.int32, device=dev)
    gx = torch.Generator(device=dev).manual_seed(44)
    x = torch.randn(B, H, generator=gx, device=dev).to(torch.bfloat16)
    dp = world > 1 and args.tp_mode == "dp"
    if dp:
        # Batch-parallel layer: every rank holds all weights and runs the whole
        # step for its B/P sequences (their KV cache lives only there); no
        # communication. x is this rank's rows of the global batch.
        layer = DecodeLayer(full, HQ, HKV)
        x = x[rank * Bl:(rank + 1) * Bl].contiguous()
    elif world > 1 and args.tp_mode == "peer":
        layer = PeerTPDecodeLayer(shard_layer_weights(full, rank, world, HQ, HKV), num_heads_q=HQ, num_heads_kv=HKV)
    elif world > 1:
        layer = TPDecodeLayer(shard_layer_weights(full, rank, world, HQ, HKV), num_heads_q=HQ, num_heads_kv=HKV)
    else:
        layer = DecodeLayer(full, HQ, HKV)
    wbytes = full.nbytes()
    del full
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        layer(x, k, v, lens)
    torch.cuda.synchronize()
    x_h = x.cpu().pin_memory()
    y_h = torch.empty(x.shape[0], H, dtype=torch.bfloat16).pin_memory()
    x_d = torch.empty_like(x)
    step, step_e2e = (lambda: layer(x, k, v, lens)), None

    def e2e_body():
        x_d.copy_(x_h, non_blocking=True)
        y_h.copy_(layer(x_d, k, v, lens), non_blocking=True)

    step_e2e = e2e_body
    use_graph = not args.no_graph
    graphs = []
    if use_graph:
        # One decode step (12 launches on 1 GPU; 13 + 5 all-gathers under TP) captured
        # once and replayed: no per-launch host work inside the timed loop.
        graphs = [torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()]
        with torch.cuda.graph(graphs[0]):
            layer(x, k, v, lens)
        with torch.cuda.graph(graphs[1]):
            e2e_body()
        torch.cuda.synchronize()
        step, step_e2e = graphs[0].replay, graphs[1].replay
        for _ in range(2):
            step()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.mark_start()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    clocks.mark_end()
    clk = clocks.stop()
    ms = a.elapsed_time(b) / args.steps
    if _native.device_error() != 0:
        raise RuntimeError("device error word set during the bench")
    # e2e: x H2D from pinned host, y D2H, inside the timed region
    a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a2.record(stream)
    for _ in range(args.steps):
        step_e2e()
    b2.record(stream)
    torch.cuda.synchronize()
    e2e_ms = a2.elapsed_time(b2) / args.steps
    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    if rank == 0:
        kv_bytes = B * (ctx + args.warmup + args.steps) * HKV * 128 * 4  # approx. mid-run lengths
        peak, kind = _peaks()
        print(json.dumps({
            "metric": "decode-layer tokens/s (Llama-3-8B-shaped layer, B=128, ctx 8192)",
            "value": round(B / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights seed 4, N(0,1) KV)",
            "config": {"workload": "decode_layer_config5", "batch": B, "context": ctx, "hidden": H, "ffn": F,
                       "heads_q": HQ, "heads_kv": HKV,
                       "parallelism": "single GPU" if world == 1 else (
                           f"dp{world}: batch-sharded layer, weights replicated, no collective" if dp else
                           f"tp{world} GEMMs + batch-sharded attention, all-gathers "
                           + ("in the GEMM / attention epilogues over peer memory" if args.tp_mode == "peer"
                              else "by NCCL")),
                       "cuda_graph": not args.no_graph,
                       "l2": "weights 436 MB + KV 4.3 GB per step exceed L2"},
            "bytes_per_step": wbytes * (world if dp else 1) + kv_bytes,  # dp: every rank streams all weights
            "achieved_TBps": round((wbytes * (world if dp else 1) + kv_bytes) / world / (ms * 1e-3) / 1e12, 3),
            "peak_GBps": peak, "peak_kind": kind,
            "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": B * H * 2, "d2h_bytes_per_step": B * H * 2},
            # this library's kernels per step: QKV (rms_split, GEMM, reduce; KV append
            # fused), attention (2), O-proj (GEMM, reduce), gate/up (rms_split, GEMM,
            # reduce), down (GEMM, reduce); under TP the append is its own kernel
            "gpu_launches": args.steps * (12 if (world == 1 or dp) else (18 if args.tp_mode == "peer" else 13)),
            "clocks": clk,
        }), flush=True)
    # Graphs that captured NCCL collectives must be freed before the process
    # group is destroyed (destroying it first hangs at exit).
    step = step_e2e = None
    graphs.clear()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        if hasattr(layer, "close"):
            layer.close()  # unmap the peers' buffers before the ranks exit
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="layer workload: launch eagerly instead of replaying a CUDA graph")
    ap.add_argument("--tp-mode", choices=["peer", "nccl", "dp"], default="peer",
                    help="layer workload on N > 1 GPUs: tensor-parallel GEMMs with the all-gathers in the kernels "
                         "over peer memory (peer) or by NCCL (nccl); or batch-parallel with replicated weights (dp)")
    ap.add_argument("--workload", choices=["attention", "layer"], default="attention",
                    help="attention: config 2 split-KV decode attention (headline); layer: config 5 decode step")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "layer":
        run_layer(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
