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

# A collective that does not complete within this many seconds raises on every
# rank instead of waiting out the caller's time limit (a rank that failed leaves
# the others in their next collective).
PG_TIMEOUT_S = 180

# DRAM bytes (read + write) per launch of the single-launch attention kernel: an
# ncu capture of profile case attn_fused_small (541.5 MB at 536.9 MB of KV),
# scaled by KV bytes to config 2 (x8.51; traffic grows in proportion).
NCU_TRAFFIC_BYTES_PER_LAUNCH = 4_608_300_000  # 541.5 MB at 536.9 MB of KV, scaled x8.51


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

    from fused_kernels_cutedsl_lib_b200 import (alloc_counters, alloc_partials, configs, dec_attn_splitkv_fwd,
                                                plan_attention, _native)
    from fused_kernels_cutedsl_lib_b200.sharding import balance_rows

    import datetime

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))

    cfg = configs.ATTN_CONFIG2
    all_lens = configs.attn_seqlens(cfg)
    rows = balance_rows(all_lens, world)[rank]
    q, k, v, lens = configs.attn_inputs(cfg, device=dev, batch_rows=rows)
    B = len(rows)
    total_kv_bytes = cfg.kv_bytes(all_lens)
    nsm = torch.cuda.get_device_properties(dev).multi_processor_count
    # The form and split count the library's default entry points pick for this
    # shard (DecodeAttention below plans the same way).
    single, S = plan_attention(B, cfg.num_heads_kv, cfg.max_seqlen, num_sms=nsm)
    out = torch.empty(B, 1, cfg.num_heads_q, 128, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, cfg.num_heads_q, dtype=torch.float32, device=dev)
    o_p, l_p = alloc_partials(B, cfg.num_heads_q, S, dev)
    ctr = alloc_counters(B, cfg.num_heads_kv, dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        dec_attn_splitkv_fwd(q, k, v, lens, out, lse, o_p, l_p, S, single_launch=single, counters=ctr)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region: K steps back to back on the launching stream ----
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks.mark_start()
    t_start.record(stream)
    for i in range(args.steps):
        step()
    t_end.record(stream)
    torch.cuda.synchronize()
    # Per-launch kernel durations for the roofline: a second loop of K steps
    # with events around each launch (single launch: the one kernel is the step).
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        evs[i][0].record(stream)
        step()
        evs[i][1].record(stream)
    torch.cuda.synchronize()
    clocks.mark_end()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    total_ms = t_start.elapsed_time(t_end)
    per_launch = [a.elapsed_time(b) for a, b in evs]
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
    attn = DecodeAttention()
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
    vals = torch.tensor([local_ms, e2e_local_ms, statistics.mean(per_launch)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
        hb = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
        dist.all_reduce(hb, op=dist.ReduceOp.SUM)
        h2d, d2h = int(hb[0]), int(hb[1])
    step_ms, e2e_ms, launch_ms = vals.tolist()

    # ---- the rest of the reference's benchmark list (configs 1, 3, 4, 5) ----
    extras = {}
    if not args.no_extras:
        del q, k, v, out, lse, o_p, l_p
        torch.cuda.empty_cache()
        extras = run_extras(args, world, rank, dev, cpu=(world == 1 and not args.no_cpu_baseline))

    if rank == 0:
        peak, peak_kind = _peaks()
        tbps = total_kv_bytes / (step_ms * 1e-3) / 1e12
        # Dominant kernel on one GPU: algorithmic bytes per launch / mean launch time.
        local_kv = cfg.kv_bytes(lens.cpu()) + B * cfg.num_heads_q * 256
        achieved_gbs = local_kv / (statistics.mean(per_launch) * 1e-3) / 1e9
        kern = "splitkv_kernel<3, true> (single launch)" if single else "splitkv_kernel<3, false> + combine_kernel"
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
                       "num_heads_kv": cfg.num_heads_kv, "head_dim": 128,
                       "form": "single launch (stream-K tiles, in-kernel merge)" if single else "two launches",
                       "num_splits": S, "sum_seqlens": int(all_lens.sum()), "kv_bytes": total_kv_bytes,
                       "parallelism": f"batch-sharded x{world} (length-balanced, no collective)",
                       "l2": "inputs (17 GB padded KV) larger than L2; no flush",
                       "launch_timing": "per-launch events in a second loop of K steps"},
            "launch_ms": round(launch_ms, 5),
            "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved_gbs / peak, 4), "peak_kind": peak_kind,
                         "frac_of_nominal_8000": round(achieved_gbs / 8000.0, 4),
                         "kernel": kern,
                         "traffic": NCU_TRAFFIC_BYTES_PER_LAUNCH},
            "e2e": {"value": round(total_kv_bytes / (e2e_ms * 1e-3) / 1e12, 4), "unit": "TB/s",
                    "ms_per_step": round(e2e_ms, 5), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "note": "per step: q + cache_seqlens H2D from pinned host, out + lse D2H, through "
                            "DecodeAttention; copies of neighbouring steps overlap the kernels on two copy "
                            "streams (double-buffered); KV cache resident"},
            "gpu_launches": (1 if single else 2) * args.steps,
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu_baseline:
            qh, kh, vh, lh = configs.attn_inputs(cfg, device="cpu", batch_rows=[0, 1])
            line["cpu_baseline"] = cpu_baseline(cfg, qh, kh, vh, lh, budget_s=args.cpu_seconds)
        line.update(extras)
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
    while t_used < budget_s and n < 200:  # cycle over the sampled rows until the budget is spent
        r = rows[n % len(rows)]
        qr, kr, vr, lr = q[r:r + 1].cpu(), k[r:r + 1, :int(lens[r])].cpu(), v[r:r + 1, :int(lens[r])].cpu(), lens[r:r + 1].cpu()
        t0 = time.perf_counter()
        oracle.decode_attention(qr, kr, vr, lr)
        t_used += time.perf_counter() - t0
        done_bytes += int(lr[0]) * cfg.num_heads_kv * 128 * 4
        n += 1
    return {"value": round(done_bytes / t_used / 1e12, 6), "unit": "TB/s", "cores": threads,
            "kind": "port", "sample": f"{n} row passes over rows {rows} of {cfg.name} ({done_bytes} KV bytes), "
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


def layer_measure(args, world, rank, dev, steps, warmup, tp_mode="peer", use_graph=True, clocks_on=True):
    """Config 5 decode step (B=128 at context 8192): ms per step on the device, e2e
    ms per step (x H2D and y D2H inside the timed region), launches per step and
    the clock record. Single GPU: DecodeLayer; N > 1: tensor-parallel
    (PeerTPDecodeLayer by default) or batch-parallel (tp_mode "dp"). Max over ranks."""
    import torch.distributed as dist

    from fused_kernels_cutedsl_lib_b200 import _native
    from fused_kernels_cutedsl_lib_b200.layer import (DecodeLayer, HybridDecodeLayer, PeerTPDecodeLayer,
                                                      TPDecodeLayer, random_layer_weights, shard_layer_weights)

    B, ctx, H, F, HQ, HKV = 128, 8192, 4096, 14336, 32, 8
    # every step appends one token per row: room for warm-up, capture and both timed loops
    Lmax = ctx + warmup + 2 * steps + 32
    full = random_layer_weights(H, F, HQ, HKV, seed=4, device=dev)
    Bl = B // world
    g = torch.Generator(device=dev).manual_seed(4 * 1000 + rank)
    k = torch.empty(Bl, Lmax, HKV, 128, dtype=torch.bfloat16, device=dev).normal_(generator=g)
    v = torch.empty_like(k).normal_(generator=g)
    lens = torch.full((Bl,), ctx, dtype=torch.int32, device=dev)
    gx = torch.Generator(device=dev).manual_seed(44)
    x = torch.randn(B, H, generator=gx, device=dev).to(torch.bfloat16)
    dp = world > 1 and tp_mode == "dp"
    if dp:
        # Batch-parallel layer: every rank holds all weights and runs the whole
        # step for its B/P sequences (their KV cache lives only there); no
        # communication. x is this rank's rows of the global batch.
        layer = DecodeLayer(full, HQ, HKV)
        x = x[rank * Bl:(rank + 1) * Bl].contiguous()
    elif world > 1 and tp_mode == "hybrid":
        layer = HybridDecodeLayer(full, num_heads_q=HQ, num_heads_kv=HKV)
    elif world > 1 and tp_mode == "peer":
        layer = PeerTPDecodeLayer(shard_layer_weights(full, rank, world, HQ, HKV), num_heads_q=HQ, num_heads_kv=HKV)
    elif world > 1:
        layer = TPDecodeLayer(shard_layer_weights(full, rank, world, HQ, HKV), num_heads_q=HQ, num_heads_kv=HKV)
    else:
        layer = DecodeLayer(full, HQ, HKV)
    wbytes = full.nbytes()
    del full
    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        layer(x, k, v, lens)
    torch.cuda.synchronize()
    x_h = x.cpu().pin_memory()
    y_h = torch.empty(x.shape[0], H, dtype=torch.bfloat16).pin_memory()
    x_d = torch.empty_like(x)
    step = lambda: layer(x, k, v, lens)  # noqa: E731

    def e2e_body():
        x_d.copy_(x_h, non_blocking=True)
        y_h.copy_(layer(x_d, k, v, lens), non_blocking=True)

    step_e2e = e2e_body
    graphs = []
    if use_graph:
        # One decode step captured once and replayed: no per-launch host work
        # inside the timed loop.
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
    clocks = ClockSampler(dev.index) if clocks_on else None
    if clocks:
        clocks.mark_start()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark_end()
    clk = clocks.stop() if clocks else None
    ms = a.elapsed_time(b) / steps
    if _native.device_error() != 0:
        raise RuntimeError("device error word set during the layer bench")
    a2, b2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a2.record(stream)
    for _ in range(steps):
        step_e2e()
    b2.record(stream)
    torch.cuda.synchronize()
    e2e_ms = a2.elapsed_time(b2) / steps
    t = torch.tensor([ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms = t.tolist()
    # Graphs that captured NCCL collectives must be freed before the process
    # group is destroyed (destroying it first hangs at exit).
    step = step_e2e = None
    graphs.clear()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        if hasattr(layer, "close"):
            layer.close()  # unmap the peers' buffers before any rank frees its own
        dist.barrier()
    kv_bytes = B * (ctx + warmup + steps) * HKV * 128 * 4  # approx. mid-run lengths
    # this library's kernels per step: QKV (rms_split, GEMM, reduce; KV append fused),
    # attention (1), O-proj (GEMM, reduce), gate/up (rms_split, GEMM, reduce), down
    # (GEMM, reduce); under TP with peer stores + 5 stage barriers and a separate append
    # hybrid: QKV and O-proj on B/P rows take the weight-streaming path (1 launch each) at B/P <= 16,
    # the tcgen05 path (3 and 2) above; + attention, gate/up (3), down (2) and 3 barriers
    launches = 11 if (world == 1 or dp) else {"peer": 18, "hybrid": 11 if Bl <= 16 else 14}.get(tp_mode, 13)
    del k, v, layer
    torch.cuda.empty_cache()
    return {"ms_per_step": ms, "e2e_ms_per_step": e2e_ms, "bytes_per_step": wbytes * (world if dp else 1) + kv_bytes,
            "launches_per_step": launches, "clocks": clk, "B": B, "ctx": ctx, "H": H, "F": F, "HQ": HQ, "HKV": HKV,
            "dp": dp}


def hybrid_parity(world, rank, dev) -> dict:
    """Small step of the hybrid layer against the single-GPU layer on the full
    batch (two eager steps, the hybrid output fed back as the next input), within
    the chained bf16 bound of the layer tests (max 5e-2, mean 1e-2 scaled error),
    and one CUDA-graph replay bit-identical to an eager step on the same state."""
    import torch.distributed as dist

    from fused_kernels_cutedsl_lib_b200.layer import DecodeLayer, HybridDecodeLayer, random_layer_weights

    B, L, H, F, HQ, HKV = 8 * world, 300, 4096, 14336, 32, 8
    full = random_layer_weights(H, F, HQ, HKV, seed=21, device=dev)
    g = torch.Generator(device=dev).manual_seed(22)
    x = torch.randn(B, H, generator=g, device=dev).bfloat16()
    k = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
    v = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
    lens = torch.tensor([200 + 5 * i for i in range(B)], dtype=torch.int32, device=dev)
    Bl = B // world
    rows = slice(rank * Bl, (rank + 1) * Bl)
    kh, vh, lh = k[rows].clone(), v[rows].clone(), lens[rows].clone()  # the single-GPU layer appends to k, v
    hyb = HybridDecodeLayer(full, num_heads_q=HQ, num_heads_kv=HKV)
    single = DecodeLayer(full, HQ, HKV)
    worst_max = worst_mean = 0.0
    xh = x
    for _ in range(2):
        ys = single(xh, k, v, lens).clone()
        yh = hyb(xh, kh, vh, lh).clone()
        torch.cuda.synchronize()
        e = (yh.float() - ys.float()).abs() / ys.float().abs().clamp_min(1.0)
        worst_max, worst_mean = max(worst_max, e.max().item()), max(worst_mean, e.mean().item())
        xh = yh
    kg, vg, lg, xg = kh.clone(), vh.clone(), lh.clone(), xh.clone()
    y_eager = hyb(xh, kh, vh, lh).clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        yg = hyb(xg, kg, vg, lg)
    graph.replay()
    torch.cuda.synchronize()
    same = torch.equal(yg, y_eager) and torch.equal(kg, kh) and torch.equal(lg, lh)
    del graph
    dist.barrier()
    hyb.close()
    dist.barrier()
    flags = torch.tensor([0.0 if same else 1.0, worst_max, worst_mean], dtype=torch.float64, device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    same = flags[0].item() == 0.0
    worst_max, worst_mean = flags[1].item(), flags[2].item()
    del full, k, v, single
    torch.cuda.empty_cache()
    return {"ok": bool(same and worst_max <= 5e-2 and worst_mean <= 1e-2), "graph_vs_eager_bitwise": bool(same),
            "vs_single_gpu_max_scaled_err": round(worst_max, 5), "vs_single_gpu_mean_scaled_err": round(worst_mean, 6),
            "case": f"B={B}, L~300, hidden 4096, ffn 14336, 32q/8kv: 2 eager steps + 1 graph replay"}


def tp_parity(world, rank, dev) -> dict:
    """Small tensor-parallel step, bitwise: the peer-memory layer against the NCCL
    all-gather layer (two eager steps and one CUDA-graph replay, y fed back as x),
    and both against the single-GPU layer on the full batch within the chained
    bf16 bound of the layer tests (max 5e-2, mean 1e-2 scaled error)."""
    import torch.distributed as dist

    from fused_kernels_cutedsl_lib_b200.layer import (DecodeLayer, PeerTPDecodeLayer, TPDecodeLayer,
                                                      random_layer_weights, shard_layer_weights)

    B, L, H, F, HQ, HKV = 8 * world, 300, 4096, 14336, 32, 8
    full = random_layer_weights(H, F, HQ, HKV, seed=21, device=dev)
    shard = shard_layer_weights(full, rank, world, HQ, HKV)
    g = torch.Generator(device=dev).manual_seed(22)
    x = torch.randn(B, H, generator=g, device=dev).bfloat16()
    k = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
    v = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
    lens = torch.tensor([200 + 5 * i for i in range(B)], dtype=torch.int32, device=dev)
    Bl = B // world
    rows = slice(rank * Bl, (rank + 1) * Bl)
    kn, vn, ln = k[rows].contiguous(), v[rows].contiguous(), lens[rows].contiguous()
    kp, vp, lp = kn.clone(), vn.clone(), ln.clone()
    ks, vs, ls = k.clone(), v.clone(), lens.clone()
    nccl_layer = TPDecodeLayer(shard, num_heads_q=HQ, num_heads_kv=HKV)
    peer_layer = PeerTPDecodeLayer(shard, num_heads_q=HQ, num_heads_kv=HKV)
    single = DecodeLayer(full, HQ, HKV)
    same, worst_max, worst_mean = True, 0.0, 0.0
    xn = xp = xs = x
    for _ in range(2):
        xn = nccl_layer(xn, kn, vn, ln).clone()
        xp = peer_layer(xp, kp, vp, lp).clone()
        ys = single(xs, ks, vs, ls).clone()
        torch.cuda.synchronize()
        same &= torch.equal(xn, xp)
        e = (xp.float() - ys.float()).abs() / ys.float().abs().clamp_min(1.0)
        worst_max, worst_mean = max(worst_max, e.max().item()), max(worst_mean, e.mean().item())
        xs = xp  # compare one step at a time: feed the TP output to both
    xg = xp.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        yg = peer_layer(xg, kp, vp, lp)
    xn = nccl_layer(xn, kn, vn, ln).clone()
    graph.replay()
    torch.cuda.synchronize()
    same &= torch.equal(xn, yg)
    del graph
    same &= torch.equal(kn, kp) and torch.equal(vn, vp) and torch.equal(ln, lp)
    dist.barrier()
    peer_layer.close()
    dist.barrier()
    flags = torch.tensor([0.0 if same else 1.0, worst_max, worst_mean], dtype=torch.float64, device=dev)
    dist.all_reduce(flags, op=dist.ReduceOp.MAX)
    same = flags[0].item() == 0.0
    worst_max, worst_mean = flags[1].item(), flags[2].item()
    ok = same and worst_max <= 5e-2 and worst_mean <= 1e-2
    del full, shard, k, v, single, nccl_layer, peer_layer
    torch.cuda.empty_cache()
    return {"ok": bool(ok), "peer_vs_nccl_bitwise": bool(same), "vs_single_gpu_max_scaled_err": round(worst_max, 5),
            "vs_single_gpu_mean_scaled_err": round(worst_mean, 6),
            "case": f"B={B}, L~300, hidden 4096, ffn 14336, 32q/8kv: 2 eager steps + 1 graph replay"}


def _roof(bytes_, us, peak, peak_kind):
    gbs = bytes_ / (us * 1e-6) / 1e9
    return {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s", "frac": round(gbs / peak, 4),
            "peak_kind": peak_kind}


def _cpu_linear(kind, M, N, K, budget_s=3.0):
    """Oracle port of a config-3/4 GEMM on the host: a slice of the weight rows, timed."""
    import oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = min(N, 2048)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(2 * rows if kind == "swiglu" else rows, K, generator=g) * 0.02).bfloat16()
    gamma = (1 + 0.1 * torch.randn(K, generator=g)).bfloat16()
    done, t_used, n = 0, 0.0, 0
    while t_used < budget_s and n < 100:
        t0 = time.perf_counter()
        if kind == "swiglu":
            oracle.swiglu(x, w)
        elif kind == "rmsnorm":
            oracle.rmsnorm_linear(x, gamma, w)
        else:
            oracle.linear(x, w)
        t_used += time.perf_counter() - t0
        done += w.numel() * 2
        n += 1
    return {"value": round(done / t_used / 1e12, 6), "unit": "TB/s", "cores": threads, "kind": "port",
            "sample": f"{n} passes over {w.shape[0]} of the weight rows (M={M}, K={K}), fp32 torch on CPU, "
                      f"{t_used:.1f} s"}


def _cpu_layer(budget_s=5.0):
    """Oracle port of one decode-layer step for one sequence at context 8192, on the host."""
    import oracle
    from fused_kernels_cutedsl_lib_b200.layer import random_layer_weights

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = random_layer_weights(4096, 14336, 32, 8, seed=4, device="cpu")
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, 4096, generator=g).bfloat16()
    k = torch.randn(1, 8193, 8, 128, generator=g).bfloat16()
    v = torch.randn(1, 8193, 8, 128, generator=g).bfloat16()
    lens = torch.tensor([8192], dtype=torch.int32)
    n, t_used = 0, 0.0
    while t_used < budget_s and n < 20:
        t0 = time.perf_counter()
        oracle.decode_layer(x, w.as_dict(), k, v, lens, num_heads_q=32, num_heads_kv=8)
        t_used += time.perf_counter() - t0
        n += 1
    return {"value": round(n / t_used, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode steps of 1 sequence at context 8192 (fp32 torch on CPU), {t_used:.1f} s"}


def run_extras(args, world, rank, dev, cpu: bool) -> dict:
    """Configs 1, 3, 4 and 5 as sub-objects of the bench line, each with its
    roofline (measured peak) and, at N = 1, a CPU baseline (oracle port).
    N > 1: config 3 column-sharded over the ranks (each rank streams its own W
    rows; aggregate TB/s = all ranks' weight bytes / the slowest rank's time),
    the tensor-parallel layer step and its parity check; configs 1 and 4 are
    one-GPU shapes and run at N = 1 only."""
    import torch.distributed as dist

    from fused_kernels_cutedsl_lib_b200 import perf

    peak, kind = _peaks()
    out = {}
    t0 = time.perf_counter()
    floor = perf.launch_floor()

    def maxr(vals):
        t = torch.tensor(vals, dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    if world == 1:
        c1 = perf.bench_attention_config1()
        c1["launch_floor"] = floor
        c1["roofline"] = _roof(c1["algorithmic_bytes"], c1["us_isolated"], peak, kind)
        c1["roofline_back_to_back"] = _roof(c1["algorithmic_bytes"], c1["us_back_to_back"], peak, kind)
        c1["TBps_isolated"] = round(c1["algorithmic_bytes"] / (c1["us_isolated"] * 1e-6) / 1e12, 3)
        if cpu:
            from fused_kernels_cutedsl_lib_b200 import configs as _cf

            qh, kh, vh, lh = _cf.attn_inputs(_cf.ATTN_CONFIG1, device="cpu", batch_rows=[0])
            c1["cpu_baseline"] = cpu_baseline(_cf.ATTN_CONFIG1, qh, kh, vh, lh, budget_s=3.0)
        out["config1"] = c1

    # config 3: skinny (M <= 16) and tcgen05 (M >= 64) GEMM, K=4096, N=14336, column-sharded at N > 1
    sk = {"workload": "config 3: y = x W^T, K=4096, N=14336, W N(0,0.02) seed 2",
          "sharding": f"weight columns over {world} GPU(s), no collective", "launch_floor": floor, "cases": []}
    for M in (1, 16, 64, 256):
        r = perf.bench_linear_shard("plain", M, 14336, 4096, 2, rank, world, include_cublas=(world == 1))
        us_iso, us_b2b = maxr([r["us_isolated"], r["us_back_to_back"]])
        total_bytes = 14336 * 4096 * 2 + M * 4096 * 2 * world + M * 14336 * 2
        case = {"M": M, "path": r["path"], "N_per_gpu": r["N_local"], "us_isolated": us_iso, "us_back_to_back": us_b2b,
                "TBps_isolated": round(total_bytes / (us_iso * 1e-6) / 1e12, 3),
                "TBps_back_to_back": round(total_bytes / (us_b2b * 1e-6) / 1e12, 3),
                "roofline": _roof(r["bytes_local"], us_iso, peak, kind),
                "roofline_back_to_back": _roof(r["bytes_local"], us_b2b, peak, kind)}
        if M >= 64:
            tfl = r["flops_local"] / (us_b2b * 1e-6) / 1e12
            case["TFLOPs_back_to_back"] = round(tfl, 1)
        for key in ("torch_us_isolated", "torch_us_back_to_back"):
            if key in r:
                case[key] = r[key]
        if cpu and M in (1, 16):
            case["cpu_baseline"] = _cpu_linear("plain", M, 14336, 4096)
        sk["cases"].append(case)
    out["skinny_gemm"] = sk

    if world == 1:
        fu = {"workload": "config 4: RMSNorm->QKV (W [6144,4096], gamma 1+N(0,0.1), eps 1e-6) and "
                          "gate/up+SwiGLU (W [2x14336,4096]), seed 3", "cases": []}
        for name, kd, M, N in (("rmsnorm_qkv", "rmsnorm", 1, 6144), ("rmsnorm_qkv", "rmsnorm", 16, 6144),
                               ("rmsnorm_qkv", "rmsnorm", 128, 6144), ("swiglu_gate_up", "swiglu", 1, 14336),
                               ("swiglu_gate_up", "swiglu", 16, 14336), ("swiglu_gate_up", "swiglu", 128, 14336)):
            r = perf.bench_linear_shard(kd, M, N, 4096, 3)
            case = {"kernel": name, "M": M, "path": r["path"], "us_isolated": r["us_isolated"],
                    "us_back_to_back": r["us_back_to_back"],
                    "roofline": _roof(r["bytes_local"], r["us_isolated"], peak, kind),
                    "roofline_back_to_back": _roof(r["bytes_local"], r["us_back_to_back"], peak, kind),
                    "torch_us_isolated": r.get("torch_us_isolated"),
                    "torch_us_back_to_back": r.get("torch_us_back_to_back")}
            if cpu and M in (1, 16):
                case["cpu_baseline"] = _cpu_linear(kd, M, N, 4096)
            fu["cases"].append(case)
        out["fused"] = fu

    # config 5: the decode layer step (CUDA graphs), tensor-parallel at N > 1
    lay = layer_measure(args, world, rank, dev, steps=args.layer_steps, warmup=3, tp_mode=args.tp_mode,
                        use_graph=True, clocks_on=False)
    lo = {"ms_per_step": round(lay["ms_per_step"], 4), "tokens_per_s": round(lay["B"] / (lay["ms_per_step"] * 1e-3), 1),
          "e2e_ms_per_step": round(lay["e2e_ms_per_step"], 4),
          "parallelism": "single GPU" if world == 1 else (
              f"dp{world}" if lay["dp"] else
              (f"hybrid{world}: attention block batch-parallel (whole W_qkv, W_o), FFN column-parallel, "
               "exchanges in the epilogues over peer memory, 3 stage barriers" if args.tp_mode == "hybrid" else
               f"tp{world} GEMMs (column shards) + batch-sharded attention, "
               + ("all-gathers in the kernels' epilogues over peer memory" if args.tp_mode == "peer" else "NCCL"))),
          "steps": args.layer_steps, "cuda_graph": True, "launches_per_step": lay["launches_per_step"],
          "roofline": _roof(lay["bytes_per_step"] / world, lay["ms_per_step"] * 1e3, peak, kind)}
    if world > 1:
        lo["tp_parity"] = hybrid_parity(world, rank, dev) if args.tp_mode == "hybrid" else tp_parity(world, rank, dev)
        # the other decompositions of the same step, measured the same way
        modes = {args.tp_mode: lo["ms_per_step"]}
        for m in ("peer", "hybrid", "dp"):
            if m not in modes:
                r = layer_measure(args, world, rank, dev, steps=args.layer_steps, warmup=3, tp_mode=m, use_graph=True,
                                  clocks_on=False)
                modes[m] = round(r["ms_per_step"], 4)
        lo["ms_per_step_by_mode"] = modes
    if cpu:
        lo["cpu_baseline"] = _cpu_layer()
    out["layer_ms_per_step"] = lo["ms_per_step"]
    out["layer"] = lo
    return out


def run_layer(args):
    """Config 5 alone: full decoder-layer decode step, B=128 at context 8192 (tensor-parallel for N > 1)."""
    import datetime

    import torch.distributed as dist

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    r = layer_measure(args, world, rank, dev, steps=args.steps, warmup=args.warmup, tp_mode=args.tp_mode,
                      use_graph=not args.no_graph)
    if rank == 0:
        ms, e2e_ms, B = r["ms_per_step"], r["e2e_ms_per_step"], r["B"]
        peak, kind = _peaks()
        dp = r["dp"]
        print(json.dumps({
            "metric": "decode-layer tokens/s (Llama-3-8B-shaped layer, B=128, ctx 8192)",
            "value": round(B / (ms * 1e-3), 1), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights seed 4, N(0,1) KV)",
            "config": {"workload": "decode_layer_config5", "batch": B, "context": r["ctx"], "hidden": r["H"],
                       "ffn": r["F"], "heads_q": r["HQ"], "heads_kv": r["HKV"],
                       "parallelism": "single GPU" if world == 1 else (
                           f"dp{world}: batch-sharded layer, weights replicated, no collective" if dp else
                           f"hybrid{world}: attention block batch-parallel, FFN column-parallel, peer-memory "
                           "exchanges" if args.tp_mode == "hybrid" else
                           f"tp{world} GEMMs + batch-sharded attention, all-gathers "
                           + ("in the GEMM / attention epilogues over peer memory" if args.tp_mode == "peer"
                              else "by NCCL")),
                       "cuda_graph": not args.no_graph,
                       "l2": "weights 436 MB + KV 4.3 GB per step exceed L2"},
            "bytes_per_step": r["bytes_per_step"],
            "achieved_TBps": round(r["bytes_per_step"] / world / (ms * 1e-3) / 1e12, 3),
            "peak_GBps": peak, "peak_kind": kind,
            "e2e": {"value": round(B / (e2e_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": B * r["H"] * 2, "d2h_bytes_per_step": B * r["H"] * 2},
            "gpu_launches": args.steps * r["launches_per_step"],
            "clocks": r["clocks"],
        }), flush=True)
    if world > 1:
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
    ap.add_argument("--tp-mode", choices=["peer", "nccl", "hybrid", "dp"], default="peer",
                    help="layer workload on N > 1 GPUs: tensor-parallel GEMMs with the all-gathers in the kernels "
                         "over peer memory (peer) or by NCCL (nccl); attention block batch-parallel with the FFN "
                         "tensor-parallel over peer memory (hybrid); or batch-parallel with replicated weights (dp)")
    ap.add_argument("--workload", choices=["attention", "layer"], default="attention",
                    help="attention: config 2 split-KV decode attention (headline) plus, unless --no-extras, "
                         "configs 1, 3, 4 and the config-5 layer step as sub-objects of the same line; "
                         "layer: config 5 decode step alone")
    ap.add_argument("--no-extras", action="store_true", help="headline only (skip configs 1, 3, 4, 5)")
    ap.add_argument("--layer-steps", type=int, default=100, help="timed layer steps inside the default run")
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
