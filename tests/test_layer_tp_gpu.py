"""Tensor-parallel decode step on 2 GPUs (NCCL) against the single-GPU layer and the oracle."""
import datetime
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu

needs_2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                             reason="needs 2 GPUs")


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        import oracle
        from fused_kernels_cutedsl_lib_b200 import _native
        from fused_kernels_cutedsl_lib_b200.layer import TPDecodeLayer, random_layer_weights, shard_layer_weights

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        B, L, H, F, HQ, HKV = 16, 300, 4096, 14336, 32, 8
        full = random_layer_weights(H, F, HQ, HKV, seed=11, device=dev)
        g = torch.Generator(device=dev).manual_seed(12)
        x = torch.randn(B, H, generator=g, device=dev).bfloat16()
        k = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
        v = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
        lens = torch.tensor([250 + 3 * i for i in range(B)], dtype=torch.int32, device=dev)
        ref, *_ = oracle.decode_layer(x, full.as_dict(), k, v, lens, num_heads_q=HQ, num_heads_kv=HKV)
        Bl = B // world
        rows = slice(rank * Bl, (rank + 1) * Bl)
        layer = TPDecodeLayer(shard_layer_weights(full, rank, world, HQ, HKV), num_heads_q=HQ, num_heads_kv=HKV)
        kr, vr, lr = k[rows].contiguous(), v[rows].contiguous(), lens[rows].contiguous()
        y = layer(x, kr, vr, lr)
        torch.cuda.synchronize()
        err = ((y.float().cpu() - ref).abs() / ref.abs().clamp_min(1.0))
        q.put((rank, err.max().item(), err.mean().item(), lr.cpu().tolist(), _native.device_error()))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, repr(e), None, None, None))


@needs_2
def test_tp2_layer_matches_oracle():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r[0]: r for r in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        _, mx, mean, lens, derr = res[r]
        assert not isinstance(mx, str), mx
        assert derr == 0
        assert mx <= 5e-2 and mean <= 1e-2, (mx, mean)  # chained bound, as for the single-GPU layer
        assert lens == [251 + 3 * i for i in range(r * 8, r * 8 + 8)]


def _peer_worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        from fused_kernels_cutedsl_lib_b200 import _native
        from fused_kernels_cutedsl_lib_b200.layer import (PeerTPDecodeLayer, TPDecodeLayer, random_layer_weights,
                                                          shard_layer_weights)

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        res = {}
        for B in (2 * world if world <= 8 else 16, 64):  # skinny (M <= 16) and tcgen05 GEMM paths
            L, H, F, HQ, HKV = 300, 1024 * max(1, world // 2), 2048 * max(1, world // 2), 16, 8
            full = random_layer_weights(H, F, HQ, HKV, seed=21, device=dev)
            shard = shard_layer_weights(full, rank, world, HQ, HKV)
            g = torch.Generator(device=dev).manual_seed(22)
            x = torch.randn(B, H, generator=g, device=dev).bfloat16()
            Bl = B // world
            k = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
            v = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
            lens = torch.tensor([200 + 5 * i for i in range(B)], dtype=torch.int32, device=dev)
            rows = slice(rank * Bl, (rank + 1) * Bl)
            kn, vn, ln = k[rows].contiguous(), v[rows].contiguous(), lens[rows].contiguous()
            kp, vp, lp = kn.clone(), vn.clone(), ln.clone()
            nccl_layer = TPDecodeLayer(shard, num_heads_q=HQ, num_heads_kv=HKV)
            peer_layer = PeerTPDecodeLayer(shard, num_heads_q=HQ, num_heads_kv=HKV)
            same = True
            xn = xp = x
            for _ in range(2):  # two eager steps, each feeding y back as x
                xn = nccl_layer(xn, kn, vn, ln).clone()
                xp = peer_layer(xp, kp, vp, lp).clone()
                torch.cuda.synchronize()
                same &= torch.equal(xn, xp)
            # CUDA graph of one peer step, replayed: the barrier counter lives on the device
            xg = xp.clone()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                yg = peer_layer(xg, kp, vp, lp)
            for _ in range(3):
                xn = nccl_layer(xn, kn, vn, ln).clone()
                graph.replay()
                torch.cuda.synchronize()
                same &= torch.equal(xn, yg)
                xg.copy_(yg)
            del graph
            same &= torch.equal(kn, kp) and torch.equal(vn, vp) and torch.equal(ln, lp)
            peer_layer.close()
            res[B] = same
        q.put((rank, res, _native.device_error()))
        dist.destroy_process_group()
    except Exception as e:
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()[-800:], None))


@needs_2
def test_tp_peer_memory_layer_matches_nccl_layer():
    """GEMM epilogues and attention pass 2 push their output blocks into every
    rank's buffer (CUDA IPC), with a stage barrier kernel: bit-identical to the
    NCCL all-gather layer, eager and under CUDA-graph replay. Runs on every GPU
    present (2 to 8 ranks)."""
    import torch.multiprocessing as mp

    world = min(8, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r[0]: r for r in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        _, same, derr = res[r]
        assert isinstance(same, dict), same
        assert derr == 0
        assert all(same.values()), same


def _hybrid_worker(rank, world, port, q):
    try:
        import torch.distributed as dist

        from fused_kernels_cutedsl_lib_b200 import _native
        from fused_kernels_cutedsl_lib_b200.layer import DecodeLayer, HybridDecodeLayer, random_layer_weights

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        res = {}
        for B in (8 * world, 64):
            if B % world:
                continue
            L, H, F, HQ, HKV = 300, 4096, 14336, 32, 8
            full = random_layer_weights(H, F, HQ, HKV, seed=31, device=dev)
            g = torch.Generator(device=dev).manual_seed(32)
            x = torch.randn(B, H, generator=g, device=dev).bfloat16()
            k = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
            v = torch.randn(B, L, HKV, 128, generator=g, device=dev).bfloat16()
            lens = torch.tensor([200 + (5 * i) % 90 for i in range(B)], dtype=torch.int32, device=dev)
            Bl = B // world
            rows = slice(rank * Bl, (rank + 1) * Bl)
            kh, vh, lh = k[rows].clone(), v[rows].clone(), lens[rows].clone()
            ks, vs, ls = k.clone(), v.clone(), lens.clone()
            hyb = HybridDecodeLayer(full, num_heads_q=HQ, num_heads_kv=HKV)
            single = DecodeLayer(full, HQ, HKV)
            worst_max = worst_mean = 0.0
            xh = x
            for _ in range(2):  # two eager steps; the single-GPU layer gets the same input each step
                ys = single(xh, ks, vs, ls).clone()
                yh = hyb(xh, kh, vh, lh).clone()
                torch.cuda.synchronize()
                e = (yh.float() - ys.float()).abs() / ys.float().abs().clamp_min(1.0)
                worst_max, worst_mean = max(worst_max, e.max().item()), max(worst_mean, e.mean().item())
                xh = yh
            cache_ok = torch.equal(lh, ls[rows]) and torch.equal(lh.cpu(), (lens[rows] + 2).cpu())
            # a CUDA graph of one step replays to the same bits as an eager step on the same state
            kg, vg, lg = kh.clone(), vh.clone(), lh.clone()
            xg = xh.clone()
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
            res[B] = (worst_max, worst_mean, cache_ok, same)
        q.put((rank, res, _native.device_error()))
        dist.destroy_process_group()
    except Exception as e:
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()[-800:], None))


@needs_2
def test_hybrid_layer_matches_single_gpu_layer():
    """Attention block batch-parallel (whole W_qkv / W_o), FFN column-parallel, exchanges
    by peer stores: within the chained bound of the single-GPU layer, KV caches
    and lengths advanced, and a CUDA-graph replay equal to an eager step. Runs on
    every GPU present (2 to 8 ranks)."""
    import torch.multiprocessing as mp

    world = min(8, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_hybrid_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {r[0]: r for r in (q.get(timeout=300) for _ in procs)}
    for p in procs:
        p.join(timeout=120)
    for r in range(world):
        _, out, derr = res[r]
        assert isinstance(out, dict), out
        assert derr == 0
        for B, (mx, mean, cache_ok, same) in out.items():
            assert mx <= 5e-2 and mean <= 1e-2, (B, mx, mean)
            assert cache_ok and same, (B, cache_ok, same)
