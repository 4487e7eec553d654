"""Host-side logic of the multi-GPU decode step on CPU ranks (gloo, world size 2).

The tensor-parallel layer's sharding, gathers and re-layouts run with the
compute steps replaced by the CPU oracle (test-only ops), and the result must
match the single-process oracle layer. Failure paths are injected on the host:
a rank that raises before a collective, seen by the peer as an error within a
short process-group timeout.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from fused_kernels_cutedsl_lib_b200.layer import LayerWeights, TPDecodeLayer, shard_layer_weights
from fused_kernels_cutedsl_lib_b200.sharding import balance_rows, column_range, shard_gate_up

HQ, HKV, HID, FFN = 4, 2, 512, 1024


class OracleOps:
    """CPU stand-ins for the kernels, with the kernels' bf16 output rounding."""

    def __init__(self, eps):
        self.eps = eps

    def rms_linear(self, x, gamma, w, out):
        out.copy_(oracle.rmsnorm_linear(x, gamma, w, self.eps).to(out.dtype))
        return out

    def linear(self, x, w, out, residual=None):
        y = oracle.linear(x, w)
        if residual is not None:
            y = y + residual.float()
        out.copy_(y.to(out.dtype))
        return out

    def rms_swiglu(self, x, gamma, w_gate_up, out):
        out.copy_(oracle.swiglu(oracle.rmsnorm(x, gamma, self.eps), w_gate_up).to(out.dtype))
        return out

    def append_and_attend(self, qkv, k_cache, v_cache, cache_seqlens, out):
        D = 128
        for b in range(qkv.shape[0]):
            L = int(cache_seqlens[b])
            k_cache[b, L] = qkv[b, HQ * D:(HQ + HKV) * D].view(HKV, D)
            v_cache[b, L] = qkv[b, (HQ + HKV) * D:].view(HKV, D)
            cache_seqlens[b] = L + 1
        o, _ = oracle.decode_attention(qkv[:, :HQ * D].reshape(-1, HQ, D), k_cache, v_cache, cache_seqlens)
        out.copy_(o.reshape(out.shape).to(out.dtype))
        return out


def _weights():
    g = torch.Generator().manual_seed(0)
    w = lambda *s: (torch.randn(*s, generator=g) * 0.05).bfloat16()
    gain = lambda n: (1 + 0.1 * torch.randn(n, generator=g)).bfloat16()
    return LayerWeights(gamma_attn=gain(HID), w_qkv=w((HQ + 2 * HKV) * 128, HID), w_o=w(HID, HQ * 128),
                        gamma_ffn=gain(HID), w_gate_up=w(2 * FFN, HID), w_down=w(HID, FFN))


def _inputs(B=4, L=64):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(B, HID, generator=g).bfloat16()
    k = torch.randn(B, L, HKV, 128, generator=g).bfloat16()
    v = torch.randn(B, L, HKV, 128, generator=g).bfloat16()
    lens = torch.tensor([40, 63, 10, 25], dtype=torch.int32)[:B]
    return x, k, v, lens


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=30))
        full = _weights()
        layer = TPDecodeLayer(shard_layer_weights(full, rank, world, HQ, HKV), num_heads_q=HQ, num_heads_kv=HKV,
                              ops=OracleOps(1e-6))
        x, k, v, lens = _inputs()
        Bl = x.shape[0] // world
        rows = slice(rank * Bl, (rank + 1) * Bl)
        y = layer(x, k[rows].clone(), v[rows].clone(), lens[rows].clone())
        q.put((rank, y.float()))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_tp_layer_matches_oracle_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for r in range(2):
        assert not isinstance(res[r], str), res[r]
    x, k, v, lens = _inputs()
    ref, *_ = oracle.decode_layer(x, _weights().as_dict(), k, v, lens, num_heads_q=HQ, num_heads_kv=HKV)
    for r in range(2):
        err = (res[r] - ref).abs() / ref.abs().clamp_min(1.0)
        assert err.max().item() < 2e-2, err.max().item()
    assert torch.equal(res[0], res[1])


def _failing_worker(rank, world, port, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if rank == 1:
            raise RuntimeError("injected failure before the all-gather")
        buf = torch.empty(2 * 4)
        dist.all_gather_into_tensor(buf, torch.ones(4))
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, type(e).__name__ + ": " + str(e)[:80]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_rank_failure_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert "injected" in res[1]
    assert res[0] != "no error"  # the surviving rank's collective errors out within the timeout


def test_sharding_helpers():
    lens = torch.tensor([100, 5, 80, 80, 0, 30, 60, 1])
    shards = balance_rows(lens, 3)
    assert sorted(sum(shards, [])) == list(range(8))
    loads = [sum(int(lens[i]) for i in s) for s in shards]
    assert max(loads) - min(loads) <= 100
    assert [column_range(14336, r, 8) for r in range(8)][3] == (5376, 7168)
    with pytest.raises(ValueError):
        column_range(100, 0, 2)
    w = torch.zeros(8, 3)  # 2N = 8 rows: N = 4 does not split into 128-column blocks
    with pytest.raises(ValueError):
        shard_gate_up(w, 0, 2)
    wg = torch.arange(512).reshape(512, 1).float()
    s1 = shard_gate_up(wg, 1, 2)
    assert s1[:128, 0].tolist() == list(range(128, 256)) and s1[128:, 0].tolist() == list(range(384, 512))
