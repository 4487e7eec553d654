"""Multi-GPU work partitioning for the decode step (one process per GPU).

* Decode attention shards by batch row with no collective: each rank owns a
  set of rows (their KV cache lives only on that GPU) chosen by greedy
  longest-first balancing of the true lengths, since ragged rows make equal
  row counts uneven in bytes.
* GEMMs shard by output column (tensor parallel): rank p owns weight rows
  ``[p*N/P, (p+1)*N/P)``; the SwiGLU gate/up weight is sharded with the same
  column range in both halves so the epilogue stays local.

The reference has no multi-GPU code; this module is new for the decode path.
"""
from __future__ import annotations

import heapq

import torch


def balance_rows(seqlens, world_size: int) -> list[list[int]]:
    """Assign batch rows to ranks, longest first onto the least-loaded rank.

    Returns ``world_size`` sorted row lists. Deterministic: ties break by rank id.
    Every rank gets at least one row when ``len(seqlens) >= world_size``.
    """
    lens = [int(x) for x in (seqlens.tolist() if isinstance(seqlens, torch.Tensor) else seqlens)]
    order = sorted(range(len(lens)), key=lambda i: (-max(lens[i], 0), i))
    heap = [(0, r) for r in range(world_size)]
    heapq.heapify(heap)
    shards: list[list[int]] = [[] for _ in range(world_size)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        # +1 keeps zero-length rows spreading instead of piling on one rank
        heapq.heappush(heap, (load + max(lens[i], 0) + 1, r))
    return [sorted(s) for s in shards]


def column_range(n: int, rank: int, world_size: int, align: int = 128) -> tuple[int, int]:
    """Rank's output-column range ``[lo, hi)`` of an N-column GEMM, in ``align`` blocks."""
    if n % align != 0:
        raise ValueError(f"N={n} must be a multiple of {align} to shard by columns")
    blocks = n // align
    lo = (blocks * rank) // world_size
    hi = (blocks * (rank + 1)) // world_size
    return lo * align, hi * align


def shard_gate_up(w_gate_up: torch.Tensor, rank: int, world_size: int) -> torch.Tensor:
    """This rank's [2*n_local, K] slice of a [2N, K] gate/up weight (gate block, then up block)."""
    n = w_gate_up.shape[0] // 2
    lo, hi = column_range(n, rank, world_size)
    return torch.cat([w_gate_up[lo:hi], w_gate_up[n + lo:n + hi]], dim=0).contiguous()
