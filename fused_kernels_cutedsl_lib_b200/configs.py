"""The decode-step workloads (the reference project's benchmark configs) and seeded input builders.

Config numbering follows the project's benchmark list:
  1. decode attention, contiguous cache: B=4, Hq=32, Hkv=8, D=128, L=4096, seed 0
  2. split-KV ragged: B=64, Lmax=32768, lengths ~U[512, 32768] (seed 1)
  3. skinny GEMM y = x W^T: K=4096, N=14336, M in {1,4,8,16,64,256}, seed 2
  4. RMSNorm->QKV (W [6144,4096], M in {1,16,128}) and SwiGLU (W [2*14336, 4096]), seed 3
  5. Llama-3-8B-shaped decoder-layer decode step, B=128 at context 8192, seed 4

The reference benchmarks on random tensors only (no dataset); these builders
are the whole workload. Inputs are bf16 N(0,1) (weights N(0, 0.02)), drawn
with the stated seeds.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

HIDDEN = 4096
FFN = 14336
HQ = 32
HKV = 8
HEAD_DIM = 128


@dataclass(frozen=True)
class AttnConfig:
    name: str
    batch: int
    max_seqlen: int
    num_heads_q: int = HQ
    num_heads_kv: int = HKV
    ragged: bool = False
    min_len: int = 512
    seed: int = 0

    def kv_bytes(self, seqlens: torch.Tensor) -> int:
        """Algorithmic KV bytes: every valid token's K and V row for every kv head."""
        return int(seqlens.to(torch.int64).clamp(0, self.max_seqlen).sum()) * self.num_heads_kv * HEAD_DIM * 2 * 2

    def io_bytes(self) -> int:
        """q + out (bf16) + lse (fp32)."""
        return self.batch * self.num_heads_q * (HEAD_DIM * 2 * 2 + 4)


ATTN_CONFIG1 = AttnConfig("decode_attn_contiguous_b4_l4096", batch=4, max_seqlen=4096, seed=0)
ATTN_CONFIG2 = AttnConfig("splitkv_ragged_b64_l32768", batch=64, max_seqlen=32768, ragged=True,
                          min_len=512, seed=1)


def attn_seqlens(cfg: AttnConfig) -> torch.Tensor:
    """int32 cache lengths on the CPU: all max_seqlen, or U[min_len, max_seqlen] from the seed."""
    if not cfg.ragged:
        return torch.full((cfg.batch,), cfg.max_seqlen, dtype=torch.int32)
    g = torch.Generator().manual_seed(cfg.seed)
    return torch.randint(cfg.min_len, cfg.max_seqlen + 1, (cfg.batch,), generator=g, dtype=torch.int64).to(torch.int32)


def attn_inputs(cfg: AttnConfig, device="cuda", batch_rows: list[int] | None = None):
    """(q [B,1,Hq,D], k_cache, v_cache [B,Lmax,Hkv,D], cache_seqlens [B]) on ``device``.

    ``batch_rows`` selects a subset of rows (for sharding): the full batch is
    drawn row by row from per-row seeds so any subset reproduces the same rows.
    """
    rows = list(range(cfg.batch)) if batch_rows is None else list(batch_rows)
    lens = attn_seqlens(cfg)[rows]
    B = len(rows)
    q = torch.empty(B, 1, cfg.num_heads_q, HEAD_DIM, dtype=torch.bfloat16, device=device)
    k = torch.empty(B, cfg.max_seqlen, cfg.num_heads_kv, HEAD_DIM, dtype=torch.bfloat16, device=device)
    v = torch.empty_like(k)
    gen = torch.Generator(device=device)
    for i, r in enumerate(rows):
        gen.manual_seed(cfg.seed * 1_000_003 + r)
        q[i].normal_(generator=gen)
        k[i].normal_(generator=gen)
        v[i].normal_(generator=gen)
    return q, k, v, lens.to(device)


@dataclass(frozen=True)
class GemmConfig:
    name: str
    m: int
    n: int
    k: int
    seed: int

    def weight_bytes(self) -> int:
        return self.n * self.k * 2


def gemm_inputs(m: int, n: int, k: int, seed: int, device="cuda", w_std: float = 0.02):
    gen = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(m, k, generator=gen, device=device, dtype=torch.float32).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=gen, device=device, dtype=torch.float32) * w_std).to(torch.bfloat16)
    return x, w
