"""Host-side partitioning logic: property tests of the sharding helpers and the
batch-parallel decomposition of the decode layer (CPU, oracle compute)."""
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

import oracle
from fused_kernels_cutedsl_lib_b200.sharding import balance_rows, column_range, shard_gate_up


@settings(max_examples=200, deadline=None)
@given(st.lists(st.integers(min_value=-3, max_value=40000), min_size=1, max_size=80), st.integers(1, 8))
def test_balance_rows_is_a_partition(lens, world):
    shards = balance_rows(lens, world)
    assert len(shards) == world
    flat = sorted(i for s in shards for i in s)
    assert flat == list(range(len(lens)))           # every row exactly once
    assert all(s == sorted(s) for s in shards)      # sorted row lists
    if len(lens) >= world:
        assert all(len(s) >= 1 for s in shards)     # nobody idle when rows suffice
    assert balance_rows(lens, world) == shards      # deterministic


@settings(max_examples=200, deadline=None)
@given(st.lists(st.integers(min_value=0, max_value=40000), min_size=8, max_size=80), st.integers(2, 8))
def test_balance_rows_load_bound(lens, world):
    """Longest-first greedy: the heaviest rank carries at most the mean plus one row."""
    shards = balance_rows(lens, world)
    loads = [sum(lens[i] + 1 for i in s) for s in shards]
    mean = sum(l + 1 for l in lens) / world
    assert max(loads) <= mean + max(lens) + 1


@settings(max_examples=200, deadline=None)
@given(st.integers(1, 64), st.integers(1, 8))
def test_column_ranges_tile_the_columns(blocks, world):
    n = 128 * blocks
    ranges = [column_range(n, r, world) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (lo, hi), (lo2, _) in zip(ranges, ranges[1:]):
        assert hi == lo2 and lo <= hi
    for lo, hi in ranges:
        assert lo % 128 == 0 and hi % 128 == 0
    sizes = [hi - lo for lo, hi in ranges]
    assert max(sizes) - min(sizes) <= 128


def test_shard_gate_up_keeps_gate_and_up_rows_together():
    n, k, world = 512, 8, 4
    w = torch.arange(2 * n * k, dtype=torch.float32).reshape(2 * n, k)
    parts = [shard_gate_up(w, r, world) for r in range(world)]
    for r, part in enumerate(parts):
        lo, hi = column_range(n, r, world)
        half = part.shape[0] // 2
        assert torch.equal(part[:half], w[lo:hi]) and torch.equal(part[half:], w[n + lo:n + hi])


def test_batch_parallel_layer_equals_the_whole_batch():
    """The decode layer is independent per sequence: running it on batch shards
    (replicated weights, no collective) gives the whole-batch result row for row."""
    g = torch.Generator().manual_seed(3)
    H, F, HQ, HKV, B, L = 256, 512, 4, 2, 6, 40

    def w(*s):
        return (0.05 * torch.randn(*s, generator=g)).bfloat16()

    weights = dict(gamma_attn=(1 + 0.1 * torch.randn(H, generator=g)).bfloat16(), w_qkv=w((HQ + 2 * HKV) * 128, H),
                   w_o=w(H, HQ * 128), gamma_ffn=(1 + 0.1 * torch.randn(H, generator=g)).bfloat16(),
                   w_gate_up=w(2 * F, H), w_down=w(H, F))
    x = torch.randn(B, H, generator=g).bfloat16()
    k = torch.randn(B, L, HKV, 128, generator=g).bfloat16()
    v = torch.randn(B, L, HKV, 128, generator=g).bfloat16()
    lens = torch.tensor([5, 39, 17, 0, 22, 30], dtype=torch.int32)
    y, k1, v1, l1 = oracle.decode_layer(x, weights, k, v, lens, num_heads_q=HQ, num_heads_kv=HKV)
    for rows in (slice(0, 2), slice(2, 3), slice(3, 6)):
        ys, ks, vs, ls = oracle.decode_layer(x[rows], weights, k[rows], v[rows], lens[rows], num_heads_q=HQ,
                                             num_heads_kv=HKV)
        assert torch.allclose(ys, y[rows], atol=1e-5, rtol=1e-5)
        assert torch.equal(ls, l1[rows])


def test_default_num_splits_pins_the_measured_shapes():
    """The split rule at the measured shapes: config 1 takes 4 splits (1024-token
    chunks, 128 units), config 2 takes 32 (1024-token chunks) with or without its
    true token count, and a case too small for even 64-token chunks to give one
    unit for three quarters of the SMs falls back to 64-token chunks."""
    from fused_kernels_cutedsl_lib_b200 import chunk_tokens, configs, default_num_splits

    assert default_num_splits(4, 8, 4096) == 4
    assert chunk_tokens(4096, 4) == 1024
    c2 = configs.ATTN_CONFIG2
    lens = configs.attn_seqlens(c2)
    assert default_num_splits(64, 8, 32768, int(lens.sum())) == 32
    assert default_num_splits(64, 8, 32768) == 32
    # 1 row x 1 kv head x 4096 tokens: 64 units even at 64-token chunks, below the threshold
    assert default_num_splits(1, 1, 4096) == 64
    assert chunk_tokens(4096, 64) == 64
    # every split count gives chunks that are multiples of the 64-token tile
    for L in (1, 63, 64, 65, 1000, 4096, 32768):
        for S in (1, 2, 3, 7, 64):
            c = chunk_tokens(L, S)
            assert c % 64 == 0 and c * S >= L


def test_plan_attention_picks_the_form_by_work_per_cta():
    """Config 1 (7 padded tiles per resident CTA) takes the two-launch form with
    4 chunks; config 2 and the decode layer's batches take the single launch
    with enough partial slots; every single-launch plan has >= 2 slots."""
    from fused_kernels_cutedsl_lib_b200 import fused_partial_slots, plan_attention

    assert plan_attention(4, 8, 4096) == (False, 4)
    assert plan_attention(64, 8, 32768) == (True, 4)
    assert plan_attention(128, 8, 8256)[0]
    for B in (1, 2, 16, 64, 128, 1024):
        for L in (64, 1000, 8256, 32768):
            single, S = plan_attention(B, 8, L)
            assert S >= (2 if single else 1)
            s = fused_partial_slots(B, 8, L)
            assert 2 <= s <= -(-L // 64) + 1
