// Split-KV decode attention for sm_100a (flash-decoding, GQA-packed).
//
// Replaces the reference's decode attention (`DAttn1`,
// python/cutedsl_kernels/decoding_attention/attn1.py:62-307, one CTA per head,
// no softmax, no split) with the softmax semantics of the reference's own
// attention references (`attn_reimpl`, attn/attempt6_epi_pipeline/attn.py:778-784;
// exp2-domain online softmax with the zero/NaN row-sum guard,
// attn/attempt6_epi_pipeline/my_softmax.py:35-105).
//
// Pass 1 (`splitkv_fwd_kernel`): a persistent grid walks work units
// (batch row b, kv head h, split s). Split s of row b covers tokens
// [s*chunk, min((s+1)*chunk, L_b)); rows contribute ceil(L_b/chunk) splits, so
// every unit is `chunk` tokens long except the tails and units are dealt to
// CTAs round-robin (balanced to within one unit, empty splits never launch).
//   * one producer warp streams K and V tiles (64 tokens x 128 dims, two
//     128B-swizzled TMA boxes each) through a STAGES-deep mbarrier ring;
//   * four consumer warps each own 16 tokens of every tile. The G query heads
//     of the GQA group are the N=8 side of mma.sync m16n8k16 (tokens are the
//     M side), so every K/V byte is read from HBM once for all G heads;
//   * each warp keeps its own exp2-domain online softmax state; at the end of
//     a unit the four states are merged through shared memory and the unit
//     writes its normalised fp32 partial O and natural-log LSE.
// Pass 2 (`combine_kernel`): one warp per (b, q head) merges the splits
// LSE-weighted and writes bf16 O and fp32 LSE.
#include <math.h>

#include <type_traits>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace attn {

constexpr int D = 128;                     // head_dim
constexpr int T = 64;                      // tokens per KV tile
constexpr int NCW = 4;                     // consumer warps (16 tokens each)
constexpr int NTHREADS = (NCW + 2) * 32;   // + one TMA producer warp + one finisher warp
constexpr int NF = 4;                      // finisher hand-off ring depth (units)
constexpr int HALF_BYTES = T * 128;        // 64 tokens x 64 dims x 2 B
constexpr int TILE_BYTES = 2 * HALF_BYTES; // K (or V) tile: 16 KB
constexpr int STAGE_BYTES = 2 * TILE_BYTES;// K + V: 32 KB

struct Params {
  const __nv_bfloat16* q;  // row b at q + b * q_stride: [Hq, D] contiguous
  long long q_stride;      // elements between batch rows of q (Hq * D when dense)
  const int* block_table;  // paged cache: [B, max_blocks] physical block of each logical block (or null)
  int max_blocks, block_size;
  const int* seqlens;      // [B]
  float* o_part;           // [S, B, Hq, D]
  float* lse_part;         // [S, B, Hq]
  int* err;
  int B, Lmax, Hq, Hkv, G, chunk;
  float scale_log2;
  // Single-launch form (counters != null): the last unit of each (row, kv head)
  // to finish merges that pair's splits and writes out / lse itself.
  int* counters;           // [B * Hkv], zero between calls (each finisher resets its entry)
  __nv_bfloat16* out;      // [B, Hq, D]
  float* lse;              // [B, Hq]
  int* seqlens_commit;     // optional: receives cache_seqlens[b] once row b is done with it
  OutPlace peers;          // optional copies of out rows in other GPUs' buffers
  int nseg_cap;            // single-launch form: partial slots per pair (leading dim of o_part), >= 2
  int withhold_tile;       // test hook: CTA 0's producer skips its n-th tile (-1: never)
};

__device__ __forceinline__ int seq_len(const Params& p, int b) {
  int L = __ldg(p.seqlens + b);
  return min(max(L, 0), p.Lmax);
}

// Walks the unit space (b-major, then h, then s) monotonically.
struct Walker {
  int b;
  int nb;          // splits of row b
  long long base;  // first unit of row b
  __device__ void init(const Params& p) {
    b = 0;
    base = 0;
    nb = (seq_len(p, 0) + p.chunk - 1) / p.chunk;
  }
  __device__ bool locate(const Params& p, long long u, int& bo, int& ho, int& so) {
    while (true) {
      if (b >= p.B) return false;
      long long cnt = (long long)nb * p.Hkv;
      if (u < base + cnt) break;
      base += cnt;
      ++b;
      if (b < p.B) nb = (seq_len(p, b) + p.chunk - 1) / p.chunk;
    }
    int r = (int)(u - base);
    bo = b;
    ho = r / nb;
    so = r - ho * nb;
    return true;
  }
};

// LSE-weighted merge of the n splits of one (row, q head) by one warp; lane owns
// dims [4*lane, 4*lane+4). kFresh: the partials were written by this grid
// (read through L2 with ld.global.cg, not the non-coherent path). Writes bf16 out
// (and its peer copies) and the natural-log lse. The sums run in split order, so
// both launch forms give the same bits.
template <bool kFresh>
__device__ __forceinline__ float ld_part(const float* p) {
  return kFresh ? __ldcg(p) : __ldg(p);
}
template <bool kFresh>
__device__ __forceinline__ float4 ld_part4(const float* p) {
  return kFresh ? __ldcg(reinterpret_cast<const float4*>(p)) : __ldg(reinterpret_cast<const float4*>(p));
}

template <bool kFresh>
__device__ __forceinline__ void combine_row(const float* o_part, const float* lse_part, size_t plane, size_t row,
                                            int n, int lane, __nv_bfloat16* out, float* lse, const OutPlace& peers) {
  constexpr int CH = 8;  // splits whose loads are in flight together
  float ls[CH];
  float4 v[CH];
  auto load_chunk = [&](int s0) {
#pragma unroll
    for (int u = 0; u < CH; ++u) {
      if (s0 + u < n) {
        ls[u] = ld_part<kFresh>(lse_part + (s0 + u) * plane + row);
        v[u] = ld_part4<kFresh>(o_part + ((s0 + u) * plane + row) * D + 4 * lane);
      } else {
        ls[u] = -INFINITY;
        v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  // The max over the splits' LSEs (exact, order-free). Up to 8 splits it comes
  // from the first chunk itself, so the whole merge is one round trip to L2.
  float M = -INFINITY;
  if (n <= CH) {
    load_chunk(0);
#pragma unroll
    for (int u = 0; u < CH; ++u) M = fmaxf(M, ls[u]);
  } else {
    for (int s = lane; s < n; s += 32) M = fmaxf(M, ld_part<kFresh>(lse_part + s * plane + row));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  }
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float W = 0.f;
  if (M != -INFINITY) {
    // The weighted sum runs in split order whatever the chunking.
    for (int s0 = 0; s0 < n; s0 += CH) {
      if (n > CH) load_chunk(s0);
#pragma unroll
      for (int u = 0; u < CH; ++u) {
        if (s0 + u < n) {
          const float wgt = expf(ls[u] - M);
          W += wgt;
          acc.x += wgt * v[u].x;
          acc.y += wgt * v[u].y;
          acc.z += wgt * v[u].z;
          acc.w += wgt * v[u].w;
        }
      }
    }
  }
  const bool ok = W > 0.f;
  const float inv = ok ? 1.f / W : 0.f;
  uint2 packed;
  packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  reinterpret_cast<uint2*>(out + row * D)[lane] = packed;
#pragma unroll
  for (int i = 0; i < kMaxPeers; ++i)  // the same rows in other GPUs' buffers (all-gather of a batch shard)
    if (i < peers.npeers) reinterpret_cast<uint2*>(peers.peer_y[i] + row * D)[lane] = packed;
  if (lane == 0) lse[row] = ok ? M + logf(W) : -INFINITY;
}

__device__ __forceinline__ uint32_t keep_mask(bool lo, bool hi) {
  return (lo ? 0x0000FFFFu : 0u) | (hi ? 0xFFFF0000u : 0u);
}

__device__ __forceinline__ int seq_tiles(const Params& p, int b) { return (seq_len(p, b) + T - 1) / T; }

// A run of consecutive 64-token tiles [i0, i1) of one (row b, kv head h) that
// one CTA processes; its partial goes to split slot `slot` of the pair's
// `nseg` slots. `final_of_cta`: the CTA has no work after it.
struct Seg {
  int b, h, i0, i1, slot, nseg;
  bool final_of_cta;
};

// Two-launch form: units (b, h, split of `chunk` tokens) dealt round-robin.
struct ChunkIter {
  Walker w;
  long long u;
  __device__ void init(const Params& p) {
    w.init(p);
    u = blockIdx.x;
  }
  __device__ bool next(const Params& p, Seg& sg) {
    int b, h, s;
    if (!w.locate(p, u, b, h, s)) return false;
    const int tpc = p.chunk / T;
    sg.b = b;
    sg.h = h;
    sg.i0 = s * tpc;
    sg.i1 = min(sg.i0 + tpc, seq_tiles(p, b));
    sg.slot = s;
    sg.nseg = w.nb;
    sg.final_of_cta = false;
    u += gridDim.x;
    return true;
  }
};

// Single-launch form (stream-K over tiles): the (row, kv head, tile) order is
// cut into `G` contiguous ranges of equal length; CTA c owns
// [c*total/G, (c+1)*total/G). A range that crosses a pair boundary gives one
// segment per pair, and a pair's segments come from consecutive CTAs, so the
// segment of CTA c writes slot c - owner(first tile of the pair).
struct StreamIter {
  long long t, t_end, total;
  int G, b, nt;
  long long row_base;
  __device__ long long start(int c) const { return (long long)c * total / G; }
  __device__ int owner(long long x) const { return (int)(((x + 1) * (long long)G - 1) / total); }
  __device__ void init(const Params& p, long long total_tiles, int g) {
    total = total_tiles;
    G = g;
    const int c = blockIdx.x;
    t = c < G ? start(c) : 0;
    t_end = c < G ? start(c + 1) : 0;
    b = 0;
    row_base = 0;
    nt = p.B > 0 ? seq_tiles(p, 0) : 0;
  }
  __device__ bool next(const Params& p, Seg& sg) {
    if (t >= t_end) return false;
    while (t >= row_base + (long long)p.Hkv * nt) {  // t < total, so a later row holds it
      row_base += (long long)p.Hkv * nt;
      ++b;
      nt = seq_tiles(p, b);
    }
    const long long r = t - row_base;
    const int h = (int)(r / nt);
    const long long pb = row_base + (long long)h * nt;
    const long long pe = pb + nt;
    const long long se = t_end < pe ? t_end : pe;
    sg.b = b;
    sg.h = h;
    sg.i0 = (int)(t - pb);
    sg.i1 = (int)(se - pb);
    sg.slot = (int)blockIdx.x - owner(pb);
    sg.nseg = owner(pe - 1) - owner(pb) + 1;
    sg.final_of_cta = (se == t_end);
    t = se;
    return true;
  }
};

// Pass 1 (FUSED = false: chunked units, partials for pass 2) or the whole
// attention in one launch (FUSED = true: stream-K segments merged in-kernel).
// Two CTAs per SM (shared memory allows two): registers are capped to fit them.
template <int STAGES, bool FUSED>
__global__ void __launch_bounds__(NTHREADS, 2)
    splitkv_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, Params p) {
  using Iter = typename std::conditional<FUSED, StreamIter, ChunkIter>::type;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* cm = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES);  // [NCW][8] row max
  float* cl = cm + NCW * 8;                                           // [NCW][8] row sum
  float* co = cl + NCW * 8;                                           // [NCW][G][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(co + NCW * p.G * D);
  uint64_t* empty = full + STAGES;
  uint64_t* fin_full = empty + STAGES;  // [NF] a segment's partial is written (one arrival per consumer warp)
  uint64_t* fin_empty = fin_full + NF;  // [NF] the finisher is done with that hand-off slot
  volatile int* s_abort = reinterpret_cast<volatile int*>(fin_empty + NF);  // a consumer wait ran out
  volatile int* s_last = s_abort + 1;                                       // this CTA merges the pair
  volatile long long* s_total = reinterpret_cast<volatile long long*>(s_abort + 2);  // tiles in the batch

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    for (int i = 0; i < NF; ++i) {
      mbar_init(&fin_full[i], NCW);
      mbar_init(&fin_empty[i], 1);
    }
    *s_abort = 0;
    fence_barrier_init();
  }
  if (warp == NCW && lane == 0) {
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  // Launched as a programmatic dependent: the set-up above overlapped the
  // previous kernel's tail; nothing that kernel may write (q, lengths, appended
  // K/V rows, partials it may still read) is touched before it has completed.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");

  Iter it;
  if constexpr (FUSED) {
    // Every CTA counts the batch's tiles (the same number everywhere) and picks
    // the number of ranges so that no pair is cut into more segments than the
    // partial buffer holds: ranges of >= ceil(max tiles per pair / (cap - 1)) tiles.
    if (warp == 0) {
      long long sum = 0;
      for (int b = lane; b < p.B; b += 32) sum += seq_tiles(p, b);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
      if (lane == 0) *s_total = sum * p.Hkv;
    }
    __syncthreads();
    const long long total = *s_total;
    const int ntmax = (p.Lmax + T - 1) / T;
    const int qmin = (ntmax + p.nseg_cap - 2) / (p.nseg_cap - 1);
    long long g = total / qmin;
    if (g > (long long)gridDim.x) g = gridDim.x;
    if (g < 1) g = 1;
    it.init(p, total, total > 0 ? (int)g : 0);
  } else {
    __syncthreads();
    it.init(p);
  }

  if (warp == NCW + 1) {
    // ------------------------------ finisher ------------------------------
    // Single-launch form only. Takes each handed-off segment's partial from the
    // consumers, counts it in for its (row, kv head) and, when it completes the
    // count, merges that pair's segments and writes out / lse, while the
    // consumers go on with the next segment.
    if constexpr (FUSED) {
      // Rows with no keys have no segments: out = 0, lse = -inf.
      for (int b = blockIdx.x; b < p.B; b += gridDim.x) {
        if (seq_len(p, b) != 0) continue;
        const size_t row0 = (size_t)b * p.Hq;
        for (int i = lane; i < p.Hq * D / 4; i += 32) {
          const uint2 z = make_uint2(0u, 0u);
          reinterpret_cast<uint2*>(p.out + row0 * D)[i] = z;
#pragma unroll
          for (int pi = 0; pi < kMaxPeers; ++pi)
            if (pi < p.peers.npeers) reinterpret_cast<uint2*>(p.peers.peer_y[pi] + row0 * D)[i] = z;
        }
        for (int i = lane; i < p.Hq; i += 32) p.lse[row0 + i] = -INFINITY;
        if (p.seqlens_commit && lane == 0) p.seqlens_commit[b] = __ldg(p.seqlens + b);
      }
      const size_t plane = (size_t)p.B * p.Hq;
      int k = 0;
      Seg sg;
      while (it.next(p, sg)) {
        if (sg.nseg == 1 || sg.final_of_cta) continue;  // the consumers finish those
        const int slot = k % NF;
        if (!mbar_wait(&fin_full[slot], (k / NF) & 1, p.err, kDevErrFullWait)) return;
        int last = 0;
        if (lane == 0) {
          // Release the partial (the consumers' stores, ordered before this
          // thread by the hand-off barrier) at GPU scope, then count it in.
          __threadfence();
          int* ctr = p.counters + (size_t)sg.b * p.Hkv + sg.h;
          last = atomicAdd(ctr, 1) == sg.nseg - 1;
          if (last) *ctr = 0;  // every segment is in: reset for the next call
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();  // acquire: the pair's other partials are visible
          for (int hh = 0; hh < p.G; ++hh)
            combine_row<true>(p.o_part, p.lse_part, plane, (size_t)sg.b * p.Hq + (size_t)sg.h * p.G + hh,
                              sg.nseg, lane, p.out, p.lse, p.peers);
          if (sg.h == 0 && lane == 0 && p.seqlens_commit) p.seqlens_commit[sg.b] = __ldg(p.seqlens + sg.b);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&fin_empty[slot]);
        ++k;
      }
    }
    return;
  }

  if (warp == NCW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      const int withhold = blockIdx.x == 0 ? p.withhold_tile : -1;
      Seg sg;
      while (it.next(p, sg)) {
        const int L = seq_len(p, sg.b);
        const int t1 = min(sg.i1 * T, L);
        for (int t = sg.i0 * T; t < t1; t += T) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kDevErrEmptyWait)) return;
          if (issued++ == withhold) {  // test hook: this stage never fills
            if (++stage == STAGES) {
              stage = 0;
              phase ^= 1;
            }
            continue;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* kd = ring + stage * STAGE_BYTES;
          uint8_t* vd = kd + TILE_BYTES;
          // Contiguous cache: (token, row). Paged: (token within block, physical
          // block); a 64-token tile never crosses a block (block_size % 64 == 0).
          int ct = t, cb = sg.b;
          if (p.block_table) {
            cb = __ldg(p.block_table + (size_t)sg.b * p.max_blocks + t / p.block_size);
            ct = t % p.block_size;
          }
          tma_load_4d(kd, &tmK, &full[stage], 0, sg.h, ct, cb, pol);
          tma_load_4d(kd + HALF_BYTES, &tmK, &full[stage], 64, sg.h, ct, cb, pol);
          tma_load_4d(vd, &tmV, &full[stage], 0, sg.h, ct, cb, pol);
          tma_load_4d(vd + HALF_BYTES, &tmV, &full[stage], 64, sg.h, ct, cb, pol);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int g = lane >> 2;  // accumulator row group / B-fragment column
  const int c = lane & 3;
  const int j = lane >> 3;  // ldmatrix sub-matrix this lane addresses
  const int r = lane & 7;   // ldmatrix row this lane addresses
  const int tw = warp * 16; // this warp's first token inside a tile
  const float NEG_INF = -INFINITY;
  const int G = p.G;

  int kfin = 0;  // segments handed to the finisher so far
  int stage = 0;
  uint32_t phase = 0;
  Seg sg;
  while (it.next(p, sg)) {
    const int b = sg.b, h = sg.h;
    const int L = seq_len(p, b);
    const int t0 = sg.i0 * T;
    const int t1 = min(sg.i1 * T, L);

    // Q^T as the B operand: column n = query head g of the group (zero if g >= G).
    uint32_t qf[8][2];
    {
      const __nv_bfloat16* qrow = p.q + (size_t)b * p.q_stride + ((size_t)h * G + g) * D;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        if (g < G) {
          qf[ks][0] = __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 2 * c));
          qf[ks][1] = __ldg(reinterpret_cast<const uint32_t*>(qrow + 16 * ks + 8 + 2 * c));
        } else {
          qf[ks][0] = 0u;
          qf[ks][1] = 0u;
        }
      }
    }

    float o[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = NEG_INF, m1 = NEG_INF;  // running max (log2 domain) of heads 2c, 2c+1
    float l0 = 0.f, l1 = 0.f;          // this lane's share of the running sums

    for (int t = t0; t < t1; t += T) {
      // A time-out leaves the tile loop; all consumer warps then meet at the
      // merge barrier below and return together.
      if (!mbar_wait_group(&full[stage], phase, p.err, kDevErrFullWait, s_abort)) break;
      const uint32_t kb = smem_u32(ring + stage * STAGE_BYTES);
      const uint32_t vb = kb + TILE_BYTES;

      // S^T[16 tokens x 8 heads] = K[16 x 128] . Q^T[128 x 8]
      float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int tok = tw + (j & 1) * 8 + r;
        const int cc = 2 * (ks & 3) + (j >> 1);
        uint32_t a[4];
        ldsm_x4(swz128(kb + (ks >> 2) * HALF_BYTES, tok, cc), a[0], a[1], a[2], a[3]);
        mma_bf16_16816(sc, a, qf[ks][0], qf[ks][1]);
      }

      const int nv = t1 - (t + tw);  // valid tokens among this warp's 16
      const float x0 = (g < nv) ? sc[0] * p.scale_log2 : NEG_INF;
      const float x1 = (g < nv) ? sc[1] * p.scale_log2 : NEG_INF;
      const float x2 = (g + 8 < nv) ? sc[2] * p.scale_log2 : NEG_INF;
      const float x3 = (g + 8 < nv) ? sc[3] * p.scale_log2 : NEG_INF;
      float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float sf0 = (mn0 == NEG_INF) ? 0.f : mn0;  // all-masked guard
      const float sf1 = (mn1 == NEG_INF) ? 0.f : mn1;
      const float al0 = exp2f(m0 - sf0), al1 = exp2f(m1 - sf1);
      const float p0 = exp2f(x0 - sf0), p1 = exp2f(x1 - sf1);
      const float p2 = exp2f(x2 - sf0), p3 = exp2f(x3 - sf1);
      l0 = l0 * al0 + (p0 + p2);
      l1 = l1 * al1 + (p1 + p3);
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] *= al0;
        o[i][1] *= al1;
        o[i][2] *= al0;
        o[i][3] *= al1;
      }

      // P^T (accumulator layout: rows = tokens) -> B operand (rows = tokens as k).
      const uint32_t xx = pack_bf16x2(p0, p2);  // head 2c: tokens g, g+8
      const uint32_t yy = pack_bf16x2(p1, p3);  // head 2c+1
      const int srcA = (2 * c) * 4 + (g >> 1);
      const uint32_t xa = __shfl_sync(0xffffffffu, xx, srcA);
      const uint32_t ya = __shfl_sync(0xffffffffu, yy, srcA);
      const uint32_t xb = __shfl_sync(0xffffffffu, xx, srcA + 4);
      const uint32_t yb = __shfl_sync(0xffffffffu, yy, srcA + 4);
      const uint32_t va = (g & 1) ? ya : xa;  // P[2c][g], P[2c+8][g]
      const uint32_t vbv = (g & 1) ? yb : xb; // P[2c+1][g], P[2c+9][g]
      const uint32_t pb0 = __byte_perm(va, vbv, 0x5410);
      const uint32_t pb1 = __byte_perm(va, vbv, 0x7632);

      // Tokens past the end may hold anything (padding): zero their V rows so a
      // NaN in the padding cannot leak through 0 * NaN.
      const bool tail = nv < 16;
      const uint32_t mk_lo = keep_mask(2 * c < nv, 2 * c + 1 < nv);
      const uint32_t mk_hi = keep_mask(2 * c + 8 < nv, 2 * c + 9 < nv);

      // O^T[128 dims x 8 heads] += V^T[128 x 16 tokens] . P^T[16 x 8]
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int tok = tw + (j >> 1) * 8 + r;
        const int cc = 2 * (i & 3) + (j & 1);
        uint32_t a[4];
        ldsm_x4_t(swz128(vb + (i >> 2) * HALF_BYTES, tok, cc), a[0], a[1], a[2], a[3]);
        if (tail) {
          a[0] &= mk_lo;
          a[1] &= mk_lo;
          a[2] &= mk_hi;
          a[3] &= mk_hi;
        }
        mma_bf16_16816(o[i], a, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }

    // ---- merge the four warps' softmax states and write the segment's result ----
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, off);
      l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    if (g == 0) {
      cm[warp * 8 + 2 * c] = m0;
      cm[warp * 8 + 2 * c + 1] = m1;
      cl[warp * 8 + 2 * c] = l0;
      cl[warp * 8 + 2 * c + 1] = l1;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (2 * c < G) {
        float* dst = co + (warp * G + 2 * c) * D + 16 * i + g;
        dst[0] = o[i][0];
        dst[8] = o[i][2];
      }
      if (2 * c + 1 < G) {
        float* dst = co + (warp * G + 2 * c + 1) * D + 16 * i + g;
        dst[0] = o[i][1];
        dst[8] = o[i][3];
      }
    }
    named_bar_sync(1, NCW * 32);
    if (*s_abort) return;  // uniform: no consumer warp writes the flag past the barrier above
    // A pair with one segment needs no merge: in the single-launch form that
    // segment writes out / lse directly (the same values pass 2 gives: the
    // weight of a lone split is exactly 1).
    const bool direct = FUSED && sg.nseg == 1;
    {
      const int d = threadIdx.x;  // 0..127
      const size_t row0 = ((size_t)sg.slot * p.B + b) * p.Hq + (size_t)h * G;
      const size_t orow0 = (size_t)b * p.Hq + (size_t)h * G;
      for (int hh = 0; hh < G; ++hh) {
        float M = NEG_INF;
#pragma unroll
        for (int ww = 0; ww < NCW; ++ww) M = fmaxf(M, cm[ww * 8 + hh]);
        float Lsum = 0.f, acc = 0.f;
        if (M != NEG_INF) {
#pragma unroll
          for (int ww = 0; ww < NCW; ++ww) {
            const float sw = exp2f(cm[ww * 8 + hh] - M);
            Lsum += sw * cl[ww * 8 + hh];
            acc += sw * co[(ww * G + hh) * D + d];
          }
        }
        const bool ok = Lsum > 0.f;
        const float ov = ok ? acc / Lsum : 0.f;
        const float lv = ok ? (M + log2f(Lsum)) * 0.69314718055994531f : NEG_INF;
        if (direct) {
          const __nv_bfloat16 bv = __float2bfloat16_rn(ov);
          p.out[(orow0 + hh) * D + d] = bv;
#pragma unroll
          for (int pi = 0; pi < kMaxPeers; ++pi)
            if (pi < p.peers.npeers) p.peers.peer_y[pi][(orow0 + hh) * D + d] = bv;
          if (d == 0) p.lse[orow0 + hh] = lv;
        } else {
          p.o_part[(row0 + hh) * D + d] = ov;
          if (d == 0) p.lse_part[row0 + hh] = lv;
        }
      }
    }
    if constexpr (FUSED) {
      if (direct) {
        if (h == 0 && threadIdx.x == 0 && p.seqlens_commit) p.seqlens_commit[b] = __ldg(p.seqlens + b);
      } else if (sg.final_of_cta) {
        // The CTA's last segment: nothing follows it, so the consumers finish
        // it themselves, one q head per warp.
        named_bar_sync(1, NCW * 32);  // every partial store of this segment is issued
        if (threadIdx.x == 0) {
          __threadfence();  // release them at GPU scope, then count the segment in
          int* ctr = p.counters + (size_t)b * p.Hkv + h;
          const int last = atomicAdd(ctr, 1) == sg.nseg - 1;
          if (last) *ctr = 0;
          *s_last = last;
        }
        named_bar_sync(1, NCW * 32);
        if (*s_last) {
          __threadfence();  // acquire: the pair's other partials are visible
          for (int hh = warp; hh < G; hh += NCW)
            combine_row<true>(p.o_part, p.lse_part, (size_t)p.B * p.Hq, (size_t)b * p.Hq + (size_t)h * G + hh,
                              sg.nseg, lane, p.out, p.lse, p.peers);
          if (h == 0 && threadIdx.x == 0 && p.seqlens_commit) p.seqlens_commit[b] = __ldg(p.seqlens + b);
        }
      } else {
        // Hand the partial to the finisher warp; a consumer waits only when
        // the ring of NF slots is full.
        const int slot = kfin % NF;
        if (kfin < NF || mbar_wait_group(&fin_empty[slot], ((kfin / NF) & 1) ^ 1, p.err, kDevErrEmptyWait,
                                         s_abort)) {
          __syncwarp();
          if (lane == 0) mbar_arrive(&fin_full[slot]);
        }
        ++kfin;
      }
    }
    named_bar_sync(1, NCW * 32);
    if (*s_abort) return;  // a hand-off wait ran out: all consumer warps leave together
  }
}

// One warp per (b, q head); lane owns dims [4*lane, 4*lane+4).
__global__ void __launch_bounds__(128) combine_kernel(const float* __restrict__ o_part,
                                                      const float* __restrict__ lse_part,
                                                      const int* __restrict__ seqlens,
                                                      __nv_bfloat16* __restrict__ out,
                                                      float* __restrict__ lse, int B, int Hq,
                                                      int Lmax, int chunk, int* seqlens_commit,
                                                      OutPlace peers) {
  // The next kernel may launch now (it waits for this grid before reading).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // Launched as a programmatic dependent of pass 1: wait for its partials.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= B * Hq) return;
  const int b = row / Hq;
  const int Lraw = __ldg(seqlens + b);
  // Optional: publish the lengths this step used to another buffer (the
  // caller's length array when a projection epilogue advanced them out of place).
  if (seqlens_commit && row == b * Hq && lane == 0) seqlens_commit[b] = Lraw;
  int L = min(max(Lraw, 0), Lmax);
  const int n = (L + chunk - 1) / chunk;
  combine_row<false>(o_part, lse_part, (size_t)B * Hq, (size_t)row, n, lane, out, lse, peers);
}

static int chunk_tokens(int Lmax, int num_splits) {
  int c = (Lmax + num_splits - 1) / num_splits;
  return ((c + T - 1) / T) * T;
}

template <int STAGES>
static size_t fwd_smem_bytes(int G) {
  return 1024 + (size_t)STAGES * STAGE_BYTES + (size_t)(2 * NCW * 8 + NCW * G * D) * 4 +
         2 * STAGES * 8 + 2 * NF * 8 + 16;
}

template <int STAGES, bool FUSED>
static int launch_fwd(const CUtensorMap& tmK, const CUtensorMap& tmV, const Params& p,
                      cudaStream_t stream) {
  auto kern = splitkv_kernel<STAGES, FUSED>;
  const size_t smem = fwd_smem_bytes<STAGES>(p.G);
  FK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int occ = 0;
  FK_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NTHREADS, smem));
  if (occ < 1) occ = 1;
  long long grid = (long long)num_sms() * occ;
  if (!FUSED) {
    // Upper bound on the number of units: every row at full length.
    const long long max_units = (long long)p.B * p.Hkv * ((p.Lmax + p.chunk - 1) / p.chunk);
    if (grid > max_units) grid = max_units;
  } else {
    const long long max_tiles = (long long)p.B * p.Hkv * ((p.Lmax + T - 1) / T);
    if (grid > max_tiles) grid = max_tiles;
  }
  if (grid < 1) grid = 1;
  // Programmatic dependent launch: barrier set-up and descriptor prefetch
  // overlap the previous kernel's tail (the kernel waits for it before
  // touching memory that kernel may write).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(NTHREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tmK, tmV, p));
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace attn
}  // namespace fk

using namespace fk;

static int check_attn_args(const void* q, const void* k, const void* v, const int32_t* seqlens,
                           int B, int Lmax, int Hq, int Hkv, int head_dim, int num_splits) {
  FK_CHECK_ARG(q && k && v && seqlens, "null tensor pointer");
  FK_CHECK_ARG(B >= 1, "batch must be >= 1");
  FK_CHECK_ARG(Lmax >= 1, "max_seqlen must be >= 1");
  FK_CHECK_ARG(head_dim == attn::D, "head_dim must be 128");
  FK_CHECK_ARG(Hkv >= 1 && Hq >= Hkv && Hq % Hkv == 0,
               "num_heads_q must be a positive multiple of num_heads_kv");
  FK_CHECK_ARG(Hq / Hkv <= 8, "GQA group size (num_heads_q / num_heads_kv) must be <= 8");
  FK_CHECK_ARG(num_splits >= 1, "num_splits must be >= 1");
  FK_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0,
               "q / k_cache / v_cache must be 16-byte aligned");
  return kOk;
}

extern "C" {

int fk_dec_attn_chunk_tokens(int max_seqlen, int num_splits) {
  if (max_seqlen < 1 || num_splits < 1) return 0;
  return attn::chunk_tokens(max_seqlen, num_splits);
}

// Test hook (fk_debug_attn_withhold_tile): tile index CTA 0's producer skips, -1 never.
static int g_withhold_tile = -1;

// What the single-launch form writes besides the partials (counters null: pass 1 only).
struct FusedOut {
  int* counters = nullptr;
  void* out = nullptr;
  float* lse = nullptr;
  int32_t* seqlens_commit = nullptr;
  OutPlace peers = {};
};

// Paged form when block_table != null: k_cache/v_cache are block pools
// [num_blocks, block_size, Hkv, D] and max_seqlen = max_blocks * block_size.
static int splitkv_fwd_impl(const void* q, long long q_stride, const void* k_cache, const void* v_cache,
                            const int32_t* cache_seqlens, float* o_partial, float* lse_partial,
                            int batch, int max_seqlen, int num_heads_q, int num_heads_kv,
                            int head_dim, int num_splits, float softmax_scale, void* stream,
                            const int32_t* block_table = nullptr, int block_size = 0, int num_blocks = 0,
                            const FusedOut& fo = FusedOut{}) {
  FK_CHECK_ARG(q_stride >= (long long)num_heads_q * head_dim && q_stride % 8 == 0,
               "q row stride must be >= num_heads_q * head_dim and a multiple of 8");
  int rc = check_attn_args(q, k_cache, v_cache, cache_seqlens, batch, max_seqlen, num_heads_q,
                           num_heads_kv, head_dim, num_splits);
  if (rc) return rc;
  FK_CHECK_ARG(o_partial && lse_partial, "null partial buffer");
  FK_CHECK_ARG(((uintptr_t)o_partial & 15) == 0, "o_partial must be 16-byte aligned");
  int* err = device_error_word();
  if (!err) return fail(kErrCuda, "device error word unavailable");

  attn::Params p;
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.q_stride = q_stride;
  p.block_table = block_table;
  p.block_size = block_table ? block_size : 0;
  p.max_blocks = block_table ? max_seqlen / block_size : 0;
  p.seqlens = cache_seqlens;
  p.o_part = o_partial;
  p.lse_part = lse_partial;
  p.err = err;
  p.B = batch;
  p.Lmax = max_seqlen;
  p.Hq = num_heads_q;
  p.Hkv = num_heads_kv;
  p.G = num_heads_q / num_heads_kv;
  p.chunk = attn::chunk_tokens(max_seqlen, num_splits);
  p.scale_log2 = softmax_scale * 1.4426950408889634f;
  p.counters = fo.counters;
  p.out = static_cast<__nv_bfloat16*>(fo.out);
  p.lse = fo.lse;
  p.seqlens_commit = fo.seqlens_commit;
  p.peers = fo.peers;
  p.withhold_tile = g_withhold_tile;
  p.nseg_cap = num_splits;
  if (fo.counters) {
    FK_CHECK_ARG(num_splits >= 2, "single-launch attention needs room for >= 2 partial slots per pair");
    FK_CHECK_ARG(fo.out && fo.lse, "null out / lse");
    FK_CHECK_ARG(((uintptr_t)fo.out & 7) == 0, "out must be 8-byte aligned");
    FK_CHECK_ARG(((uintptr_t)fo.counters & 3) == 0, "counters must be 4-byte aligned");
    FK_CHECK_ARG(fo.seqlens_commit != (int32_t*)cache_seqlens, "seqlens_commit must not alias cache_seqlens");
  }

  // K/V cache [B, Lmax, Hkv, 128] bf16 viewed as a 4-D tensor (dim, head, token, batch).
  CUtensorMap tmK, tmV;
  const uint64_t rows = block_table ? (uint64_t)block_size : (uint64_t)max_seqlen;
  const uint64_t outer = block_table ? (uint64_t)num_blocks : (uint64_t)batch;
  const uint64_t dims[4] = {(uint64_t)attn::D, (uint64_t)num_heads_kv, rows, outer};
  const uint64_t strides[3] = {(uint64_t)attn::D * 2, (uint64_t)num_heads_kv * attn::D * 2,
                               rows * num_heads_kv * attn::D * 2};
  const uint32_t box[4] = {64, 1, (uint32_t)attn::T, 1};
  rc = encode_tma(&tmK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(k_cache), dims,
                  strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  rc = encode_tma(&tmV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(v_cache), dims,
                  strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (fo.counters) {
    if (p.G <= 4) return attn::launch_fwd<3, true>(tmK, tmV, p, st);
    return attn::launch_fwd<2, true>(tmK, tmV, p, st);
  }
  if (p.G <= 4) return attn::launch_fwd<3, false>(tmK, tmV, p, st);
  return attn::launch_fwd<2, false>(tmK, tmV, p, st);
}

int fk_dec_attn_splitkv_fwd(const void* q, const void* k_cache, const void* v_cache,
                            const int32_t* cache_seqlens, float* o_partial, float* lse_partial,
                            int batch, int max_seqlen, int num_heads_q, int num_heads_kv,
                            int head_dim, int num_splits, float softmax_scale, void* stream) {
  return splitkv_fwd_impl(q, (long long)num_heads_q * head_dim, k_cache, v_cache, cache_seqlens, o_partial,
                          lse_partial, batch, max_seqlen, num_heads_q, num_heads_kv, head_dim, num_splits,
                          softmax_scale, stream);
}

int fk_dec_attn_fwd_ex(const void* q, long long q_batch_stride, const void* k_cache, const void* v_cache,
                       const int32_t* cache_seqlens, void* out, float* lse, float* o_partial,
                       float* lse_partial, int batch, int max_seqlen, int num_heads_q, int num_heads_kv,
                       int head_dim, int num_splits, float softmax_scale, void* stream) {
  int rc = splitkv_fwd_impl(q, q_batch_stride, k_cache, v_cache, cache_seqlens, o_partial, lse_partial, batch,
                            max_seqlen, num_heads_q, num_heads_kv, head_dim, num_splits, softmax_scale, stream);
  if (rc) return rc;
  return fk_dec_attn_combine(o_partial, lse_partial, cache_seqlens, out, lse, batch, max_seqlen, num_heads_q,
                             head_dim, num_splits, stream);
}

int fk_dec_attn_fwd_paged(const void* q, const void* k_pool, const void* v_pool, const int32_t* block_table,
                          const int32_t* cache_seqlens, void* out, float* lse, float* o_partial,
                          float* lse_partial, int batch, int max_blocks_per_seq, int block_size, int num_blocks,
                          int num_heads_q, int num_heads_kv, int head_dim, int num_splits, float softmax_scale,
                          void* stream) {
  FK_CHECK_ARG(block_table != nullptr, "block_table is null");
  FK_CHECK_ARG(block_size >= 64 && block_size % 64 == 0, "block_size must be a positive multiple of 64");
  FK_CHECK_ARG(max_blocks_per_seq >= 1 && num_blocks >= 1, "max_blocks_per_seq and num_blocks must be >= 1");
  const long long Lmax = (long long)max_blocks_per_seq * block_size;
  FK_CHECK_ARG(Lmax < (1LL << 31), "max_blocks_per_seq * block_size too large");
  int rc = splitkv_fwd_impl(q, (long long)num_heads_q * head_dim, k_pool, v_pool, cache_seqlens, o_partial,
                            lse_partial, batch, (int)Lmax, num_heads_q, num_heads_kv, head_dim, num_splits,
                            softmax_scale, stream, block_table, block_size, num_blocks);
  if (rc) return rc;
  return fk_dec_attn_combine(o_partial, lse_partial, cache_seqlens, out, lse, batch, (int)Lmax, num_heads_q,
                             head_dim, num_splits, stream);
}

static int combine_impl(const float* o_partial, const float* lse_partial, const int32_t* cache_seqlens,
                        int32_t* seqlens_commit, void* out, float* lse, int batch, int max_seqlen,
                        int num_heads_q, int head_dim, int num_splits, void* stream,
                        const OutPlace& peers = OutPlace{}) {
  FK_CHECK_ARG(o_partial && lse_partial && cache_seqlens && out && lse, "null tensor pointer");
  FK_CHECK_ARG(seqlens_commit != (int32_t*)cache_seqlens, "seqlens_commit must not alias cache_seqlens");
  FK_CHECK_ARG(batch >= 1 && max_seqlen >= 1 && num_heads_q >= 1 && num_splits >= 1,
               "sizes must be positive");
  FK_CHECK_ARG(head_dim == attn::D, "head_dim must be 128");
  FK_CHECK_ARG(((uintptr_t)o_partial & 15) == 0 && ((uintptr_t)out & 7) == 0,
               "o_partial must be 16-byte and out 8-byte aligned");
  const int rows = batch * num_heads_q;
  const int chunk = attn::chunk_tokens(max_seqlen, num_splits);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((rows + 3) / 4), 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, attn::combine_kernel, o_partial, lse_partial, cache_seqlens,
                                   static_cast<__nv_bfloat16*>(out), lse, batch, num_heads_q, max_seqlen,
                                   chunk, seqlens_commit, peers));
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}

int fk_dec_attn_combine(const float* o_partial, const float* lse_partial,
                        const int32_t* cache_seqlens, void* out, float* lse, int batch,
                        int max_seqlen, int num_heads_q, int head_dim, int num_splits,
                        void* stream) {
  return combine_impl(o_partial, lse_partial, cache_seqlens, nullptr, out, lse, batch, max_seqlen, num_heads_q,
                      head_dim, num_splits, stream);
}

int fk_dec_attn_fwd_peers(const void* q, long long q_batch_stride, const void* k_cache, const void* v_cache,
                          const int32_t* cache_seqlens, void* out, void* const* peer_out, int npeers, float* lse,
                          float* o_partial, float* lse_partial, int batch, int max_seqlen, int num_heads_q,
                          int num_heads_kv, int head_dim, int num_splits, float softmax_scale, void* stream) {
  FK_CHECK_ARG(npeers >= 0 && npeers <= kMaxPeers, "npeers must be in [0, 7]");
  OutPlace peers = {};
  peers.npeers = npeers;
  for (int i = 0; i < npeers; ++i) {
    FK_CHECK_ARG(peer_out && peer_out[i] && ((uintptr_t)peer_out[i] & 7) == 0, "peer output must be 8-byte aligned");
    peers.peer_y[i] = static_cast<__nv_bfloat16*>(peer_out[i]);
  }
  int rc = splitkv_fwd_impl(q, q_batch_stride, k_cache, v_cache, cache_seqlens, o_partial, lse_partial, batch,
                            max_seqlen, num_heads_q, num_heads_kv, head_dim, num_splits, softmax_scale, stream);
  if (rc) return rc;
  return combine_impl(o_partial, lse_partial, cache_seqlens, nullptr, out, lse, batch, max_seqlen, num_heads_q,
                      head_dim, num_splits, stream, peers);
}

int fk_dec_attn_fwd_commit(const void* q, long long q_batch_stride, const void* k_cache, const void* v_cache,
                           const int32_t* block_table, const int32_t* cache_seqlens, int32_t* seqlens_commit,
                           void* out, float* lse, float* o_partial, float* lse_partial, int batch, int max_seqlen,
                           int block_size, int num_blocks, int num_heads_q, int num_heads_kv, int head_dim,
                           int num_splits, float softmax_scale, void* stream) {
  if (block_table) {
    FK_CHECK_ARG(block_size >= 64 && block_size % 64 == 0, "block_size must be a positive multiple of 64");
    FK_CHECK_ARG(max_seqlen % block_size == 0 && num_blocks >= 1,
                 "paged cache: max_seqlen must be max_blocks_per_seq * block_size, num_blocks >= 1");
  }
  int rc = splitkv_fwd_impl(q, q_batch_stride, k_cache, v_cache, cache_seqlens, o_partial, lse_partial, batch,
                            max_seqlen, num_heads_q, num_heads_kv, head_dim, num_splits, softmax_scale, stream,
                            block_table, block_size, num_blocks);
  if (rc) return rc;
  return combine_impl(o_partial, lse_partial, cache_seqlens, seqlens_commit, out, lse, batch, max_seqlen,
                      num_heads_q, head_dim, num_splits, stream);
}

int fk_dec_attn_fwd_fused(const void* q, long long q_batch_stride, const void* k_cache, const void* v_cache,
                          const int32_t* block_table, const int32_t* cache_seqlens, int32_t* seqlens_commit,
                          void* out, void* const* peer_out, int npeers, float* lse, float* o_partial,
                          float* lse_partial, int32_t* counters, int batch, int max_seqlen, int block_size,
                          int num_blocks, int num_heads_q, int num_heads_kv, int head_dim, int num_splits,
                          float softmax_scale, void* stream) {
  FK_CHECK_ARG(counters != nullptr, "counters is null");
  FK_CHECK_ARG(npeers >= 0 && npeers <= kMaxPeers, "npeers must be in [0, 7]");
  if (block_table) {
    FK_CHECK_ARG(block_size >= 64 && block_size % 64 == 0, "block_size must be a positive multiple of 64");
    FK_CHECK_ARG(max_seqlen % block_size == 0 && num_blocks >= 1,
                 "paged cache: max_seqlen must be max_blocks_per_seq * block_size, num_blocks >= 1");
  }
  FusedOut fo;
  fo.counters = counters;
  fo.out = out;
  fo.lse = lse;
  fo.seqlens_commit = seqlens_commit;
  fo.peers.npeers = npeers;
  for (int i = 0; i < npeers; ++i) {
    FK_CHECK_ARG(peer_out && peer_out[i] && ((uintptr_t)peer_out[i] & 7) == 0, "peer output must be 8-byte aligned");
    fo.peers.peer_y[i] = static_cast<__nv_bfloat16*>(peer_out[i]);
  }
  return splitkv_fwd_impl(q, q_batch_stride, k_cache, v_cache, cache_seqlens, o_partial, lse_partial, batch,
                          max_seqlen, num_heads_q, num_heads_kv, head_dim, num_splits, softmax_scale, stream,
                          block_table, block_size, num_blocks, fo);
}

int fk_debug_attn_withhold_tile(int tile) {
  g_withhold_tile = tile < 0 ? -1 : tile;
  return kOk;
}

int fk_dec_attn_fwd(const void* q, const void* k_cache, const void* v_cache,
                    const int32_t* cache_seqlens, void* out, float* lse, float* o_partial,
                    float* lse_partial, int batch, int max_seqlen, int num_heads_q,
                    int num_heads_kv, int head_dim, int num_splits, float softmax_scale,
                    void* stream) {
  int rc = fk_dec_attn_splitkv_fwd(q, k_cache, v_cache, cache_seqlens, o_partial, lse_partial,
                                   batch, max_seqlen, num_heads_q, num_heads_kv, head_dim,
                                   num_splits, softmax_scale, stream);
  if (rc) return rc;
  return fk_dec_attn_combine(o_partial, lse_partial, cache_seqlens, out, lse, batch, max_seqlen,
                             num_heads_q, head_dim, num_splits, stream);
}

}  // extern "C"
