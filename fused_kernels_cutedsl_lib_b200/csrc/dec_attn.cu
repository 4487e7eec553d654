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

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace attn {

constexpr int D = 128;                     // head_dim
constexpr int T = 64;                      // tokens per KV tile
constexpr int NCW = 4;                     // consumer warps (16 tokens each)
constexpr int NTHREADS = (NCW + 1) * 32;   // + one TMA producer warp
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

__device__ __forceinline__ uint32_t keep_mask(bool lo, bool hi) {
  return (lo ? 0x0000FFFFu : 0u) | (hi ? 0xFFFF0000u : 0u);
}

template <int STAGES>
__global__ void __launch_bounds__(NTHREADS, 1)
    splitkv_fwd_kernel(const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  float* cm = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES);  // [NCW][8] row max
  float* cl = cm + NCW * 8;                                           // [NCW][8] row sum
  float* co = cl + NCW * 8;                                           // [NCW][G][D]
  uint64_t* full = reinterpret_cast<uint64_t*>(co + NCW * p.G * D);
  uint64_t* empty = full + STAGES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    fence_barrier_init();
  }
  __syncthreads();

  Walker w;
  w.init(p);
  // Pass 2 may be scheduled now; it waits for this grid's completion itself.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == NCW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const uint64_t pol = l2_policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      for (long long u = blockIdx.x;; u += gridDim.x) {
        int b, h, s;
        if (!w.locate(p, u, b, h, s)) break;
        const int L = seq_len(p, b);
        const int t0 = s * p.chunk;
        const int t1 = min(t0 + p.chunk, L);
        for (int t = t0; t < t1; t += T) {
          if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kDevErrEmptyWait)) return;
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* kd = ring + stage * STAGE_BYTES;
          uint8_t* vd = kd + TILE_BYTES;
          // Contiguous cache: (token, row). Paged: (token within block, physical
          // block); a 64-token tile never crosses a block (block_size % 64 == 0).
          int ct = t, cb = b;
          if (p.block_table) {
            cb = __ldg(p.block_table + (size_t)b * p.max_blocks + t / p.block_size);
            ct = t % p.block_size;
          }
          tma_load_4d(kd, &tmK, &full[stage], 0, h, ct, cb, pol);
          tma_load_4d(kd + HALF_BYTES, &tmK, &full[stage], 64, h, ct, cb, pol);
          tma_load_4d(vd, &tmV, &full[stage], 0, h, ct, cb, pol);
          tma_load_4d(vd + HALF_BYTES, &tmV, &full[stage], 64, h, ct, cb, pol);
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

  int stage = 0;
  uint32_t phase = 0;
  for (long long u = blockIdx.x;; u += gridDim.x) {
    int b, h, s;
    if (!w.locate(p, u, b, h, s)) break;
    const int L = seq_len(p, b);
    const int t0 = s * p.chunk;
    const int t1 = min(t0 + p.chunk, L);

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
      if (!mbar_wait(&full[stage], phase, p.err, kDevErrFullWait)) return;
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

    // ---- merge the four warps' softmax states and write the unit's partial ----
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
    {
      const int d = threadIdx.x;  // 0..127
      const size_t row0 = ((size_t)s * p.B + b) * p.Hq + (size_t)h * G;
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
        p.o_part[(row0 + hh) * D + d] = ok ? acc / Lsum : 0.f;
        if (d == 0) p.lse_part[row0 + hh] = ok ? (M + log2f(Lsum)) * 0.69314718055994531f : NEG_INF;
      }
    }
    named_bar_sync(1, NCW * 32);
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
  const size_t plane = (size_t)B * Hq;
  float M = -INFINITY;
  for (int s = lane; s < n; s += 32) M = fmaxf(M, __ldg(lse_part + s * plane + row));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float W = 0.f;
  if (M != -INFINITY) {
    // Four splits' loads in flight per iteration (the loop is latency-bound
    // otherwise); the sum still runs in split order.
    int s = 0;
    for (; s + 4 <= n; s += 4) {
      float ls[4];
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        ls[u] = __ldg(lse_part + (s + u) * plane + row);
        v[u] = __ldg(reinterpret_cast<const float4*>(o_part + ((s + u) * plane + row) * D) + lane);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float wgt = expf(ls[u] - M);
        W += wgt;
        acc.x += wgt * v[u].x;
        acc.y += wgt * v[u].y;
        acc.z += wgt * v[u].z;
        acc.w += wgt * v[u].w;
      }
    }
    for (; s < n; ++s) {
      const float ls = __ldg(lse_part + s * plane + row);
      const float wgt = expf(ls - M);
      const float4 v = __ldg(reinterpret_cast<const float4*>(o_part + (s * plane + row) * D) + lane);
      W += wgt;
      acc.x += wgt * v.x;
      acc.y += wgt * v.y;
      acc.z += wgt * v.z;
      acc.w += wgt * v.w;
    }
  }
  const bool ok = W > 0.f;
  const float inv = ok ? 1.f / W : 0.f;
  uint2 packed;
  packed.x = pack_bf16x2(acc.x * inv, acc.y * inv);
  packed.y = pack_bf16x2(acc.z * inv, acc.w * inv);
  reinterpret_cast<uint2*>(out + (size_t)row * D)[lane] = packed;
#pragma unroll
  for (int i = 0; i < kMaxPeers; ++i)  // the same rows in other GPUs' buffers (all-gather of a batch shard)
    if (i < peers.npeers) reinterpret_cast<uint2*>(peers.peer_y[i] + (size_t)row * D)[lane] = packed;
  if (lane == 0) lse[row] = ok ? M + logf(W) : -INFINITY;
}

static int chunk_tokens(int Lmax, int num_splits) {
  int c = (Lmax + num_splits - 1) / num_splits;
  return ((c + T - 1) / T) * T;
}

template <int STAGES>
static size_t fwd_smem_bytes(int G) {
  return 1024 + (size_t)STAGES * STAGE_BYTES + (size_t)(2 * NCW * 8 + NCW * G * D) * 4 +
         2 * STAGES * 8;
}

template <int STAGES>
static int launch_fwd(const CUtensorMap& tmK, const CUtensorMap& tmV, const Params& p,
                      cudaStream_t stream) {
  auto kern = splitkv_fwd_kernel<STAGES>;
  const size_t smem = fwd_smem_bytes<STAGES>(p.G);
  FK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int occ = 0;
  FK_CHECK_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, NTHREADS, smem));
  if (occ < 1) occ = 1;
  // Upper bound on the number of units: every row at full length.
  const long long max_units =
      (long long)p.B * p.Hkv * ((p.Lmax + p.chunk - 1) / p.chunk);
  long long grid = (long long)num_sms() * occ;
  if (grid > max_units) grid = max_units;
  if (grid < 1) grid = 1;
  kern<<<(unsigned)grid, NTHREADS, smem, stream>>>(tmK, tmV, p);
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

// Paged form when block_table != null: k_cache/v_cache are block pools
// [num_blocks, block_size, Hkv, D] and max_seqlen = max_blocks * block_size.
static int splitkv_fwd_impl(const void* q, long long q_stride, const void* k_cache, const void* v_cache,
                            const int32_t* cache_seqlens, float* o_partial, float* lse_partial,
                            int batch, int max_seqlen, int num_heads_q, int num_heads_kv,
                            int head_dim, int num_splits, float softmax_scale, void* stream,
                            const int32_t* block_table = nullptr, int block_size = 0, int num_blocks = 0) {
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
  if (p.G <= 4) return attn::launch_fwd<3>(tmK, tmV, p, st);
  return attn::launch_fwd<2>(tmK, tmV, p, st);
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
