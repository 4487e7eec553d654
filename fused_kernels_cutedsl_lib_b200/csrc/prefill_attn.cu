// Prefill (full-sequence) attention on sm_100a tensor cores:
//   O[b, h] = softmax(Q[b, h] K[b, hk]^T * scale) V[b, hk],  hk = h / (H / Hkv)
// for Q [B, H, Lq, D], K/V [B, Hkv, Lkv, D], O [B, H, Lq, D] bf16 (D = 64 or
// 128), non-causal, with an optional natural-log LSE [B, H, Lq] fp32.
//
// Replaces the reference's FlashSM90 (python/cutedsl_kernels/attn/
// attempt6_epi_pipeline/attn.py:73-241: wgmma S = Q K^T, exp2-domain online
// softmax in registers (my_softmax.py:35-105), O += P V, checked against
// F.scaled_dot_product_attention in tests.py:85 and attn_reimpl attn.py:778-784).
//
// One CTA per (256 queries = two 128-row tiles A and B, b*h), 320 threads:
//   warps 0-3   softmax of tile A, warps 4-7 softmax of tile B: thread = query
//               row = TMEM lane (warp w reads lanes 32*(w%4)..). Two softmax
//               warps per SM sub-partition hide each other's latency.
//               tcgen05.ld S_t(j), mask keys past Lkv, exp2-domain running max;
//               the O rescale (tcgen05.ld/st of the row) runs only when a
//               warp's max grows by more than 2^8, otherwise P keeps the stale
//               max, which the final 1/l normalisation cancels exactly. P_t(j)
//               is rounded to bf16 pairs and written over S_t(j) in TMEM
//               (tcgen05.st), where the P V MMA reads it as its A operand.
//               Epilogue: O / l to bf16, LSE = (m + log2 l) ln 2.
//   warp 8      TMA producer: both Q tiles once, then K_0, V_0, K_1, V_1, ...
//               (128 keys each) through one ring shared by the two tiles
//               (3-D tensor maps: keys past Lkv read as zero)
//   warp 9      allocates TMEM (S_A | S_B | O_A | O_B); one lane issues
//               tcgen05.mma: per j and tile, O_t += P_t(j) V_j (A = P from
//               TMEM, B = V MN-major straight from the TMA tile), then
//               S_t(j+1) = Q_t K_{j+1}^T into the same columns. The tensor pipe
//               runs in issue order, so S_t(j+1) overwrites P_t(j) only after
//               it was read, and the completion of S_t(j+1) also means
//               P_t(j) V_j is in O_t: the softmax never waits for it.
// Every mbarrier wait is bounded (device error word + orderly exit).
#include <math.h>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace fa {

constexpr int BM = 128;  // queries per tile (UMMA M, TMEM lanes)
constexpr int NT = 2;    // query tiles per CTA
constexpr int BN = 128;  // keys per tile
constexpr int NTHREADS = 320;
constexpr int TMA_WARP = 8, MMA_WARP = 9;
constexpr int ATOM = 128 * 128;  // one 128-row x 64-element bf16 swizzle block: 16 KB
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr size_t kSmemLimit = 227 * 1024;

template <int D>
struct Cfg {
  static constexpr int TILE = D * 256;  // 128 rows x D x 2 B
  static constexpr int NS = D == 64 ? 10 : 5;  // K/V ring stages (P lives in TMEM)
  static constexpr int Q_OFF = 0;
  static constexpr int KV_OFF = Q_OFF + NT * TILE;
  static constexpr int BAR_OFF = KV_OFF + NS * TILE;
  static constexpr int NBAR = 1 + 2 * NS + 3 * NT + 1;
  static constexpr size_t SMEM = 1024 + BAR_OFF + NBAR * 8 + 16;
  static_assert(SMEM <= kSmemLimit, "shared memory budget");
  static constexpr int O_COL = NT * BN;  // O_t at column O_COL + t * D
};

struct Params {
  __nv_bfloat16* o;
  float* lse;
  int* err;
  int H, G, Lq, Lkv, nkv;
  float scale_log2;
};

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128B swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// MN-major operand, 128B swizzle: 64-element MN chunks `lbo` bytes apart,
// 8-row K groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_mn_sw128(uint32_t saddr, uint32_t lbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) | (64ull << 32) |
         (1ull << 46) | (2ull << 61);
}
// kind::f16, A = B = bf16, D = f32, M = 128, N = n; b_mn selects an MN-major B.
__host__ __device__ constexpr uint32_t idesc_bf16(int n, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn ? (1u << 16) : 0u) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
// D += A . B with A (M = 128 x K = 16, bf16 pairs packed per 32-bit column) in TMEM.
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
      "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]),
      "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 consecutive TMEM columns of this thread's lane (no wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x on the special-function unit (PTX ex2.approx; flushes subnormal results).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int D>
__global__ void __launch_bounds__(NTHREADS, 1)
    fmha_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, Params p) {
  using C = Cfg<D>;
  constexpr int NS = C::NS;
  constexpr int NA = D / 64;  // 64-element swizzle atoms along D
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;    // [NS]
  uint64_t* kv_empty = kv_full + NS; // [NS]
  uint64_t* s_full = kv_empty + NS;  // [NT]
  uint64_t* p_full = s_full + NT;    // [NT]: P_t(j) written over S_t(j) in TMEM
  uint64_t* p_empty = p_full + NT;   // [NT]: also "O_t holds P_t(j) V_j"
  uint64_t* done = p_empty + NT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, bh = blockIdx.y;
  const int kv_bh = (bh / p.H) * (p.H / p.G) + (bh % p.H) / p.G;
  const int n = p.nkv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int t = 0; t < NT; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&p_empty[t], 1);
    }
    mbar_init(done, 8);
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == TMA_WARP) {
    // ------------------------------ TMA producer ------------------------------
    // Ring items: K_j = item 2j, V_j = item 2j + 1, stage = item % NS.
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const uint64_t pol_q = l2_policy_evict_first();
      const uint64_t pol_kv = l2_policy_evict_last();  // re-read by every query tile of the head
      mbar_arrive_expect_tx(q_full, NT * C::TILE);
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int a = 0; a < NA; ++a)
          tma_load_3d(smem + C::Q_OFF + t * C::TILE + a * ATOM, &tmQ, q_full, a * 64, (qt * NT + t) * BM, bh, pol_q);
      for (int it = 0; it < 2 * n; ++it) {
        const int st = it % NS;
        if (!mbar_wait(&kv_empty[st], ((it / NS) & 1) ^ 1, p.err, kDevErrEmptyWait)) break;
        mbar_arrive_expect_tx(&kv_full[st], C::TILE);
        const CUtensorMap* map = (it & 1) ? &tmV : &tmK;
#pragma unroll
        for (int a = 0; a < NA; ++a)
          tma_load_3d(smem + C::KV_OFF + st * C::TILE + a * ATOM, map, &kv_full[st], a * 64, (it >> 1) * BN, kv_bh,
                      pol_kv);
      }
    }
    __syncwarp();
    return;
  }

  if (warp == MMA_WARP) {
    // ------------------------------ MMA issuer ------------------------------
    bool ok = true;
    if (lane == 0) {
      constexpr uint32_t IDS = idesc_bf16(BN, false);
      constexpr uint32_t IDO = idesc_bf16(D, true);
      // S_t(j) = Q_t K_j^T into TMEM columns [t*BN, t*BN + BN).
      auto issue_s_tile = [&](int t, int j, uint32_t k_base) {
        const uint32_t q_base = smem_u32(smem + C::Q_OFF + t * C::TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * ATOM + (kk & 3) * 32;
          umma(tmem + t * BN, desc_k_sw128(q_base + off), desc_k_sw128(k_base + off), IDS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      if (!mbar_wait(q_full, 0, p.err, kDevErrFullWait)) ok = false;
      if (ok && n > 0) {
        if (!mbar_wait(&kv_full[0], 0, p.err, kDevErrFullWait)) ok = false;
        if (ok) {
          tc_fence_after();
          const uint32_t k_base = smem_u32(smem + C::KV_OFF);
          for (int t = 0; t < NT; ++t) issue_s_tile(t, 0, k_base);
          umma_commit(&kv_empty[0]);
        }
      }
      // Per j and tile: O_t += P_t(j) V_j (P from TMEM, where it overwrote
      // S_t(j)), then S_t(j+1) into the same columns: the tensor pipe runs in
      // issue order, so S_t(j+1) lands after P_t(j) has been read, and
      // s_full_t(j+1) also tells the softmax that P_t(j) V_j is in O_t.
      for (int j = 0; ok && j < n; ++j) {
        const int itv = 2 * j + 1, sv = itv % NS;
        const int itk = 2 * j + 2, sk = itk % NS;
        const bool more = j + 1 < n;
        if (!mbar_wait(&kv_full[sv], (itv / NS) & 1, p.err, kDevErrFullWait)) { ok = false; break; }
        if (more && !mbar_wait(&kv_full[sk], (itk / NS) & 1, p.err, kDevErrFullWait)) { ok = false; break; }
        const uint32_t v_base = smem_u32(smem + C::KV_OFF + sv * C::TILE);
        const uint32_t k_base = smem_u32(smem + C::KV_OFF + sk * C::TILE);
        for (int t = 0; t < NT && ok; ++t) {
          if (!mbar_wait(&p_full[t], j & 1, p.err, kDevErrMmaWait)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const uint64_t db = desc_mn_sw128(v_base + kk * 2048, ATOM);
            umma_ts(tmem + C::O_COL + t * D, tmem + t * BN + kk * 8, db, IDO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&p_empty[t]);
          if (more) issue_s_tile(t, j + 1, k_base);
        }
        if (!ok) break;
        umma_commit(&kv_empty[sv]);
        if (more) umma_commit(&kv_empty[sk]);
      }
    }
    __syncwarp();
    // TMEM is freed only after the softmax warps have read O.
    mbar_wait(done, 0, p.err, kDevErrMmaWait);
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
    return;
  }

  // --------------------------------- softmax ---------------------------------
  const int t = warp >> 2;  // query tile
  const int quarter = warp & 3;
  const int row = 32 * quarter + lane;
  const uint32_t tlane = tmem + ((uint32_t)(32 * quarter) << 16);
  const uint32_t s_col = t * BN, o_col = C::O_COL + t * D;
  float m_used = -INFINITY, l = 0.f;
  float s[BN];
  bool ok = true;
  for (int j = 0; j < n; ++j) {
    if (!mbar_wait(&s_full[t], j & 1, p.err, kDevErrMmaWait)) {
      ok = false;
      break;
    }
    tc_fence_after();
#pragma unroll
    for (int c = 0; c < BN / 32; ++c) tmem_ld32(tlane + s_col + c * 32, s + c * 32);
    tmem_ld_wait();

    const int valid = p.Lkv - j * BN;  // keys of this tile inside the sequence
    if (valid < BN) {                  // tail tile only (warp-uniform)
#pragma unroll
      for (int i = 0; i < BN; ++i)
        if (i >= valid) s[i] = -INFINITY;
    }
    // Row max of the raw scores (scale > 0), as a tree: 4 independent chains.
    float mx4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) mx4[u] = s[u];
#pragma unroll
    for (int i = 4; i < BN; i += 4)
#pragma unroll
      for (int u = 0; u < 4; ++u) mx4[u] = fmaxf(mx4[u], s[i + u]);
    const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
    // New reference max only when some row's max grew past the threshold
    // (warp-uniform, since the O rescale below uses warp-collective tcgen05.ld/st).
    // Rows whose max did not move get alpha = 1. P_t(j-1) V_{j-1} is already in
    // O_t: it was issued before S_t(j), whose completion this warp waited for.
    const bool grow = mx > m_used + kRescaleThreshold;
    const bool rescale = __any_sync(0xffffffffu, grow);
    float alpha = 1.f;
    if (rescale) {
      const float m_new = fmaxf(m_used, mx);
      alpha = ex2(m_used - m_new);  // 0 on the first tile (m_used = -inf)
      l *= alpha;
      m_used = m_new;
    }
    // p = 2^(s * scale_log2 - m), packed to bf16 pairs and written over S_t in
    // TMEM (64 columns), 64 scores at a time; row sum as 4 chains.
    const float neg_m = -m_used;
    float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float e0 = ex2(fmaf(s[64 * h + 2 * i], p.scale_log2, neg_m));
        const float e1 = ex2(fmaf(s[64 * h + 2 * i + 1], p.scale_log2, neg_m));
        rs4[i & 3] += e0 + e1;
        pk[i] = pack_bf16x2(e0, e1);
      }
      tmem_st32u(tlane + s_col + 32 * h, pk);
      tmem_st_wait();
    }
    l += (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
    // O_t *= alpha before P_t(j) V_j accumulates into it.
    if (rescale && j > 0) {
      float o[32];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        tmem_ld32(tlane + o_col + c * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= alpha;
        tmem_st32(tlane + o_col + c * 32, o);
      }
      tmem_st_wait();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&p_full[t]);
  }

  // ------------------------------ epilogue ------------------------------
  const int qrow = (qt * NT + t) * BM + row;
  if (ok && n > 0 && mbar_wait(&p_empty[t], (n - 1) & 1, p.err, kDevErrMmaWait)) {
    tc_fence_after();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __nv_bfloat16* orow = p.o + ((size_t)bh * p.Lq + qrow) * D;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      float o[32];
      tmem_ld32(tlane + o_col + c * 32, o);
      tmem_ld_wait();
      if (qrow < p.Lq) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 v;
          v.x = pack_bf16x2(o[i + 0] * inv, o[i + 1] * inv);
          v.y = pack_bf16x2(o[i + 2] * inv, o[i + 3] * inv);
          v.z = pack_bf16x2(o[i + 4] * inv, o[i + 5] * inv);
          v.w = pack_bf16x2(o[i + 6] * inv, o[i + 7] * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + i) = v;
        }
      }
    }
    if (p.lse && qrow < p.Lq)
      p.lse[(size_t)bh * p.Lq + qrow] = l > 0.f ? (m_used + __log2f(l)) * 0.69314718055994531f : -INFINITY;
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(done);
}

template <int D>
static int launch(const void* q, const void* k, const void* v, void* o, float* lse, int B, int H, int Hkv, int Lq,
                  int Lkv, float scale, cudaStream_t stream) {
  using Cf = Cfg<D>;
  int* err = device_error_word();
  if (!err) return fail(kErrCuda, "device error word unavailable");
  CUtensorMap tmQ, tmK, tmV;
  const uint32_t box[3] = {64, 128, 1};
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)Lq, (uint64_t)B * H};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)Lq * D * 2};
    int rc = encode_tma(&tmQ, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)Lkv, (uint64_t)B * Hkv};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)Lkv * D * 2};
    int rc = encode_tma(&tmK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(k), dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    rc = encode_tma(&tmV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(v), dims, strides, box,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  Params p;
  p.o = static_cast<__nv_bfloat16*>(o);
  p.lse = lse;
  p.err = err;
  p.H = H;
  p.G = H / Hkv;
  p.Lq = Lq;
  p.Lkv = Lkv;
  p.nkv = (Lkv + BN - 1) / BN;
  p.scale_log2 = scale * 1.4426950408889634f;
  auto kern = fmha_fwd_kernel<D>;
  FK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::SMEM));
  const dim3 grid((unsigned)((Lq + NT * BM - 1) / (NT * BM)), (unsigned)(B * H), 1);
  kern<<<grid, NTHREADS, Cf::SMEM, stream>>>(tmQ, tmK, tmV, p);
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace fa
}  // namespace fk

using namespace fk;

extern "C" int fk_prefill_attn_fwd(const void* q, const void* k, const void* v, void* out, float* lse, int batch,
                                   int num_heads_q, int num_heads_kv, int seqlen_q, int seqlen_kv, int head_dim,
                                   float softmax_scale, void* stream) {
  FK_CHECK_ARG(q && k && v && out, "null tensor pointer");
  FK_CHECK_ARG(batch >= 1 && seqlen_q >= 1 && seqlen_kv >= 1, "sizes must be positive");
  FK_CHECK_ARG(num_heads_kv >= 1 && num_heads_q >= num_heads_kv && num_heads_q % num_heads_kv == 0,
               "num_heads_q must be a positive multiple of num_heads_kv");
  FK_CHECK_ARG(head_dim == 64 || head_dim == 128, "head_dim must be 64 or 128");
  FK_CHECK_ARG((long long)batch * num_heads_q <= 65535, "batch * num_heads_q must be <= 65535");
  FK_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v & 15) == 0 &&
                   ((uintptr_t)out & 15) == 0,
               "tensors must be 16-byte aligned");
  FK_CHECK_ARG(softmax_scale > 0.f, "softmax_scale must be positive");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (head_dim == 64)
    return fa::launch<64>(q, k, v, out, lse, batch, num_heads_q, num_heads_kv, seqlen_q, seqlen_kv, softmax_scale,
                          st);
  return fa::launch<128>(q, k, v, out, lse, batch, num_heads_q, num_heads_kv, seqlen_q, seqlen_kv, softmax_scale,
                         st);
}
