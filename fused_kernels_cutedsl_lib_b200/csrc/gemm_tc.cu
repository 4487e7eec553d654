// tcgen05/TMEM GEMM for 16 < M <= 256 tokens per tile on sm_100a:
//   y[M, N] = epilogue( x[M, K] . W[N, K]^T )
//
// Replaces the reference's wgmma GEMMs (Gemm4SM90,
// python/cutedsl_kernels/gemm/kernel/attempt4.py:48-550; RMSNormLinear1SM90,
// rmsnorm_linear/attempt1/gemm.py:51-703; Swiglu2SM90, swiglu/attempt1/gemm2.py:68-688)
// for M large enough to be a dense contraction. Operands are swapped as in the
// reference's skinny projection (decoding_attention/attempt2.py:120-121): a
// 128-row W tile is the UMMA M side and the tokens are the N side
// (N_mma = M rounded up to 16, <= 256), so the accumulator is 128 TMEM lanes
// (output features) x N_mma columns (tokens). No cluster multicast.
//
// Roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: W box {64 k, 128 rows} (+ the SwiGLU up rows),
//               x box {64 k, N_mma rows}, gamma box {64} per stage
//   warp 1      allocates TMEM, one lane issues tcgen05.mma (4 x K=16 per
//               stage) and tcgen05.commit to free stages / publish results
//   warps 2-5   RMSNorm: multiply the x tile by gamma in shared memory in fp32,
//               split it into bf16 hi (in place) + lo (second tile) parts that
//               both go through the MMA, and accumulate the per-token sum of squares;
//               epilogue: tcgen05.ld the accumulators 16 columns at a time,
//               scale by rsqrt(ss/K + eps), SwiGLU, residual, bf16 store
// Work is split stream-K over (row block, k block) exactly as in the skinny
// kernel: partial row blocks go to the caller's workspace and the last
// contributor (counter) merges them in contributor order and resets the counter.
#include <math.h>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace tc {

constexpr int BM = 128;       // W rows per row block (UMMA M)
constexpr int BK = 64;        // k per stage: one 128B swizzle atom of bf16
constexpr int NTHREADS = 192; // 6 warps
constexpr int EPI_WARP0 = 2;
constexpr int EPI_THREADS = 128;
constexpr int WBOX = BM * 128;  // 16 KB
constexpr size_t kSmemBudget = 227 * 1024;

template <int NMMA, bool SWIGLU, bool NORM>
struct Layout {
  static constexpr int W_BYTES = WBOX * (SWIGLU ? 2 : 1);
  static constexpr int X_OFF = W_BYTES;
  static constexpr int X_BYTES = NMMA * 128;
  static constexpr int G_OFF = X_OFF + X_BYTES;
  // RMSNorm: the low bf16 part of x*gamma, same swizzled layout as the x tile.
  static constexpr int XL_OFF = (G_OFF + 128 + 1023) / 1024 * 1024;
  static constexpr int TX = W_BYTES + X_BYTES + (NORM ? 128 : 0);
  static constexpr int STAGE_BYTES = NORM ? XL_OFF + X_BYTES : (G_OFF + 1023) / 1024 * 1024;
  static constexpr int STAGES_FIT = (int)((kSmemBudget - 1024 - 2048) / STAGE_BYTES);
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int ACC_COLS = NMMA * (SWIGLU ? 2 : 1);
  static constexpr int TMEM_COLS = ACC_COLS <= 32 ? 32 : ACC_COLS <= 64 ? 64 : ACC_COLS <= 128 ? 128
                                   : ACC_COLS <= 256 ? 256 : 512;
  // barriers: full, xready, empty per stage + acc_full + acc_empty; tmem addr; flag; ss[256]
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + (3 * STAGES + 2) * 8 + 16 + 256 * 4;
};

__host__ __device__ constexpr int slot_floats(int nmma, bool swiglu) { return nmma * BM * (swiglu ? 2 : 1) + nmma; }

struct Params {
  const __nv_bfloat16* residual;
  __nv_bfloat16* y;
  int* counters;
  float* partials;
  int* err;
  int M, N, K, KI, num_rb, up_row_offset;
  long long total;
  int G;
  float eps, inv_k;
};

__device__ __forceinline__ long long it_start(const Params& p, int c) { return (long long)c * p.total / p.G; }
__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

// UMMA shared-memory descriptor: K-major operand, 128B swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor: kind::f16, A = B = bf16 (K-major), D = f32, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

template <int NMMA, bool SWIGLU, bool NORM>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmWu,
                   const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmG, Params p) {
  using LY = Layout<NMMA, SWIGLU, NORM>;
  constexpr int S = LY::STAGES;
  constexpr int NMAT = SWIGLU ? 2 : 1;
  constexpr int SLOT = slot_floats(NMMA, SWIGLU);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * LY::STAGE_BYTES);
  uint64_t* xready = full + S;
  uint64_t* empty = xready + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_sm = reinterpret_cast<uint32_t*>(acc_empty + 1);
  int* flag_sm = reinterpret_cast<int*>(tmem_sm + 1);
  volatile int* abort_sm = flag_sm + 1;
  float* ss_sm = reinterpret_cast<float*>(tmem_sm + 4);  // [256]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const long long it_begin = it_start(p, cta);
  const long long it_end = it_start(p, cta + 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&xready[i], 4);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    *abort_sm = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_sm)),
                 "r"(LY::TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_sm;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      tma_prefetch_desc(&tmX);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      for (long long it = it_begin; it < it_end; ++it) {
        const int rb = (int)(it / p.KI);
        const int k0 = (int)(it - (long long)rb * p.KI) * BK;
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kDevErrEmptyWait)) {
          *abort_sm = 1;
          break;
        }
        uint8_t* st = smem + stage * LY::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[stage], LY::TX);
        tma_load_2d(st, &tmW, &full[stage], k0, rb * BM, pol_w);
        if (SWIGLU) tma_load_2d(st + WBOX, &tmWu, &full[stage], k0, p.up_row_offset + rb * BM, pol_w);
        tma_load_2d(st + LY::X_OFF, &tmX, &full[stage], k0, 0, pol_x);
        if (NORM) {
          asm volatile(
              "cp.async.bulk.tensor.1d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
              " [%0], [%1, {%2}], [%3], %4;" ::"r"(smem_u32(st + LY::G_OFF)),
              "l"(reinterpret_cast<uint64_t>(&tmG)), "r"(k0), "r"(smem_u32(&full[stage])), "l"(pol_x)
              : "memory");
        }
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    constexpr uint32_t idesc = umma_idesc_bf16(NMMA);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t acc_phase = 0;
    long long it = it_begin;
    bool ok = true;
    while (ok && it < it_end) {
      const int rb = (int)(it / p.KI);
      const long long seg_hi = min(it_end, (long long)(rb + 1) * p.KI);
      if (!mbar_wait(acc_empty, acc_phase ^ 1, p.err, kDevErrMmaWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      bool first = true;
      for (; it < seg_hi; ++it) {
        uint64_t* ready = NORM ? &xready[stage] : &full[stage];
        if (!mbar_wait(ready, phase, p.err, kDevErrFullWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sb = smem_u32(smem + stage * LY::STAGE_BYTES);
          const uint64_t da = umma_desc_sw128(sb);
          const uint64_t db = umma_desc_sw128(sb + LY::X_OFF);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t acc = (first && kk == 0) ? 0u : 1u;
            umma_bf16(tmem, da + 2 * kk, db + 2 * kk, idesc, acc);
            if (SWIGLU) {
              const uint64_t du = umma_desc_sw128(sb + WBOX);
              umma_bf16(tmem + NMMA, du + 2 * kk, db + 2 * kk, idesc, acc);
            }
            if (NORM) {  // low part of x*gamma into the same accumulators
              const uint64_t dl = umma_desc_sw128(sb + LY::XL_OFF);
              umma_bf16(tmem, da + 2 * kk, dl + 2 * kk, idesc, 1u);
              if (SWIGLU) umma_bf16(tmem + NMMA, umma_desc_sw128(sb + WBOX) + 2 * kk, dl + 2 * kk, idesc, 1u);
            }
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        first = false;
        if (++stage == S) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(acc_full);
      __syncwarp();
      acc_phase ^= 1;
    }
    if (!ok) *abort_sm = 1;
  } else {
    // ------------------------- transform + epilogue -------------------------
    const int et = threadIdx.x - EPI_WARP0 * 32;  // 0..127
    const int q = warp & 3;                       // TMEM lane quarter of this warp
    const int row = 32 * q + lane;                // output feature within the row block
    const uint32_t trow = tmem + ((uint32_t)(32 * q) << 16);
    int stage = 0;
    uint32_t phase = 0;
    uint32_t acc_phase = 0;
    long long it = it_begin;
    bool ok = true;
    while (ok && it < it_end) {
      const int rb = (int)(it / p.KI);
      const long long seg_lo = it;
      const long long seg_hi = min(it_end, (long long)(rb + 1) * p.KI);
      const bool full_rb = (seg_lo == (long long)rb * p.KI) && (seg_hi == (long long)(rb + 1) * p.KI);
      float ss0 = 0.f, ss1 = 0.f;  // tokens et and et + 128
      if (NORM) {
        for (; it < seg_hi; ++it) {
          if (!mbar_wait(&full[stage], phase, p.err, kDevErrFullWait)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * LY::STAGE_BYTES;
          const uint4* gam = reinterpret_cast<const uint4*>(st + LY::G_OFF);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int tok = et + half * 128;
            if (tok < NMMA) {  // rows >= M are TMA zero-fill: their lo part is written as zero too
              uint4* xr = reinterpret_cast<uint4*>(st + LY::X_OFF + tok * 128);
              uint4* xl = reinterpret_cast<uint4*>(st + LY::XL_OFF + tok * 128);
              float ssl = 0.f;
#pragma unroll
              for (int pc = 0; pc < 8; ++pc) {
                uint4 xv = xr[pc];
                uint4 lv;
                const uint4 gv = gam[pc ^ (tok & 7)];
                uint32_t* xw = reinterpret_cast<uint32_t*>(&xv);
                uint32_t* lw = reinterpret_cast<uint32_t*>(&lv);
                const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xw[e]));
                  const float2 gg = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[e]));
                  ssl = fmaf(f.x, f.x, fmaf(f.y, f.y, ssl));
                  const float p0 = f.x * gg.x, p1 = f.y * gg.y;
                  const __nv_bfloat162 hi = __floats2bfloat162_rn(p0, p1);
                  const float2 hf = __bfloat1622float2(hi);
                  xw[e] = *reinterpret_cast<const uint32_t*>(&hi);
                  lw[e] = pack_bf16x2(p0 - hf.x, p1 - hf.y);
                }
                xr[pc] = xv;
                xl[pc] = lv;
              }
              if (half == 0) ss0 += ssl; else ss1 += ssl;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(&xready[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ss_sm[et] = ss0;
        if (et + 128 < 256) ss_sm[et + 128] = ss1;
      } else {
        it = seg_hi;
      }
      named_bar_sync(1, EPI_THREADS);  // ss_sm complete

      if (!mbar_wait(acc_full, acc_phase, p.err, kDevErrMmaWait)) {
        ok = false;
        break;
      }
      acc_phase ^= 1;
      tc_fence_after();

      const int col = rb * BM + row;
      if (full_rb) {
        for (int c0 = 0; c0 < NMMA && c0 < p.M; c0 += 16) {
          float a[16], u[16];
          tmem_ld16(trow + c0, a);
          if (SWIGLU) tmem_ld16(trow + NMMA + c0, u);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int m = c0 + i;
            if (m < p.M && col < p.N) {
              float rs = 1.f;
              if (NORM) rs = rsqrtf(ss_sm[m] * p.inv_k + p.eps);
              float val = SWIGLU ? silu_f(a[i] * rs) * (u[i] * rs) : a[i] * rs;
              const size_t off = (size_t)m * p.N + col;
              if (p.residual) val += __bfloat162float(p.residual[off]);
              p.y[off] = __float2bfloat16_rn(val);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);
      } else {
        const int slot = 2 * cta + (seg_lo == it_begin ? 0 : 1);
        float* sp = p.partials + (size_t)slot * SLOT;
        for (int c0 = 0; c0 < NMMA && c0 < p.M; c0 += 16) {
          float a[16];
          tmem_ld16(trow + c0, a);
#pragma unroll
          for (int i = 0; i < 16; ++i) __stcg(sp + (size_t)(c0 + i) * BM + row, a[i]);
          if (SWIGLU) {
            tmem_ld16(trow + NMMA + c0, a);
#pragma unroll
            for (int i = 0; i < 16; ++i) __stcg(sp + (size_t)NMMA * BM + (size_t)(c0 + i) * BM + row, a[i]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty);
        if (NORM) {
          for (int m = et; m < NMMA; m += EPI_THREADS) __stcg(sp + (size_t)NMAT * NMMA * BM + m, ss_sm[m]);
        }
        __threadfence();
        named_bar_sync(1, EPI_THREADS);
        if (et == 0) {
          const int cnt = (int)(seg_hi - seg_lo);
          const int prev = atomicAdd(p.counters + rb, cnt);
          const int last = (prev + cnt == p.KI);
          if (last) p.counters[rb] = 0;
          *flag_sm = last;
        }
        named_bar_sync(1, EPI_THREADS);
        if (*flag_sm) {
          __threadfence();
          const long long lo = (long long)rb * p.KI, hi = lo + p.KI;
          int cf = (int)(lo * p.G / p.total);
          while (cf > 0 && it_start(p, cf) > lo) --cf;
          while (it_start(p, cf + 1) <= lo) ++cf;
          // total sum of squares per token (NORM), staged in ss_sm
          if (NORM) {
            named_bar_sync(1, EPI_THREADS);
            for (int m = et; m < NMMA; m += EPI_THREADS) {
              float s = 0.f;
              for (int cc = cf; cc < p.G && it_start(p, cc) < hi; ++cc) {
                if (it_start(p, cc + 1) == it_start(p, cc)) continue;
                const int sl = 2 * cc + (it_start(p, cc) >= lo ? 0 : 1);
                s += __ldcg(p.partials + (size_t)sl * SLOT + (size_t)NMAT * NMMA * BM + m);
              }
              ss_sm[m] = s;
            }
            named_bar_sync(1, EPI_THREADS);
          }
          // Sum the contributors' partials 16 tokens at a time: 16 (or 32)
          // independent loads in flight per contributor keep this
          // throughput-bound instead of latency-bound.
          for (int c0 = 0; c0 < NMMA && c0 < p.M; c0 += 16) {
            float g[16], u[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) g[i] = u[i] = 0.f;
            for (int cc = cf; cc < p.G && it_start(p, cc) < hi; ++cc) {
              if (it_start(p, cc + 1) == it_start(p, cc)) continue;
              const int sl = 2 * cc + (it_start(p, cc) >= lo ? 0 : 1);
              const float* qp = p.partials + (size_t)sl * SLOT + (size_t)c0 * BM + row;
#pragma unroll
              for (int i = 0; i < 16; ++i) g[i] += __ldcg(qp + i * BM);
              if (SWIGLU) {
#pragma unroll
                for (int i = 0; i < 16; ++i) u[i] += __ldcg(qp + (size_t)NMMA * BM + i * BM);
              }
            }
            if (col < p.N) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int m = c0 + i;
                if (m < p.M) {
                  float rs = 1.f;
                  if (NORM) rs = rsqrtf(ss_sm[m] * p.inv_k + p.eps);
                  float val = SWIGLU ? silu_f(g[i] * rs) * (u[i] * rs) : g[i] * rs;
                  const size_t off = (size_t)m * p.N + col;
                  if (p.residual) val += __bfloat162float(p.residual[off]);
                  p.y[off] = __float2bfloat16_rn(val);
                }
              }
            }
          }
        }
      }
      named_bar_sync(1, EPI_THREADS);  // ss_sm / flag reuse by the next segment
    }
    if (!ok) *abort_sm = 1;
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(LY::TMEM_COLS));
  }
}

template <int NMMA, bool SWIGLU, bool NORM>
static int launch(const CUtensorMap& tmW, const CUtensorMap& tmWu, const CUtensorMap& tmX, const CUtensorMap& tmG,
                  const Params& p, cudaStream_t stream) {
  using LY = Layout<NMMA, SWIGLU, NORM>;
  static_assert(LY::STAGES >= 2, "stage does not fit");
  auto kern = gemm_tc_kernel<NMMA, SWIGLU, NORM>;
  FK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LY::SMEM));
  kern<<<p.G, NTHREADS, LY::SMEM, stream>>>(tmW, tmWu, tmX, tmG, p);
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}

template <bool SWIGLU, bool NORM>
static int launch_n(int nmma, const CUtensorMap& a, const CUtensorMap& b, const CUtensorMap& c, const CUtensorMap& d,
                    const Params& p, cudaStream_t st) {
  switch (nmma) {
    case 32: return launch<32, SWIGLU, NORM>(a, b, c, d, p, st);
    case 64: return launch<64, SWIGLU, NORM>(a, b, c, d, p, st);
    case 128: return launch<128, SWIGLU, NORM>(a, b, c, d, p, st);
    case 256: return launch<256, SWIGLU, NORM>(a, b, c, d, p, st);
    default: return fail(kErrUnsupported, "unsupported token tile");
  }
}

// Token tile: the smallest of {32, 64, 128, 256} covering M (capped at 256).
static int token_tile(int M) { return M <= 32 ? 32 : M <= 64 ? 64 : M <= 128 ? 128 : 256; }

}  // namespace tc

size_t tc_workspace_bytes(int M, int N, int K, bool swiglu) {
  (void)K;
  const int num_rb = (N + tc::BM - 1) / tc::BM;
  (void)num_rb;
  return kCounterBytes + (size_t)2 * num_sms() * tc::slot_floats(tc::token_tile(M), swiglu) * 4;
}

int tc_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
              const void* residual, void* y, int M, int N, int K, float eps, void* workspace, size_t workspace_bytes,
              cudaStream_t stream) {
  FK_CHECK_ARG(x && w && y, "null tensor pointer");
  FK_CHECK_ARG(M >= 1 && N >= 1 && K >= 1, "sizes must be positive");
  FK_CHECK_ARG(K % 8 == 0, "K must be a multiple of 8 (16-byte rows for TMA)");
  FK_CHECK_ARG((N + 127) / 128 <= kMaxRowBlocks, "N too large: at most 4096 row blocks of 128");
  FK_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 && (!w_up || ((uintptr_t)w_up & 15) == 0) &&
                   (!gamma || ((uintptr_t)gamma & 15) == 0),
               "x, w, gamma must be 16-byte aligned");
  FK_CHECK_ARG(workspace != nullptr && ((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  const bool sw = w_up != nullptr;
  const bool norm = gamma != nullptr;
  FK_CHECK_ARG(workspace_bytes >= tc_workspace_bytes(M, N, K, sw), "workspace too small");
  int* err = device_error_word();
  if (!err) return fail(kErrCuda, "device error word unavailable");

  const int num_rb = (N + tc::BM - 1) / tc::BM;
  const int KI = (K + tc::BK - 1) / tc::BK;
  tc::Params p;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.counters = static_cast<int*>(workspace);
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  p.err = err;
  p.N = N;
  p.K = K;
  p.KI = KI;
  p.num_rb = num_rb;
  p.up_row_offset = up_row_offset;
  p.total = (long long)num_rb * KI;
  int G = num_sms();
  if ((long long)G > p.total) G = (int)p.total;
  p.G = G;
  p.eps = eps;
  p.inv_k = 1.f / (float)K;

  CUtensorMap tmW, tmWu, tmG;
  const uint64_t strides[1] = {(uint64_t)K * 2};
  const uint32_t wbox[2] = {64, (uint32_t)tc::BM};
  const uint64_t wdims[2] = {(uint64_t)K, (uint64_t)(sw && w_up == w ? up_row_offset + N : N)};
  int rc = encode_tma(&tmW, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), wdims, strides, wbox,
                      CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  if (sw) {
    const uint64_t udims[2] = {(uint64_t)K, (uint64_t)(up_row_offset + N)};
    rc = encode_tma(&tmWu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w_up), udims, strides, wbox,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    tmWu = tmW;
  }
  if (norm) {
    const uint64_t gdims[1] = {(uint64_t)K};
    const uint32_t gbox[1] = {(uint32_t)tc::BK};
    rc = encode_tma(&tmG, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 1, const_cast<void*>(gamma), gdims, nullptr, gbox,
                    CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  } else {
    tmG = tmW;
  }
  // Token tiles of up to 256: one launch per tile, in order on the stream.
  for (int m0 = 0; m0 < M; m0 += 256) {
    const int mt = M - m0 < 256 ? M - m0 : 256;
    const int nmma = tc::token_tile(mt);
    CUtensorMap tmX;
    const uint64_t xdims[2] = {(uint64_t)K, (uint64_t)mt};
    const uint32_t xbox[2] = {64, (uint32_t)nmma};
    rc = encode_tma(&tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                    const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(x)) + (size_t)m0 * K, xdims, strides,
                    xbox, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    p.M = mt;
    p.y = static_cast<__nv_bfloat16*>(y) + (size_t)m0 * N;
    p.residual = residual ? static_cast<const __nv_bfloat16*>(residual) + (size_t)m0 * N : nullptr;
    if (!norm) tmG = tmX;
    if (sw) {
      rc = norm ? tc::launch_n<true, true>(nmma, tmW, tmWu, tmX, tmG, p, stream)
                : tc::launch_n<true, false>(nmma, tmW, tmWu, tmX, tmG, p, stream);
    } else {
      rc = norm ? tc::launch_n<false, true>(nmma, tmW, tmWu, tmX, tmG, p, stream)
                : tc::launch_n<false, false>(nmma, tmW, tmWu, tmX, tmG, p, stream);
    }
    if (rc) return rc;
  }
  return kOk;
}

}  // namespace fk
