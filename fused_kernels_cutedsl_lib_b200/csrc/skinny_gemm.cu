// Persistent stream-K weight-streaming GEMM for M <= 16 on sm_100a:
//   y[M, N] = epilogue( x[M, K] . W[N, K]^T )
//
// Replaces, for decode-sized M, the reference's GEMM family: Gemm4SM90
// (python/cutedsl_kernels/gemm/kernel/attempt4.py:48-550), RMSNormLinear1SM90
// (rmsnorm_linear/attempt1/gemm.py:51-703) and Swiglu2SM90
// (swiglu/attempt1/gemm2.py:68-688), and the operand swap of the reference's
// skinny projection DAttn2 (decoding_attention/attempt2.py:120-121): W supplies
// the 16-row M side of mma.sync m16n8k16 and the M<=16 tokens are the N side.
//
// Work decomposition (stream-K): the iteration space is
// (row block of 128 output features) x (k block of 128). Every CTA of a
// persistent grid (one per SM) takes an equal contiguous share of it, so all
// SMs stream the same number of weight bytes. A row block finished inside one
// CTA goes straight to the epilogue. A row block split between CTAs is merged
// by whichever contributor arrives last at its counter: contributors write
// fp32 partials to the caller's workspace, fence, and add their k-block count
// to the counter; the CTA that completes the count sums all partials in
// contributor order (deterministic), applies the epilogue and resets the
// counter to zero for the next call. No CTA ever waits on another.
//
// Pipeline: one producer warp issues TMA loads of the W tile (128 rows x 128 k,
// two 128B-swizzled boxes; a second tile for the SwiGLU up rows), the x tile
// (M padded to 8/16 rows; out-of-range rows are zero-filled by TMA) and, for
// RMSNorm, the gamma slice, into a STAGES-deep mbarrier ring. Eight consumer
// warps each own 16 output features: ldmatrix A (W) and B (x) fragments, two
// independent mma.sync accumulator chains.
//
// Epilogues:
//   plain    y = acc (+ residual)
//   RMSNorm  x is multiplied by gamma on the B fragments in fp32 and split
//            into bf16 hi + lo parts, both fed to the MMA (~16-bit mantissa);
//            the per-token sum of squares of x is accumulated from the same
//            fragments and y = acc * rsqrt(ss/K + eps) — the normalisation of
//            rmsnorm_linear/attempt1/gemm.py:509-547 computed in the mainloop,
//            with gamma added.
//   SwiGLU   y = silu(acc_gate) * acc_up, gate rows [n0,n1) paired with up rows
//            (swiglu/attempt1/gemm2.py:63-66, 375; demo/swiglu.py:47-49).
#include <math.h>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace sk {

constexpr int RB = 128;                       // output features per row block
constexpr int KT = 128;                       // k per pipeline stage
constexpr int NCW = 8;                        // consumer warps, 16 features each
constexpr int NTHREADS = (NCW + 1) * 32;
constexpr int WBOX_BYTES = RB * 128;          // 128 rows x 64 k x 2 B
constexpr int WTILE_BYTES = 2 * WBOX_BYTES;   // 128 rows x 128 k
constexpr int MAXM = 16;
constexpr size_t kSmemBudget = 227 * 1024;

template <int NT, bool SWIGLU, bool NORM>
struct Layout {
  static constexpr int XBOX_BYTES = NT * 8 * 128;
  static constexpr int W_BYTES = WTILE_BYTES * (SWIGLU ? 2 : 1);
  static constexpr int X_OFF = W_BYTES;
  static constexpr int G_OFF = X_OFF + 2 * XBOX_BYTES;
  static constexpr int TX_BYTES = W_BYTES + 2 * XBOX_BYTES + (NORM ? KT * 2 : 0);
  static constexpr int STAGE_BYTES = ((G_OFF + (NORM ? KT * 2 : 0)) + 1023) / 1024 * 1024;
  static constexpr int STAGES_FIT = (int)((kSmemBudget - 2048) / STAGE_BYTES);
  // RMSNorm at M <= 8: a 4-stage ring (measured 16.9 vs 17.5 us back to back for
  // the 50 MB QKV projection at M = 1; no change at M = 16 or without RMSNorm).
  static constexpr int STAGES_CAP = (NORM && NT == 1) ? 4 : 8;
  static constexpr int STAGES = STAGES_FIT > STAGES_CAP ? STAGES_CAP : STAGES_FIT;
  static constexpr size_t SMEM = 1024 + (size_t)STAGES * STAGE_BYTES + 2 * STAGES * 8 + 16 * 4 + 16;
};

// Floats per partial slot: accumulators [RB][16] (x2 for SwiGLU) + sum of squares [16].
__host__ __device__ constexpr int slot_floats(bool swiglu) { return RB * 16 * (swiglu ? 2 : 1) + 16; }

struct Params {
  const __nv_bfloat16* residual;  // [M, N] or null
  __nv_bfloat16* y;               // [M, N]
  int* counters;                  // [num_rb], zero between calls
  float* partials;                // [2 * G][slot_floats]
  int* err;
  int M, N, K, KI, num_rb, up_row_offset;
  int KI_main;                    // k blocks of x . W^T; blocks [KI_main, KI) are the LoRA segment
  long long total;                // num_rb * KI
  int G;
  float eps, inv_k;
  KvAppend kv;
  OutPlace out;                   // row strides of y / residual and peer copies of y
  int has_ext;                    // peers or KV append present
  PeerWait wait;                  // cross-GPU stage wait before x is read (counter null: none)
};

__device__ __forceinline__ long long it_start(const Params& p, int c) {
  return (long long)c * p.total / p.G;
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.f + __expf(-g)); }

template <int NT, bool SWIGLU, bool NORM>
__global__ void __launch_bounds__(NTHREADS, 1)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmWu,
                       const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmG,
                       Params p) {
  using LY = Layout<NT, SWIGLU, NORM>;
  constexpr int STAGES = LY::STAGES;
  constexpr int NMAT = SWIGLU ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * LY::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  float* ss_sm = reinterpret_cast<float*>(empty + STAGES);  // [16]
  int* flag_sm = reinterpret_cast<int*>(ss_sm + 16);
  volatile int* s_abort = reinterpret_cast<volatile int*>(flag_sm + 1);  // a consumer wait ran out

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const long long it_begin = it_start(p, cta);
  const long long it_end = it_start(p, cta + 1);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    *s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == NCW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      if (SWIGLU) tma_prefetch_desc(&tmWu);
      tma_prefetch_desc(&tmX);
      if (NORM) tma_prefetch_desc(&tmG);
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_x = l2_policy_evict_last();
      // LoRA (plain linear only): k blocks past KI_main read B (in the tmWu slot)
      // and x . A^T (in the tmG slot) instead of W and x; the zero fill past
      // the rank makes the extra columns contribute nothing.
      auto load_w = [&](int s, long long it) {
        const int rb = (int)(it / p.KI);
        const int kb = (int)(it - (long long)rb * p.KI);
        const bool lora = !SWIGLU && !NORM && kb >= p.KI_main;
        const CUtensorMap* wm = lora ? &tmWu : &tmW;
        const int k0 = (lora ? kb - p.KI_main : kb) * KT;
        uint8_t* st = smem + s * LY::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], LY::TX_BYTES);
        tma_load_2d(st, wm, &full[s], k0, rb * RB, pol_w);
        tma_load_2d(st + WBOX_BYTES, wm, &full[s], k0 + 64, rb * RB, pol_w);
        if (SWIGLU) {
          tma_load_2d(st + WTILE_BYTES, &tmWu, &full[s], k0, p.up_row_offset + rb * RB, pol_w);
          tma_load_2d(st + WTILE_BYTES + WBOX_BYTES, &tmWu, &full[s], k0 + 64, p.up_row_offset + rb * RB, pol_w);
        }
      };
      auto load_x = [&](int s, long long it) {
        const int kb = (int)(it % p.KI);
        const bool lora = !SWIGLU && !NORM && kb >= p.KI_main;
        const CUtensorMap* xm = lora ? &tmG : &tmX;
        const int k0 = (lora ? kb - p.KI_main : kb) * KT;
        uint8_t* st = smem + s * LY::STAGE_BYTES;
        tma_load_2d(st + LY::X_OFF, xm, &full[s], k0, 0, pol_x);
        tma_load_2d(st + LY::X_OFF + LY::XBOX_BYTES, xm, &full[s], k0 + 64, 0, pol_x);
        if (NORM) {
          asm volatile(
              "cp.async.bulk.tensor.1d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
              " [%0], [%1, {%2}], [%3], %4;" ::"r"(smem_u32(st + LY::G_OFF)),
              "l"(reinterpret_cast<uint64_t>(&tmG)), "r"(k0), "r"(smem_u32(&full[s])), "l"(pol_x)
              : "memory");
        }
      };
      // Weights never depend on the previous kernel on the stream: the first
      // ring of W tiles is requested before waiting for it (programmatic
      // dependent launch); x (the previous kernel's output) only after.
      const long long pre_end = it_begin + STAGES < it_end ? it_begin + STAGES : it_end;
      for (long long it = it_begin; it < pre_end; ++it) load_w((int)(it - it_begin), it);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      // x may be the output of other GPUs' stage: wait for their signals. The
      // consumers write y only after consuming x, so they are ordered after this.
      peer_wait(p.wait, p.err);
      for (long long it = it_begin; it < pre_end; ++it) load_x((int)(it - it_begin), it);
      int stage = (int)((pre_end - it_begin) % STAGES);
      uint32_t phase = (pre_end - it_begin) >= STAGES ? 1u : 0u;
      for (long long it = pre_end; it < it_end; ++it) {
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kDevErrEmptyWait)) return;
        load_w(stage, it);
        load_x(stage, it);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int g = lane >> 2;
  const int c = lane & 3;
  const int j = lane >> 3;
  const int r = lane & 7;
  const int ctid = threadIdx.x;  // 0..255
  asm volatile("griddepcontrol.wait;" ::: "memory");  // writes only after the previous kernel completed
  int stage = 0;
  uint32_t phase = 0;

  long long it = it_begin;
  while (it < it_end) {
    const int rb = (int)(it / p.KI);
    const long long seg_lo = it;
    const long long seg_hi = min(it_end, (long long)(rb + 1) * p.KI);
    const bool full_rb = (seg_lo == (long long)rb * p.KI) && (seg_hi == (long long)(rb + 1) * p.KI);

    float acc[NMAT][2][NT][4];
#pragma unroll
    for (int a = 0; a < NMAT; ++a)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int t = 0; t < NT; ++t) acc[a][h][t][0] = acc[a][h][t][1] = acc[a][h][t][2] = acc[a][h][t][3] = 0.f;
    float ss[NT];
#pragma unroll
    for (int t = 0; t < NT; ++t) ss[t] = 0.f;

    for (; it < seg_hi; ++it) {
      // A time-out leaves the k loop; every consumer warp then stops at the
      // barrier after it and all return together.
      if (!mbar_wait_group(&full[stage], phase, p.err, kDevErrFullWait, s_abort)) break;
      const uint8_t* st = smem + stage * LY::STAGE_BYTES;
      const uint32_t wb = smem_u32(st);
      const uint32_t xb = smem_u32(st + LY::X_OFF);

      // B fragments (x^T): bx[t][s][0..1] for k-steps s = 0..7 of this stage.
      uint32_t bx[NT][8][2];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int s = 0; s < 8; s += 2) {
          const uint32_t base = xb + (s >> 2) * LY::XBOX_BYTES;
          ldsm_x4(swz128(base, t * 8 + r, 2 * (s & 3) + j), bx[t][s][0], bx[t][s][1], bx[t][s + 1][0],
                  bx[t][s + 1][1]);
        }
      // RMSNorm: x*gamma is split into bf16 hi + lo parts (hi = bf16(x*gamma),
      // lo = bf16(x*gamma - hi)) and both are multiplied into the same
      // accumulators, so the product keeps ~16 mantissa bits instead of 8.
      uint32_t bl[NORM ? NT : 1][8][2];
      if (NORM) {
        const uint32_t* gam = reinterpret_cast<const uint32_t*>(st + LY::G_OFF);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          const float2 g0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gam[(16 * s + 2 * c) >> 1]));
          const float2 g1 =
              __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gam[(16 * s + 8 + 2 * c) >> 1]));
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float2 f0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bx[t][s][0]));
            const float2 f1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bx[t][s][1]));
            if (warp == 0) {
              ss[t] = fmaf(f0.x, f0.x, ss[t]);
              ss[t] = fmaf(f0.y, f0.y, ss[t]);
              ss[t] = fmaf(f1.x, f1.x, ss[t]);
              ss[t] = fmaf(f1.y, f1.y, ss[t]);
            }
            const float p0 = f0.x * g0.x, p1 = f0.y * g0.y, p2 = f1.x * g1.x, p3 = f1.y * g1.y;
            const __nv_bfloat162 h0 = __floats2bfloat162_rn(p0, p1);
            const __nv_bfloat162 h1 = __floats2bfloat162_rn(p2, p3);
            const float2 q0 = __bfloat1622float2(h0), q1 = __bfloat1622float2(h1);
            bx[t][s][0] = *reinterpret_cast<const uint32_t*>(&h0);
            bx[t][s][1] = *reinterpret_cast<const uint32_t*>(&h1);
            bl[NORM ? t : 0][s][0] = pack_bf16x2(p0 - q0.x, p1 - q0.y);
            bl[NORM ? t : 0][s][1] = pack_bf16x2(p2 - q1.x, p3 - q1.y);
          }
        }
      }
#pragma unroll
      for (int a = 0; a < NMAT; ++a) {
        const uint32_t abase = wb + a * WTILE_BYTES;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          uint32_t af[4];
          ldsm_x4(swz128(abase + (s >> 2) * WBOX_BYTES, 16 * warp + (j & 1) * 8 + r, 2 * (s & 3) + (j >> 1)),
                  af[0], af[1], af[2], af[3]);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            mma_bf16_16816(acc[a][s & 1][t], af, bx[t][s][0], bx[t][s][1]);
            if (NORM) mma_bf16_16816(acc[a][(s & 1) ^ 1][t], af, bl[NORM ? t : 0][s][0], bl[NORM ? t : 0][s][1]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1;
      }
    }

    named_bar_sync(1, NCW * 32);
    if (*s_abort) return;  // uniform: the flag is only written inside the k loop above

    // ------------------------- segment epilogue -------------------------
    float v[NMAT][NT][4];
#pragma unroll
    for (int a = 0; a < NMAT; ++a)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) v[a][t][e] = acc[a][0][t][e] + acc[a][1][t][e];
    if (NORM && warp == 0) {
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], 1);
        ss[t] += __shfl_xor_sync(0xffffffffu, ss[t], 2);
      }
    }
    const int row = 16 * warp + g;  // local feature row of c0/c1; c2/c3 are row + 8

    bool do_epilogue = full_rb;
    if (!full_rb) {
      // Write this segment's partial, then count it in.
      const int slot = 2 * cta + (seg_lo == it_begin ? 0 : 1);
      float* sp = p.partials + (size_t)slot * slot_floats(SWIGLU);
#pragma unroll
      for (int a = 0; a < NMAT; ++a)
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          float* d = sp + a * RB * 16 + row * 16 + t * 8 + 2 * c;
          __stcg(reinterpret_cast<float2*>(d), make_float2(v[a][t][0], v[a][t][1]));
          __stcg(reinterpret_cast<float2*>(d + 8 * 16), make_float2(v[a][t][2], v[a][t][3]));
        }
      if (NORM && warp == 0 && c == 0) {
#pragma unroll
        for (int t = 0; t < NT; ++t) __stcg(sp + NMAT * RB * 16 + t * 8 + g, ss[t]);
      }
      __threadfence();
      named_bar_sync(1, NCW * 32);
      if (ctid == 0) {
        const int cnt = (int)(seg_hi - seg_lo);
        const int prev = atomicAdd(p.counters + rb, cnt);
        const int last = (prev + cnt == p.KI);
        if (last) p.counters[rb] = 0;  // every contribution is in: reset for the next call
        *flag_sm = last;
      }
      named_bar_sync(1, NCW * 32);
      do_epilogue = (*flag_sm != 0);
      if (do_epilogue) {
        __threadfence();
        // Sum every contributor's partial, in contributor order.
        const long long lo = (long long)rb * p.KI, hi = lo + p.KI;
        int cf = (int)(lo * p.G / p.total);
        while (cf > 0 && it_start(p, cf) > lo) --cf;
        while (it_start(p, cf + 1) <= lo) ++cf;
#pragma unroll
        for (int a = 0; a < NMAT; ++a)
#pragma unroll
          for (int t = 0; t < NT; ++t) v[a][t][0] = v[a][t][1] = v[a][t][2] = v[a][t][3] = 0.f;
        float ssum[2 * NT];
#pragma unroll
        for (int e = 0; e < 2 * NT; ++e) ssum[e] = 0.f;
        for (int cc = cf; cc < p.G && it_start(p, cc) < hi; ++cc) {
          if (it_start(p, cc + 1) == it_start(p, cc)) continue;  // empty range: no partial
          const int sl = 2 * cc + (it_start(p, cc) >= lo ? 0 : 1);
          const float* q = p.partials + (size_t)sl * slot_floats(SWIGLU);
#pragma unroll
          for (int a = 0; a < NMAT; ++a)
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              const float* s0 = q + a * RB * 16 + row * 16 + t * 8 + 2 * c;
              const float2 u0 = __ldcg(reinterpret_cast<const float2*>(s0));
              const float2 u1 = __ldcg(reinterpret_cast<const float2*>(s0 + 8 * 16));
              v[a][t][0] += u0.x;
              v[a][t][1] += u0.y;
              v[a][t][2] += u1.x;
              v[a][t][3] += u1.y;
            }
          if (NORM) {
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              ssum[2 * t] += __ldcg(q + NMAT * RB * 16 + t * 8 + 2 * c);
              ssum[2 * t + 1] += __ldcg(q + NMAT * RB * 16 + t * 8 + 2 * c + 1);
            }
          }
        }
        if (NORM) {
          // Per-thread: token m = t*8 + 2c (+1)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const float r0 = rsqrtf(ssum[2 * t] * p.inv_k + p.eps);
            const float r1 = rsqrtf(ssum[2 * t + 1] * p.inv_k + p.eps);
#pragma unroll
            for (int a = 0; a < NMAT; ++a) {
              v[a][t][0] *= r0;
              v[a][t][1] *= r1;
              v[a][t][2] *= r0;
              v[a][t][3] *= r1;
            }
          }
        }
      }
    } else if (NORM) {
      if (warp == 0 && c == 0) {
#pragma unroll
        for (int t = 0; t < NT; ++t) ss_sm[t * 8 + g] = ss[t];
      }
      named_bar_sync(1, NCW * 32);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const float r0 = rsqrtf(ss_sm[t * 8 + 2 * c] * p.inv_k + p.eps);
        const float r1 = rsqrtf(ss_sm[t * 8 + 2 * c + 1] * p.inv_k + p.eps);
#pragma unroll
        for (int a = 0; a < NMAT; ++a) {
          v[a][t][0] *= r0;
          v[a][t][1] *= r1;
          v[a][t][2] *= r0;
          v[a][t][3] *= r1;
        }
      }
      named_bar_sync(1, NCW * 32);  // ss_sm is rewritten by the next segment
    }

    if (do_epilogue) {
      const int col0 = rb * RB + row;
      __nv_bfloat16 o[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int m = t * 8 + 2 * c + (e & 1);
          const int col = col0 + (e >> 1) * 8;
          if (m < p.M && col < p.N) {
            float val = SWIGLU ? silu_f(v[0][t][e]) * v[NMAT - 1][t][e] : v[0][t][e];
            if (p.residual) val += __bfloat162float(p.residual[(size_t)m * p.out.ldr + col]);
            o[t][e] = __float2bfloat16_rn(val);
            p.y[(size_t)m * p.out.ldy + col] = o[t][e];
          }
        }
      // Extra destinations (peer copies, KV append) in their own loop, only when
      // present: inlined into every store above they slow the kernel through code size.
      if (p.has_ext) {
        for (int t = 0; t < NT; ++t)
          for (int e = 0; e < 4; ++e) {
            const int m = t * 8 + 2 * c + (e & 1);
            const int col = col0 + (e >> 1) * 8;
            if (m < p.M && col < p.N) {
              store_out_all(p.out, p.y, (size_t)m * p.out.ldy + col, o[t][e]);
              kv_append_store(p.kv, m, col, o[t][e]);
            }
          }
      }
    }
  }
}

template <int NT, bool SWIGLU, bool NORM>
static int launch(const CUtensorMap& tmW, const CUtensorMap& tmWu, const CUtensorMap& tmX,
                  const CUtensorMap& tmG, Params p, cudaStream_t stream) {
  using LY = Layout<NT, SWIGLU, NORM>;
  static_assert(LY::STAGES >= 2, "stage does not fit");
  auto kern = skinny_gemm_kernel<NT, SWIGLU, NORM>;
  FK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LY::SMEM));
  // Programmatic dependent launch: the weight stream of this GEMM may start
  // while the previous kernel on the stream drains (see the producer).
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.G, 1, 1);
  cfg.blockDim = dim3(NTHREADS, 1, 1);
  cfg.dynamicSmemBytes = LY::SMEM;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, kern, tmW, tmWu, tmX, tmG, p));
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}

}  // namespace sk

// Workspace layout shared by the skinny path: [counters: num_rb ints, 256-B aligned][partials].
size_t skinny_workspace_bytes(int N, int G, bool swiglu) {
  const int num_rb = (N + sk::RB - 1) / sk::RB;
  (void)num_rb;
  return kCounterBytes + (size_t)2 * G * sk::slot_floats(swiglu) * 4;
}

// Shared entry used by every skinny-path C function. `w_up` null => no SwiGLU.
int skinny_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                  const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
                  size_t workspace_bytes, int grid_override, cudaStream_t stream, const LinearExtras* ex) {
  FK_CHECK_ARG(x && w && y, "null tensor pointer");
  FK_CHECK_ARG(M >= 1 && M <= sk::MAXM, "skinny path takes 1 <= M <= 16");
  const bool lora = ex && ex->lora_xa;
  FK_CHECK_ARG(!lora || (!gamma && !w_up), "LoRA is supported on the plain linear only");
  FK_CHECK_ARG(!lora || (ex->lora_b && ex->lora_rank >= 8 && ex->lora_rank % 8 == 0 &&
                         ((uintptr_t)ex->lora_xa & 15) == 0 && ((uintptr_t)ex->lora_b & 15) == 0),
               "LoRA: rank must be a positive multiple of 8 and xA / B 16-byte aligned");
  FK_CHECK_ARG(N >= 1 && K >= 1, "N and K must be positive");
  FK_CHECK_ARG(K % 8 == 0, "K must be a multiple of 8 (16-byte rows for TMA)");
  FK_CHECK_ARG((N + 127) / 128 <= kMaxRowBlocks, "N too large: at most 4096 row blocks of 128");
  FK_CHECK_ARG(((uintptr_t)x & 15) == 0 && ((uintptr_t)w & 15) == 0 && (!w_up || ((uintptr_t)w_up & 15) == 0) &&
                   (!gamma || ((uintptr_t)gamma & 15) == 0),
               "x, w, gamma must be 16-byte aligned");
  FK_CHECK_ARG(workspace != nullptr && ((uintptr_t)workspace & 255) == 0, "workspace must be 256-byte aligned");
  const bool sw = w_up != nullptr;
  const bool norm = gamma != nullptr;
  const int num_rb0 = (N + sk::RB - 1) / sk::RB;
  const int KI_main = (K + sk::KT - 1) / sk::KT;
  const int KI_all = KI_main + (lora ? (ex->lora_rank + sk::KT - 1) / sk::KT : 0);
  const long long total0 = (long long)num_rb0 * KI_all;
  int G = grid_override > 0 ? grid_override : num_sms();
  if ((long long)G > total0) G = (int)total0;
  FK_CHECK_ARG(workspace_bytes >= skinny_workspace_bytes(N, G, sw), "workspace too small");
  int* err = device_error_word();
  if (!err) return fail(kErrCuda, "device error word unavailable");

  sk::Params p;
  p.residual = static_cast<const __nv_bfloat16*>(residual);
  p.y = static_cast<__nv_bfloat16*>(y);
  p.counters = static_cast<int*>(workspace);
  const int num_rb = (N + sk::RB - 1) / sk::RB;
  p.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kCounterBytes);
  p.err = err;
  p.M = M;
  p.N = N;
  p.K = K;
  p.KI = KI_all;
  p.KI_main = KI_main;
  p.kv = {};
  p.out = {};
  p.wait = {};
  if (ex) {
    p.kv = ex->kv;
    p.kv.m_base = 0;
    p.out = ex->out;
    p.wait = ex->wait;
  }
  if (p.out.ldy <= 0) p.out.ldy = N;
  if (p.out.ldr <= 0) p.out.ldr = N;
  p.has_ext = (p.out.npeers > 0 || p.kv.k_cache != nullptr) ? 1 : 0;
  p.num_rb = num_rb;
  p.up_row_offset = up_row_offset;
  p.total = (long long)num_rb * p.KI;
  p.G = G;
  p.eps = eps;
  p.inv_k = 1.f / (float)K;

  const int NT = M <= 8 ? 1 : 2;
  CUtensorMap tmW, tmWu, tmX, tmG;
  {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)(sw && w_up == w ? up_row_offset + N : N)};
    const uint64_t strides[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {64, (uint32_t)sk::RB};
    int rc = encode_tma(&tmW, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w), dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (sw) {
      const uint64_t dims_u[2] = {(uint64_t)K, (uint64_t)(up_row_offset + N)};
      rc = encode_tma(&tmWu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(w_up), dims_u, strides, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    } else {
      tmWu = tmW;
    }
    const uint64_t xdims[2] = {(uint64_t)K, (uint64_t)M};
    const uint32_t xbox[2] = {64, (uint32_t)(NT * 8)};
    rc = encode_tma(&tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), xdims, strides, xbox,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (lora) {
      const int r = ex->lora_rank;
      const uint64_t bdims[2] = {(uint64_t)r, (uint64_t)N};
      const uint64_t bstr[1] = {(uint64_t)r * 2};
      rc = encode_tma(&tmWu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ex->lora_b), bdims, bstr, box,
                      CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
      const uint64_t adims[2] = {(uint64_t)r, (uint64_t)M};
      rc = encode_tma(&tmG, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ex->lora_xa), adims, bstr, xbox,
                      CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    } else if (norm) {
      const uint64_t gdims[1] = {(uint64_t)K};
      const uint32_t gbox[1] = {(uint32_t)sk::KT};
      rc = encode_tma(&tmG, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 1, const_cast<void*>(gamma), gdims, nullptr, gbox,
                      CU_TENSOR_MAP_SWIZZLE_NONE);
      if (rc) return rc;
    } else {
      tmG = tmX;
    }
  }
#define FK_SK_LAUNCH(NTV, SWV, NV) return sk::launch<NTV, SWV, NV>(tmW, tmWu, tmX, tmG, p, stream)
  if (NT == 1) {
    if (sw) {
      if (norm) FK_SK_LAUNCH(1, true, true);
      FK_SK_LAUNCH(1, true, false);
    }
    if (norm) FK_SK_LAUNCH(1, false, true);
    FK_SK_LAUNCH(1, false, false);
  }
  if (sw) {
    if (norm) FK_SK_LAUNCH(2, true, true);
    FK_SK_LAUNCH(2, true, false);
  }
  if (norm) FK_SK_LAUNCH(2, false, true);
  FK_SK_LAUNCH(2, false, false);
#undef FK_SK_LAUNCH
}

}  // namespace fk
