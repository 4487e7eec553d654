// tcgen05/TMEM GEMM for M > 16 tokens on sm_100a:
//   y[M, N] = epilogue( x[M, K] . W[N, K]^T )
//
// Replaces the reference's wgmma GEMMs (Gemm4SM90,
// python/cutedsl_kernels/gemm/kernel/attempt4.py:48-550; RMSNormLinear1SM90,
// rmsnorm_linear/attempt1/gemm.py:51-703; Swiglu2SM90, swiglu/attempt1/gemm2.py:68-688)
// for M large enough to be a dense contraction. Operands are swapped as in the
// reference's skinny projection (decoding_attention/attempt2.py:120-121): a
// 128-row W tile is the UMMA M side and the tokens are the N side
// (N_mma = tokens rounded up to 32/64/128/256), so the accumulator is 128 TMEM
// lanes (output features) x N_mma columns (tokens). No cluster multicast.
//
// Roles (224 threads, one CTA per SM):
//   warp 0      weight TMA producer: W box {64 k, 128 rows} (+ the SwiGLU up
//               rows) into a deep ring; starts before griddepcontrol.wait
//   warp 6      token TMA producer: x box {64 k, N_mma rows} into a shallow
//               ring (x is re-read from L2); starts after griddepcontrol.wait
//   warp 1      allocates TMEM, one lane issues tcgen05.mma (4 x K=16 per
//               stage) and tcgen05.commit to free both rings' stages and to
//               publish results; frees TMEM once the epilogue warps report done
//   warps 2-5   epilogue: tcgen05.ld the accumulators 16 columns at a time
//               (double-buffered in TMEM when two fit in 512 columns),
//               RMSNorm scale, SwiGLU, residual, bf16 store
// Work is split stream-K over (row block, k block): every CTA streams the same
// number of weight bytes. Row blocks finished inside one CTA are written by the
// GEMM; split ones leave fp32 partials in the caller's workspace and a
// reduction kernel, launched as a programmatic dependent of the GEMM, sums them
// in contributor order (deterministic) with one CTA per (row block, 8 tokens).
//
// RMSNorm: a prologue kernel (rms_split_kernel) computes rstd per token and
// splits x*gamma into bf16 hi and lo parts, stored as token rows [0, Mp) and
// [Mp, 2Mp) of a workspace matrix; the GEMM multiplies both in one MMA (N =
// 2Mp) and the epilogue adds the two halves and scales by rstd. x*gamma is
// thus represented to ~16 mantissa bits and computed once per call instead of
// once per k block per CTA.
#include <math.h>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace tc {

constexpr int BM = 128;         // W rows per row block (UMMA M)
constexpr int BK = 64;          // k per stage: one 128B swizzle atom of bf16
constexpr int NTHREADS = 224;   // 7 warps
constexpr int EPI_WARP0 = 2;
constexpr int EPI_THREADS = 128;
constexpr int WBOX = BM * 128;  // 16 KB
constexpr int NORM_TILE = 128;  // tokens per launch with RMSNorm (hi + lo = 256 columns)
constexpr size_t kSmemBudget = 227 * 1024;
constexpr int kMaxGrid = 192;   // persistent grid bound (148 SMs on B200)
// Output staging tile of the epilogue (16 tokens x 128 features, bf16): with
// peer copies the outputs go out as 16-byte rows of 8 features instead of one
// 2-byte element per lane.
constexpr int STAGE_OUT = 16 * BM * 2;

// Two TMA rings: a deep one for the weight tiles (streamed from HBM, long
// latency) and a shallower one for the x tiles (re-read from L2 every k block,
// short latency), so that large token tiles do not crowd weights out of the
// bytes in flight.
template <int NMMA, bool SWIGLU>
struct Layout {
  static constexpr int W_BYTES = WBOX * (SWIGLU ? 2 : 1);
  static constexpr int X_BYTES = NMMA * 128;
  static constexpr int SX = X_BYTES >= 32768 ? (SWIGLU ? 2 : 3) : (X_BYTES >= 16384 ? 5 : 6);
  static constexpr int SW_FIT = (int)((kSmemBudget - 4096 - STAGE_OUT - (size_t)SX * X_BYTES) / (W_BYTES + 16));
  // As many weight stages as shared memory holds: the kernel streams at the
  // rate of (weight bytes in flight per SM) / (HBM latency under load), so a
  // deeper ring is directly faster.
  static constexpr int SW = SW_FIT > 16 ? 16 : SW_FIT;
  static constexpr int STAGES = SW;
  static constexpr int X_RING = SW * W_BYTES;
  static constexpr int ACC_COLS = NMMA * (SWIGLU ? 2 : 1);
  // Two accumulator buffers when they fit in TMEM's 512 columns: the MMA warp
  // fills one while the epilogue drains the other.
  static constexpr int NBUF = 2 * ACC_COLS <= 512 ? 2 : 1;
  static constexpr int TMEM_NEED = NBUF * ACC_COLS;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64 : TMEM_NEED <= 128 ? 128
                                   : TMEM_NEED <= 256 ? 256 : 512;
  // barriers: full + empty per W and x stage, acc_full[2], acc_empty[2], done; TMEM address
  static constexpr size_t SMEM =
      1024 + (size_t)SW * W_BYTES + (size_t)SX * X_BYTES + STAGE_OUT + (2 * SW + 2 * SX + 5) * 8 + 16;
};

__host__ __device__ constexpr int slot_floats(int nmma, bool swiglu) { return nmma * BM * (swiglu ? 2 : 1); }

struct Params {
  const __nv_bfloat16* residual;
  __nv_bfloat16* y;
  const float* rstd;  // [Mp] (RMSNorm) or null
  float* partials;
  int* err;
  int M, N, K, KI, num_rb, up_row_offset;
  int Mp;             // RMSNorm: column offset of the lo half (tokens rounded up to 16)
  long long total;
  int G;
  int KI_main;        // k blocks of x . W^T; blocks [KI_main, KI) are the LoRA segment
  KvAppend kv;
  OutPlace out;       // row strides of y / residual and peer copies of y
  int has_ext;        // peers or KV append present (store_ext needed)
  int vec_out;        // peers, no KV append, y / peers / ldy 16-byte aligned: staged 16-byte stores
  PeerWait wait;      // cross-GPU stage wait before x is read (counter null: none)
  int starts[kMaxGrid + 1];  // starts[c] = c * total / G: first iteration of CTA c
};

#ifdef FK_TC_TRACE
__device__ unsigned long long g_tc_trace[256 * 32];
#define TC_TRACE(i) g_tc_trace[blockIdx.x * 32 + (i)] = global_timer_ns()
#else
#define TC_TRACE(i) ((void)0)
#endif

__device__ __forceinline__ long long it_start(const Params& p, int c) { return p.starts[c]; }
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

// 16 accumulator columns for tokens [c0, c0+16) of one matrix; with RMSNorm the
// hi and lo halves are added (the rstd scale is applied by the caller).
template <bool NORM>
__device__ __forceinline__ void load_tokens(uint32_t trow, int c0, int Mp, float (&a)[16]) {
  tmem_ld16(trow + c0, a);
  if (NORM) {
    float b[16];
    tmem_ld16(trow + Mp + c0, b);
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] += b[i];
  }
}

// Final value of output (m, col): RMSNorm scale, SwiGLU, residual, bf16 (not stored).
__device__ __forceinline__ __nv_bfloat16 compute_out(const Params& p, int m, int col, float g, float u, bool swiglu) {
  float rs = p.rstd ? __ldg(p.rstd + m) : 1.f;
  float val = swiglu ? silu_f(g * rs) * (u * rs) : g * rs;
  if (p.residual) val += __bfloat162float(p.residual[(size_t)m * p.out.ldr + col]);
  return __float2bfloat16_rn(val);
}

// Writes a staged tile [ntok][128 features] (bf16, row-major in shared memory)
// for tokens m0.. and features col0.. to y and every peer copy as 16-byte
// rows of 8 features; a row running past N falls back to 2-byte stores.
__device__ __forceinline__ void store_staged(const Params& p, const __nv_bfloat16* st, int ntok, int m0, int col0,
                                             int tid, int nthreads) {
  for (int i = tid; i < ntok * (BM / 8); i += nthreads) {
    const int t = i / (BM / 8), f = (i % (BM / 8)) * 8;
    const int m = m0 + t, col = col0 + f;
    if (m >= p.M || col >= p.N) continue;
    const size_t off = (size_t)m * p.out.ldy + col;
    if (col + 8 <= p.N) {
      const uint4 v = *reinterpret_cast<const uint4*>(st + t * BM + f);
      *reinterpret_cast<uint4*>(p.y + off) = v;
#pragma unroll
      for (int k = 0; k < kMaxPeers; ++k)
        if (k < p.out.npeers) *reinterpret_cast<uint4*>(p.out.peer_y[k] + off) = v;
    } else {
      for (int e = 0; col + e < p.N && e < 8; ++e) store_out_all(p.out, p.y, off + e, st[t * BM + f + e]);
    }
  }
}

// Final value of output (m, col): RMSNorm scale, SwiGLU, residual, bf16; stored to y.
__device__ __forceinline__ __nv_bfloat16 store_out(const Params& p, int m, int col, float g, float u, bool swiglu) {
  float rs = p.rstd ? __ldg(p.rstd + m) : 1.f;
  float val = swiglu ? silu_f(g * rs) * (u * rs) : g * rs;
  if (p.residual) val += __bfloat162float(p.residual[(size_t)m * p.out.ldr + col]);
  const __nv_bfloat16 out = __float2bfloat16_rn(val);
  p.y[(size_t)m * p.out.ldy + col] = out;
  return out;
}
// The optional extra destinations of a stored value (peer copies, KV-cache
// append). Kept out of the per-element store above and run in a separate loop
// only when a call has them: inlined into every store they cost 5-15 % of the
// GEMM through code size.
__device__ __forceinline__ void store_ext(const Params& p, int m, int col, __nv_bfloat16 v) {
  store_out_all(p.out, p.y, (size_t)m * p.out.ldy + col, v);  // rewrites y too (same value)
  kv_append_store(p.kv, m, col, v);
}

template <int NMMA, bool SWIGLU, bool NORM>
__global__ void __launch_bounds__(NTHREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmWu,
                   const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmXa, Params p) {
  using LY = Layout<NMMA, SWIGLU>;
  constexpr int SW = LY::SW;
  constexpr int SX = LY::SX;
  constexpr int SLOT = slot_floats(NMMA, SWIGLU);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xring = smem + LY::X_RING;
  __nv_bfloat16* ostage = reinterpret_cast<__nv_bfloat16*>(xring + SX * LY::X_BYTES);  // [16][BM]
  uint64_t* full = reinterpret_cast<uint64_t*>(xring + SX * LY::X_BYTES + STAGE_OUT);  // W ring [SW]
  uint64_t* empty = full + SW;
  uint64_t* fullx = empty + SW;  // x ring [SX]
  uint64_t* emptyx = fullx + SX;
  uint64_t* acc_full = emptyx + SX;  // [2]
  uint64_t* acc_empty = acc_full + 2;  // [2]
  uint64_t* done = acc_empty + 2;
  uint32_t* tmem_sm = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* epi_abort = reinterpret_cast<volatile int*>(tmem_sm + 1);  // an epilogue wait ran out

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int cta = blockIdx.x;
  const long long it_begin = it_start(p, cta);
  const long long it_end = it_start(p, cta + 1);
  // token columns the epilogue reads: the valid tokens (NORM: of each half)
  const int mcols = NORM ? p.M : (p.M < NMMA ? p.M : NMMA);

  if (threadIdx.x == 0) {
    for (int i = 0; i < SW; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < SX; ++i) {
      mbar_init(&fullx[i], 1);
      mbar_init(&emptyx[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(done, 4);
    *epi_abort = 0;
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
  if (threadIdx.x == 0) TC_TRACE(0);
  // The split-row-block reduction kernel may be scheduled as soon as SMs free
  // up; it waits (griddepcontrol.wait) for this grid to complete before reading.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (warp == 0) {
    // --------------------------- weight TMA producer ---------------------------
    // Weights never depend on the previous kernel on the stream, so this ring
    // streams from the start, overlapping that kernel's tail (programmatic
    // dependent launch).
    if (lane == 0) {
      tma_prefetch_desc(&tmW);
      const uint64_t pol_w = l2_policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      for (long long it = it_begin; it < it_end; ++it) {
        const int rb = (int)(it / p.KI);
        const int kb = (int)(it - (long long)rb * p.KI);
        // LoRA (plain linear only): k blocks past KI_main read B from the tmWu slot.
        const bool lora = !SWIGLU && kb >= p.KI_main;
        const int k0 = (lora ? kb - p.KI_main : kb) * BK;
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err, kDevErrEmptyWait)) break;
        uint8_t* st = smem + stage * LY::W_BYTES;
        mbar_arrive_expect_tx(&full[stage], LY::W_BYTES);
        tma_load_2d(st, lora ? &tmWu : &tmW, &full[stage], k0, rb * BM, pol_w);
        if (SWIGLU) tma_load_2d(st + WBOX, &tmWu, &full[stage], k0, p.up_row_offset + rb * BM, pol_w);
        if (++stage == SW) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    __syncwarp();
    return;
  }

  if (warp == 6) {
    // ----------------------------- x TMA producer -----------------------------
    // x is the previous kernel's output: loaded only after griddepcontrol.wait.
    if (lane == 0) {
      tma_prefetch_desc(&tmX);
      const uint64_t pol_x = l2_policy_evict_last();
      asm volatile("griddepcontrol.wait;" ::: "memory");
      // x may be the output of other GPUs' stage: wait for their signals (the
      // epilogue writes only results that depend on x, so it is ordered after).
      peer_wait(p.wait, p.err);
      int stage = 0;
      uint32_t phase = 0;
      for (long long it = it_begin; it < it_end; ++it) {
        const int kb = (int)(it % p.KI);
        const bool lora = kb >= p.KI_main;  // LoRA: x . A^T
        const int k0 = (lora ? kb - p.KI_main : kb) * BK;
        if (!mbar_wait(&emptyx[stage], phase ^ 1, p.err, kDevErrEmptyWait)) break;
        mbar_arrive_expect_tx(&fullx[stage], LY::X_BYTES);
        tma_load_2d(xring + stage * LY::X_BYTES, lora ? &tmXa : &tmX, &fullx[stage], k0, 0, pol_x);
        if (++stage == SX) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    __syncwarp();
    return;
  }

  if (warp == 1) {
    // ------------------------------ MMA issuer ------------------------------
    constexpr uint32_t idesc = umma_idesc_bf16(NMMA);
    int stage = 0, xstage = 0;
    uint32_t phase = 0, xphase = 0;
    int seg = 0;  // segment counter: buffer seg % NBUF, use (seg / NBUF)
    long long it = it_begin;
    bool ok = true;
    while (ok && it < it_end) {
      const int rb = (int)(it / p.KI);
      const long long seg_hi = min(it_end, (long long)(rb + 1) * p.KI);
      const int buf = seg % LY::NBUF;
      const uint32_t use_par = (uint32_t)((seg / LY::NBUF) & 1);
      const uint32_t tacc = tmem + buf * LY::ACC_COLS;
      if (!mbar_wait(&acc_empty[buf], use_par ^ 1, p.err, kDevErrMmaWait)) {
        ok = false;
        break;
      }
      tc_fence_after();
      bool first = true;
      for (; it < seg_hi; ++it) {
        if (!mbar_wait(&full[stage], phase, p.err, kDevErrFullWait) ||
            !mbar_wait(&fullx[xstage], xphase, p.err, kDevErrFullWait)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t sb = smem_u32(smem + stage * LY::W_BYTES);
          const uint64_t da = umma_desc_sw128(sb);
          const uint64_t db = umma_desc_sw128(smem_u32(xring + xstage * LY::X_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint32_t acc = (first && kk == 0) ? 0u : 1u;
            umma_bf16(tacc, da + 2 * kk, db + 2 * kk, idesc, acc);
            if (SWIGLU) umma_bf16(tacc + NMMA, umma_desc_sw128(sb + WBOX) + 2 * kk, db + 2 * kk, idesc, acc);
          }
          umma_commit(&empty[stage]);
          umma_commit(&emptyx[xstage]);
        }
        __syncwarp();
        first = false;
        if (++stage == SW) {
          stage = 0;
          phase ^= 1;
        }
        if (++xstage == SX) {
          xstage = 0;
          xphase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&acc_full[buf]);
      __syncwarp();
      ++seg;
    }
    // Free TMEM only after the epilogue warps have read their last accumulator.
    mbar_wait(done, 0, p.err, kDevErrMmaWait);
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(LY::TMEM_COLS));
    return;
  }

  // --------------------------------- epilogue ---------------------------------
  const int et = threadIdx.x - EPI_WARP0 * 32;  // 0..127
  const int q = warp & 3;                       // TMEM lane quarter of this warp
  const int row = 32 * q + lane;                // output feature within the row block
  const uint32_t trow0 = tmem + ((uint32_t)(32 * q) << 16);
  asm volatile("griddepcontrol.wait;" ::: "memory");  // writes only after the previous kernel completed
  int seg = 0;
  long long it = it_begin;
  while (it < it_end) {
    const int buf = seg % LY::NBUF;
    const uint32_t use_par = (uint32_t)((seg / LY::NBUF) & 1);
    const uint32_t trow = trow0 + buf * LY::ACC_COLS;
    ++seg;
    const int rb = (int)(it / p.KI);
    const long long seg_lo = it;
    const long long seg_hi = min(it_end, (long long)(rb + 1) * p.KI);
    it = seg_hi;
    const bool full_rb = (seg_lo == (long long)rb * p.KI) && (seg_hi == (long long)(rb + 1) * p.KI);
    // The four epilogue warps leave together on a time-out (they meet at named
    // barriers in the staged-output path).
    if (!mbar_wait_group(&acc_full[buf], use_par, p.err, kDevErrMmaWait, epi_abort)) break;
    tc_fence_after();
    if (et == 0) TC_TRACE(3 + 5 * (seg_lo != it_begin));
    const int col = rb * BM + row;

    if (full_rb && p.vec_out) {
      // Peer copies: stage 16 tokens x 128 features, then 16-byte rows.
      for (int c0 = 0; c0 < mcols; c0 += 16) {
        float a[16], u[16];
        load_tokens<NORM>(trow, c0, p.Mp, a);
        if (SWIGLU) load_tokens<NORM>(trow + NMMA, c0, p.Mp, u);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          ostage[i * BM + row] = (col < p.N && c0 + i < p.M) ? compute_out(p, c0 + i, col, a[i], SWIGLU ? u[i] : 0.f,
                                                                           SWIGLU)
                                                             : __float2bfloat16_rn(0.f);
        named_bar_sync(2, EPI_THREADS);
        store_staged(p, ostage, 16, c0, rb * BM, et, EPI_THREADS);
        named_bar_sync(2, EPI_THREADS);  // the tile is rewritten by the next 16 tokens
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      continue;
    }
    if (full_rb) {
      for (int c0 = 0; c0 < mcols; c0 += 16) {
        float a[16], u[16];
        load_tokens<NORM>(trow, c0, p.Mp, a);
        if (SWIGLU) load_tokens<NORM>(trow + NMMA, c0, p.Mp, u);
        if (col < p.N) {
          __nv_bfloat16 o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (c0 + i < p.M) o[i] = store_out(p, c0 + i, col, a[i], SWIGLU ? u[i] : 0.f, SWIGLU);
          if (p.has_ext) {
            for (int i = 0; i < 16 && c0 + i < p.M; ++i) store_ext(p, c0 + i, col, o[i]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
      continue;
    }

    // Partial row block: [matrix][token][row] fp32 — a warp's store of one token
    // is 128 contiguous bytes, and so is the reduction kernel's load.
    const int slot = 2 * cta + (seg_lo == it_begin ? 0 : 1);
    float* sp = p.partials + (size_t)slot * SLOT + row;
    for (int c0 = 0; c0 < mcols; c0 += 16) {
      float a[16];
      load_tokens<NORM>(trow, c0, p.Mp, a);
#pragma unroll
      for (int i = 0; i < 16; ++i) __stcg(sp + (size_t)(c0 + i) * BM, a[i]);
      if (SWIGLU) {
        load_tokens<NORM>(trow + NMMA, c0, p.Mp, a);
#pragma unroll
        for (int i = 0; i < 16; ++i) __stcg(sp + (size_t)NMMA * BM + (size_t)(c0 + i) * BM, a[i]);
      }
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&acc_empty[buf]);  // this buffer may be refilled
    if (et == 0) TC_TRACE(5 + 5 * (seg_lo != it_begin));
  }
  tc_fence_before();
  __syncwarp();
  if (lane == 0) mbar_arrive(done);
  if (et == 0) TC_TRACE(12);
}

// RMSNorm prologue: one CTA per token row m < Mp. rstd[m] = rsqrt(mean(x^2) + eps);
// xs[m] = bf16(x*gamma), xs[Mp + m] = bf16(x*gamma - xs[m]); rows m >= M are zero.
__global__ void __launch_bounds__(256) rms_split_kernel(const __nv_bfloat16* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ gamma, float eps, int K,
                                                        int M, int Mp, __nv_bfloat16* __restrict__ xs,
                                                        float* __restrict__ rstd, PeerWait wait, int* err) {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // let the GEMM start streaming W
  if (wait.counter) {  // x is the output of other GPUs' stage: wait for their signals
    if (threadIdx.x == 0) peer_wait(wait, err);
    __syncthreads();
  }
  const int m = blockIdx.x;
  uint4* hi = reinterpret_cast<uint4*>(xs + (size_t)m * K);
  uint4* lo = reinterpret_cast<uint4*>(xs + (size_t)(Mp + m) * K);
  const int nv = K / 8;
  if (m >= M) {
    for (int i = threadIdx.x; i < nv; i += blockDim.x) hi[i] = lo[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) rstd[m] = 0.f;
    return;
  }
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)m * K);
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  float ss = 0.f;
  for (int i = threadIdx.x; i < nv; i += blockDim.x) {
    const uint4 xv = __ldg(xr + i);
    const uint4 gv = __ldg(gr + i);
    const uint32_t* xw = reinterpret_cast<const uint32_t*>(&xv);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gv);
    uint4 hv, lv;
    uint32_t* hw = reinterpret_cast<uint32_t*>(&hv);
    uint32_t* lw = reinterpret_cast<uint32_t*>(&lv);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&xw[e]));
      const float2 gg = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&gw[e]));
      ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      const float p0 = f.x * gg.x, p1 = f.y * gg.y;
      const __nv_bfloat162 h = __floats2bfloat162_rn(p0, p1);
      const float2 hf = __bfloat1622float2(h);
      hw[e] = *reinterpret_cast<const uint32_t*>(&h);
      lw[e] = pack_bf16x2(p0 - hf.x, p1 - hf.y);
    }
    hi[i] = hv;
    lo[i] = lv;
  }
  __shared__ float red[8];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    rstd[m] = rsqrtf(t / (float)K + eps);
  }
}


// Split row blocks: sum the contributors' fp32 partials (in contributor order,
// deterministic) and apply the epilogue. Grid (row block, 16-token chunk),
// 128 threads = the block's 128 output features; row blocks finished inside
// one CTA of the GEMM were already written and exit here at once. Launched as
// a programmatic dependent of the GEMM: griddepcontrol.wait returns once the
// GEMM grid has completed and its writes are visible.
template <int NMMA, bool SWIGLU>
__global__ void __launch_bounds__(128) tc_reduce_kernel(Params p) {
  // The next kernel may launch now (it waits for this grid before reading).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int rb = blockIdx.x;
  const int c0 = blockIdx.y * 8;
  const long long lo = (long long)rb * p.KI, hi = lo + p.KI;
  int cf = (int)((double)lo * p.G / (double)p.total);
  if (cf > p.G - 1) cf = p.G - 1;
  while (cf > 0 && it_start(p, cf) > lo) --cf;
  while (it_start(p, cf + 1) <= lo) ++cf;
  if (it_start(p, cf) <= lo && it_start(p, cf + 1) >= hi) return;  // whole block inside one CTA
  int cl = cf;
  while (cl + 1 < p.G && it_start(p, cl + 1) < hi) ++cl;  // last contributor
  constexpr int SLOT = slot_floats(NMMA, SWIGLU);
  const int row = threadIdx.x;
  const size_t roff = (size_t)c0 * BM + row;  // token c0, this feature row; next token +BM
  float g[8], u[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) g[i] = u[i] = 0.f;
  // Four contributors per batch: all their loads are in flight before the adds
  // (which stay in contributor order).
  for (int cb = cf; cb <= cl; cb += 4) {
    float tg[4][8], tu[4][8];
    bool use[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int cc = cb + k;
      use[k] = cc <= cl && it_start(p, cc + 1) != it_start(p, cc);
      const int sl = use[k] ? 2 * cc + (it_start(p, cc) >= lo ? 0 : 1) : 0;
      const float* base = p.partials + (size_t)sl * SLOT + roff;
#pragma unroll
      for (int i = 0; i < 8; ++i) tg[k][i] = use[k] ? __ldcg(base + i * BM) : 0.f;
      if (SWIGLU) {
#pragma unroll
        for (int i = 0; i < 8; ++i) tu[k][i] = use[k] ? __ldcg(base + (size_t)NMMA * BM + i * BM) : 0.f;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (!use[k]) continue;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        g[i] += tg[k][i];
        if (SWIGLU) u[i] += tu[k][i];
      }
    }
  }
  const int col = rb * BM + row;
  if (p.vec_out) {
    // Peer copies: stage 8 tokens x 128 features, then one 16-byte row per thread.
    __shared__ __align__(16) __nv_bfloat16 st[8 * BM];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      st[i * BM + row] = (col < p.N && c0 + i < p.M) ? compute_out(p, c0 + i, col, g[i], u[i], SWIGLU)
                                                     : __float2bfloat16_rn(0.f);
    __syncthreads();
    store_staged(p, st, 8, c0, rb * BM, row, BM);
    return;
  }
  if (col >= p.N) return;
  __nv_bfloat16 o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (c0 + i < p.M) o[i] = store_out(p, c0 + i, col, g[i], u[i], SWIGLU);
  if (p.has_ext) {
    for (int i = 0; i < 8 && c0 + i < p.M; ++i) store_ext(p, c0 + i, col, o[i]);
  }
}

template <int NMMA, bool SWIGLU, bool NORM>
static int launch(const CUtensorMap& tmW, const CUtensorMap& tmWu, const CUtensorMap& tmX, const CUtensorMap& tmXa,
                  const Params& p, cudaStream_t stream) {
  using LY = Layout<NMMA, SWIGLU>;
  static_assert(LY::STAGES >= 2, "stage does not fit");
  auto kern = gemm_tc_kernel<NMMA, SWIGLU, NORM>;
  FK_CHECK_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)LY::SMEM));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  {
    cudaLaunchConfig_t g = {};
    g.gridDim = dim3((unsigned)p.G, 1, 1);
    g.blockDim = dim3(NTHREADS, 1, 1);
    g.dynamicSmemBytes = LY::SMEM;
    g.stream = stream;
    g.attrs = attr;
    g.numAttrs = 1;
    FK_CHECK_CUDA(cudaLaunchKernelEx(&g, kern, tmW, tmWu, tmX, tmXa, p));
  }
  // Reduction of split row blocks, as a programmatic dependent launch.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.num_rb, (unsigned)((p.M + 7) / 8), 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, tc_reduce_kernel<NMMA, SWIGLU>, p));
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

// Token tile: the smallest of {32, 64, 128, 256} covering n columns.
static int token_tile(int n) { return n <= 32 ? 32 : n <= 64 ? 64 : n <= 128 ? 128 : 256; }
static int round16(int n) { return (n + 15) / 16 * 16; }

// Largest token tile any launch of a call with M tokens uses (plain or RMSNorm).
static int max_tile(int M) {
  const int plain = token_tile(M < 256 ? M : 256);
  const int mt = M < NORM_TILE ? M : NORM_TILE;
  const int norm = token_tile(2 * round16(mt));
  return plain > norm ? plain : norm;
}

}  // namespace tc

// Workspace: [16 KB header (unused here)][RMSNorm split x: 2*128*K bf16][rstd: 128 fp32][partials].
static size_t tc_xs_bytes(int K) { return ((size_t)2 * tc::NORM_TILE * K * 2 + 255) / 256 * 256; }
static size_t tc_rstd_bytes() { return 512; }

size_t tc_workspace_bytes(int M, int N, int K, bool swiglu) {
  (void)N;
  return kCounterBytes + tc_xs_bytes(K) + tc_rstd_bytes() +
         (size_t)2 * num_sms() * tc::slot_floats(tc::max_tile(M), swiglu) * 4;
}

int tc_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
              const void* residual, void* y, int M, int N, int K, float eps, void* workspace, size_t workspace_bytes,
              cudaStream_t stream, const LinearExtras* ex) {
  FK_CHECK_ARG(x && w && y, "null tensor pointer");
  const bool lora = ex && ex->lora_xa;
  FK_CHECK_ARG(!lora || (!gamma && !w_up), "LoRA is supported on the plain linear only");
  FK_CHECK_ARG(!lora || (ex->lora_b && ex->lora_rank >= 8 && ex->lora_rank % 8 == 0 &&
                         ((uintptr_t)ex->lora_xa & 15) == 0 && ((uintptr_t)ex->lora_b & 15) == 0),
               "LoRA: rank must be a positive multiple of 8 and xA / B 16-byte aligned");
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

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ws + kCounterBytes);
  float* rstd = reinterpret_cast<float*>(ws + kCounterBytes + tc_xs_bytes(K));
  const int num_rb = (N + tc::BM - 1) / tc::BM;
  const int KI_main = (K + tc::BK - 1) / tc::BK;
  const int KI = KI_main + (lora ? (ex->lora_rank + tc::BK - 1) / tc::BK : 0);
  tc::Params p;
  p.KI_main = KI_main;
  p.kv = {};
  if (ex) p.kv = ex->kv;
  p.wait = ex ? ex->wait : PeerWait{};
  const OutPlace out0 = ex ? ex->out : OutPlace{};
  const int ldy = out0.ldy > 0 ? out0.ldy : N, ldr = out0.ldr > 0 ? out0.ldr : N;
  p.partials = reinterpret_cast<float*>(ws + kCounterBytes + tc_xs_bytes(K) + tc_rstd_bytes());
  p.err = err;
  p.N = N;
  p.K = K;
  p.KI = KI;
  p.num_rb = num_rb;
  p.up_row_offset = up_row_offset;
  p.total = (long long)num_rb * KI;
  FK_CHECK_ARG(p.total < (1LL << 31), "problem too large for the iteration table");
  int G = num_sms();
  if (G > tc::kMaxGrid) G = tc::kMaxGrid;
  // At least 8 k blocks per CTA: small GEMMs (the column shards of a
  // tensor-parallel layer) otherwise split each row block over dozens of CTAs
  // and pay more for the partials than for the weights (measured best of 4-32).
  constexpr int kMinIters = 8;
  if (p.total / kMinIters < G) G = p.total >= kMinIters ? (int)(p.total / kMinIters) : 1;
  if ((long long)G > p.total) G = (int)p.total;
  p.G = G;
  for (int c = 0; c <= G; ++c) p.starts[c] = (int)((long long)c * p.total / G);

  CUtensorMap tmW, tmWu;
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
  } else if (lora) {
    const uint64_t bdims[2] = {(uint64_t)ex->lora_rank, (uint64_t)N};
    const uint64_t bstr[1] = {(uint64_t)ex->lora_rank * 2};
    rc = encode_tma(&tmWu, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ex->lora_b), bdims, bstr, wbox,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  } else {
    tmWu = tmW;
  }
  // Token tiles: one launch per tile, in order on the stream (RMSNorm: 128 tokens
  // per tile, each preceded by its split prologue).
  const int tile = norm ? tc::NORM_TILE : 256;
  for (int m0 = 0; m0 < M; m0 += tile) {
    const int mt = M - m0 < tile ? M - m0 : tile;
    const __nv_bfloat16* xt = static_cast<const __nv_bfloat16*>(x) + (size_t)m0 * K;
    CUtensorMap tmX;
    int nmma, xrows;
    const void* xsrc;
    if (norm) {
      const int Mp = tc::round16(mt);
      tc::rms_split_kernel<<<Mp, 256, 0, stream>>>(xt, static_cast<const __nv_bfloat16*>(gamma), eps, K, mt, Mp, xs,
                                                   rstd, p.wait, p.err);
      FK_CHECK_CUDA(cudaGetLastError());
      p.Mp = Mp;
      p.rstd = rstd;
      xrows = 2 * Mp;
      nmma = tc::token_tile(2 * Mp);
      xsrc = xs;
    } else {
      p.Mp = 0;
      p.rstd = nullptr;
      xrows = mt;
      nmma = tc::token_tile(mt);
      xsrc = xt;
    }
    const uint64_t xdims[2] = {(uint64_t)K, (uint64_t)xrows};
    const uint32_t xbox[2] = {64, (uint32_t)nmma};
    rc = encode_tma(&tmX, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(xsrc), xdims, strides, xbox,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    p.M = mt;
    p.y = static_cast<__nv_bfloat16*>(y) + (size_t)m0 * ldy;
    p.residual = residual ? static_cast<const __nv_bfloat16*>(residual) + (size_t)m0 * ldr : nullptr;
    p.out = out0;
    p.out.ldy = ldy;
    p.out.ldr = ldr;
    for (int i = 0; i < out0.npeers; ++i) p.out.peer_y[i] = out0.peer_y[i] + (size_t)m0 * ldy;
    p.has_ext = (out0.npeers > 0 || p.kv.k_cache != nullptr) ? 1 : 0;
    {
      bool al = out0.npeers > 0 && p.kv.k_cache == nullptr && ldy % 8 == 0 && ((uintptr_t)p.y & 15) == 0;
      for (int i = 0; i < out0.npeers; ++i) al = al && ((uintptr_t)p.out.peer_y[i] & 15) == 0;
      p.vec_out = al ? 1 : 0;
    }
    CUtensorMap tmXa = tmX;
    if (lora) {
      const uint64_t adims[2] = {(uint64_t)ex->lora_rank, (uint64_t)mt};
      const uint64_t astr[1] = {(uint64_t)ex->lora_rank * 2};
      rc = encode_tma(&tmXa, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                      const_cast<__nv_bfloat16*>(static_cast<const __nv_bfloat16*>(ex->lora_xa) +
                                                 (size_t)m0 * ex->lora_rank),
                      adims, astr, xbox, CU_TENSOR_MAP_SWIZZLE_128B);
      if (rc) return rc;
    }
    p.kv.m_base = m0;
    if (sw)
      rc = norm ? tc::launch_n<true, true>(nmma, tmW, tmWu, tmX, tmXa, p, stream)
                : tc::launch_n<true, false>(nmma, tmW, tmWu, tmX, tmXa, p, stream);
    else
      rc = norm ? tc::launch_n<false, true>(nmma, tmW, tmWu, tmX, tmXa, p, stream)
                : tc::launch_n<false, false>(nmma, tmW, tmWu, tmX, tmXa, p, stream);
    if (rc) return rc;
  }
  return kOk;
}

}  // namespace fk

#ifdef FK_TC_TRACE
extern "C" int fk_tc_trace_dump(unsigned long long* host, int n) {
  return cudaMemcpyFromSymbol(host, fk::tc::g_tc_trace, sizeof(unsigned long long) * n) == cudaSuccess ? 0 : -3;
}
#endif
