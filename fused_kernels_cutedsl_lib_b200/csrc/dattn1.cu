// Reference-semantics decode attention: O[h] = (Q[h] K[h]^T) V[h]^T with the
// score matrix rounded to bf16 and no softmax, V given transposed [H, D, P].
//
// This is the computation of the reference's DAttn1 kernel
// (python/cutedsl_kernels/decoding_attention/attn1.py:204-251: P = K Q^T,
// cast to bf16, O^T += V^T P^T; check demo/dec_attn_second_part.py:33-34), kept
// so that callers of DAttn1 get identical results; the softmax decode path is
// dec_attn.cu. The reference ignores its softmax_scale argument and so does
// this kernel. Unlike the reference it handles any head count (its persistent
// grid skips heads beyond 132) and any P that is a multiple of 8 (it drops the
// tail past a multiple of 128).
//
// One CTA per head, two CTAs per SM. A TMA producer warp streams 64-token
// tiles of K (two 128B-swizzled boxes of 64 dims) and of V^T (one box of
// 128 dims x 64 tokens) through a 3-stage mbarrier ring; tokens past P are
// zero-filled by TMA, so they add nothing. Four consumer warps each own 16
// tokens of a tile: S (16 queries x 16 tokens) = Q K^T with mma.sync m16n8k16,
// the fp32 scores are rounded to bf16 and reused in registers as the A operand
// of O (16 x 128) += S V^T. The four warps' O partials are summed through
// shared memory in a fixed order. Every wait is bounded; a consumer warp whose
// wait runs out makes all four leave together.
#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace da1 {

constexpr int D = 128;
constexpr int MQ = 16;
constexpr int T = 64;                        // tokens per tile
constexpr int NCW = 4;                       // consumer warps, 16 tokens each
constexpr int NTHREADS = (NCW + 1) * 32;     // + the TMA producer warp
constexpr int STAGES = 3;
constexpr int KHALF = T * 128;               // 64 tokens x 64 dims x 2 B
constexpr int KBYTES = 2 * KHALF;            // K tile: 16 KB
constexpr int VBYTES = D * T * 2;            // V^T tile (128 dims x 64 tokens): 16 KB
constexpr int STAGE_BYTES = KBYTES + VBYTES; // 32 KB
constexpr int QROW = D + 8;                  // Q rows in shared memory (272 B: conflict-free ldmatrix)
constexpr size_t kSmem = 1024 + (size_t)STAGES * STAGE_BYTES + (size_t)MQ * QROW * 2 + 2 * STAGES * 8 + 16;
static_assert((size_t)NCW * MQ * D * 4 <= (size_t)STAGES * STAGE_BYTES, "reduction buffer must fit in the ring");

__global__ void __launch_bounds__(NTHREADS, 2)
    dattn1_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                  const __nv_bfloat16* __restrict__ Q, __nv_bfloat16* __restrict__ O, int M, int P, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(ring + STAGES * STAGE_BYTES);  // [16][QROW]
  uint64_t* full = reinterpret_cast<uint64_t*>(sq + MQ * QROW);
  uint64_t* empty = full + STAGES;
  volatile int* s_abort = reinterpret_cast<volatile int*>(empty + STAGES);
  const int h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (P + T - 1) / T;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NCW);
    }
    *s_abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == NCW) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const uint64_t pol = l2_policy_evict_first();
      int stage = 0;
      uint32_t phase = 0;
      for (int t = 0; t < ntiles; ++t) {
        if (!mbar_wait(&empty[stage], phase ^ 1, err, kDevErrEmptyWait)) return;
        mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
        uint8_t* kd = ring + stage * STAGE_BYTES;
        tma_load_3d(kd, &tmK, &full[stage], 0, t * T, h, pol);
        tma_load_3d(kd + KHALF, &tmK, &full[stage], 64, t * T, h, pol);
        tma_load_3d(kd + KBYTES, &tmV, &full[stage], t * T, 0, h, pol);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int g = lane >> 2, c = lane & 3, j = lane >> 3, r = lane & 7;
  const int tid = threadIdx.x;  // 0..127
  const __nv_bfloat16* qh = Q + (size_t)h * M * D;
  // Q (rows >= M are zero) into shared memory, then A fragments for the 8 k-steps.
  for (int i = tid; i < MQ * D / 8; i += NCW * 32) {
    const int row = i / (D / 8), col = (i % (D / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < M) v = __ldg(reinterpret_cast<const uint4*>(qh + (size_t)row * D + col));
    *reinterpret_cast<uint4*>(sq + row * QROW + col) = v;
  }
  named_bar_sync(1, NCW * 32);
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int row = (j & 1) * 8 + r, col = 16 * ks + (j >> 1) * 8;
    ldsm_x4(smem_u32(sq + row * QROW + col), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  const int tw = 16 * warp;  // this warp's first token inside a tile
  int stage = 0;
  uint32_t phase = 0;
  for (int t = 0; t < ntiles; ++t) {
    if (!mbar_wait_group(&full[stage], phase, err, kDevErrFullWait, s_abort)) break;
    const uint32_t kb = smem_u32(ring + stage * STAGE_BYTES);
    const uint32_t vb = kb + KBYTES;
    // S = Q K^T for this warp's 16 tokens (two n8 tiles)
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b[4];
      ldsm_x4(swz128(kb + (ks >> 2) * KHALF, tw + (j >> 1) * 8 + r, 2 * (ks & 3) + (j & 1)), b[0], b[1], b[2],
              b[3]);
      mma_bf16_16816(s0, qa[ks], b[0], b[1]);
      mma_bf16_16816(s1, qa[ks], b[2], b[3]);
    }
    // bf16 S as the A operand (queries x tokens) of O += S V^T
    uint32_t pa[4];
    pa[0] = pack_bf16x2(s0[0], s0[1]);
    pa[1] = pack_bf16x2(s0[2], s0[3]);
    pa[2] = pack_bf16x2(s1[0], s1[1]);
    pa[3] = pack_bf16x2(s1[2], s1[3]);
#pragma unroll
    for (int pr = 0; pr < 8; ++pr) {
      uint32_t b[4];
      ldsm_x4(swz128(vb, 16 * pr + (j >> 1) * 8 + r, 2 * warp + (j & 1)), b[0], b[1], b[2], b[3]);
      mma_bf16_16816(o[2 * pr], pa, b[0], b[1]);
      mma_bf16_16816(o[2 * pr + 1], pa, b[2], b[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[stage]);
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1;
    }
  }
  named_bar_sync(1, NCW * 32);
  if (*s_abort) return;  // uniform: written only inside the loop above

  // Every tile was consumed, so the ring is free: sum the warps' O in a fixed
  // order (warp 0 + warp 1 + warp 2 + warp 3) through it.
  float* red = reinterpret_cast<float*>(ring);  // [4][16][128] fp32 = 32 KB
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int col = nt * 8 + 2 * c;
    float* r0 = red + (warp * MQ + g) * D + col;
    float* r1 = red + (warp * MQ + g + 8) * D + col;
    r0[0] = o[nt][0];
    r0[1] = o[nt][1];
    r1[0] = o[nt][2];
    r1[1] = o[nt][3];
  }
  named_bar_sync(1, NCW * 32);
  for (int i = tid; i < M * D; i += NCW * 32) {
    const float v = ((red[i] + red[MQ * D + i]) + red[2 * MQ * D + i]) + red[3 * MQ * D + i];
    O[(size_t)h * M * D + i] = __float2bfloat16_rn(v);
  }
}

}  // namespace da1
}  // namespace fk

using namespace fk;

extern "C" int fk_dattn1(const void* q, const void* k, const void* v_t, void* out, int num_heads, int seq_q,
                         int seqlen_kv, int head_dim, void* stream) {
  FK_CHECK_ARG(q && k && v_t && out, "null tensor pointer");
  FK_CHECK_ARG(num_heads >= 1 && seqlen_kv >= 1, "sizes must be positive");
  FK_CHECK_ARG(head_dim == da1::D, "head_dim must be 128");
  FK_CHECK_ARG(seq_q >= 1 && seq_q <= da1::MQ, "seq_q (query rows per head) must be in [1, 16]");
  FK_CHECK_ARG(seqlen_kv % 8 == 0, "seqlen_kv must be a multiple of 8");
  FK_CHECK_ARG(((uintptr_t)q & 15) == 0 && ((uintptr_t)k & 15) == 0 && ((uintptr_t)v_t & 15) == 0,
               "tensors must be 16-byte aligned");
  int* err = device_error_word();
  if (!err) return fail(kErrCuda, "device error word unavailable");
  const uint64_t P = (uint64_t)seqlen_kv, H = (uint64_t)num_heads;
  // K [H, P, 128] as (dim, token, head); V^T [H, 128, P] as (token, dim, head).
  CUtensorMap tmK, tmV;
  {
    const uint64_t dims[3] = {(uint64_t)da1::D, P, H};
    const uint64_t strides[2] = {(uint64_t)da1::D * 2, P * da1::D * 2};
    const uint32_t box[3] = {64, (uint32_t)da1::T, 1};
    int rc = encode_tma(&tmK, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(k), dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {P, (uint64_t)da1::D, H};
    const uint64_t strides[2] = {P * 2, (uint64_t)da1::D * P * 2};
    const uint32_t box[3] = {(uint32_t)da1::T, (uint32_t)da1::D, 1};
    int rc = encode_tma(&tmV, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(v_t), dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  FK_CHECK_CUDA(cudaFuncSetAttribute(da1::dattn1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)da1::kSmem));
  da1::dattn1_kernel<<<num_heads, da1::NTHREADS, da1::kSmem, static_cast<cudaStream_t>(stream)>>>(
      tmK, tmV, static_cast<const __nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(out), seq_q, seqlen_kv, err);
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}
