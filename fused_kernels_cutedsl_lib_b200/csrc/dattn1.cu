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
// One CTA per head, 8 warps. Warp w takes token tiles w, w+8, ... of 16
// tokens: S (16 queries x 16 tokens) = Q K^T with mma.sync m16n8k16, the
// fp32 accumulators are rounded to bf16 and reused in registers as the A
// operand of O (16 x 128) += S V^T. The eight warps' O partials are summed
// through shared memory in a fixed order.
#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace da1 {

constexpr int D = 128;
constexpr int MQ = 16;
constexpr int WARPS = 8;
constexpr int KROW = D + 8;   // K / Q tile row, bf16 (272 B: conflict-free ldmatrix)
constexpr int VROW = 16 + 8;  // V tile row: 16 tokens + pad (48 B)
constexpr int KTILE = 16 * KROW;
constexpr int VTILE = D * VROW;
constexpr int WARP_ELEMS = KTILE + VTILE;

__global__ void __launch_bounds__(WARPS * 32) dattn1_kernel(const __nv_bfloat16* __restrict__ Q,
                                                            const __nv_bfloat16* __restrict__ K,
                                                            const __nv_bfloat16* __restrict__ V,
                                                            __nv_bfloat16* __restrict__ O, int M, int P) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  __nv_bfloat16* sq = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [16][KROW]
  __nv_bfloat16* swarp = sq + MQ * KROW;                            // per warp: K tile, V tile
  const int h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3, j = lane >> 3, r = lane & 7;
  const __nv_bfloat16* qh = Q + (size_t)h * M * D;
  const __nv_bfloat16* kh = K + (size_t)h * P * D;
  const __nv_bfloat16* vh = V + (size_t)h * D * P;

  // Q (rows >= M are zero) into shared memory, then A fragments for the 8 k-steps.
  for (int i = threadIdx.x; i < MQ * D / 8; i += blockDim.x) {
    const int row = i / (D / 8), col = (i % (D / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < M) v = *reinterpret_cast<const uint4*>(qh + (size_t)row * D + col);
    *reinterpret_cast<uint4*>(sq + row * KROW + col) = v;
  }
  __syncthreads();
  uint32_t qa[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int row = (j & 1) * 8 + r, col = 16 * ks + (j >> 1) * 8;
    ldsm_x4(smem_u32(sq + row * KROW + col), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
  }

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  __nv_bfloat16* sk = swarp + warp * WARP_ELEMS;
  __nv_bfloat16* sv = sk + KTILE;
  const int ntiles = (P + 15) / 16;

  for (int t = warp; t < ntiles; t += WARPS) {
    const int p0 = t * 16;
    // K tile: 16 token rows x 128 dims; V tile: 128 dim rows x 16 tokens. Past P: zeros.
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int i = lane + 32 * m;  // 0..255
      const int kr = i >> 4, kc = (i & 15) * 8;
      uint4 kv = make_uint4(0, 0, 0, 0);
      if (p0 + kr < P) kv = __ldg(reinterpret_cast<const uint4*>(kh + (size_t)(p0 + kr) * D + kc));
      *reinterpret_cast<uint4*>(sk + kr * KROW + kc) = kv;
      const int vd = i >> 1, vhalf = (i & 1) * 8;
      uint4 vv = make_uint4(0, 0, 0, 0);
      if (p0 + vhalf < P) vv = __ldg(reinterpret_cast<const uint4*>(vh + (size_t)vd * P + p0 + vhalf));
      *reinterpret_cast<uint4*>(sv + vd * VROW + vhalf) = vv;
    }
    __syncwarp();
    // S = Q K^T for 16 tokens (two n8 tiles)
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      uint32_t b[4];
      const int tok = (j >> 1) * 8 + r, col = 16 * ks + (j & 1) * 8;
      ldsm_x4(smem_u32(sk + tok * KROW + col), b[0], b[1], b[2], b[3]);
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
      const int d = 16 * pr + (j >> 1) * 8 + r, col = (j & 1) * 8;
      ldsm_x4(smem_u32(sv + d * VROW + col), b[0], b[1], b[2], b[3]);
      mma_bf16_16816(o[2 * pr], pa, b[0], b[1]);
      mma_bf16_16816(o[2 * pr + 1], pa, b[2], b[3]);
    }
    __syncwarp();
  }

  // Sum the warps' O in a fixed order: warps 4-7 add into 0-3, then 4 partials summed.
  __syncthreads();
  float* red = reinterpret_cast<float*>(swarp);  // [4][16][128] fp32 = 32 KB (reuses the tiles)
  auto put = [&](float* dst, bool add) {
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int col = nt * 8 + 2 * c;
      float* r0 = dst + g * D + col;
      float* r1 = dst + (g + 8) * D + col;
      if (add) {
        r0[0] += o[nt][0]; r0[1] += o[nt][1]; r1[0] += o[nt][2]; r1[1] += o[nt][3];
      } else {
        r0[0] = o[nt][0]; r0[1] = o[nt][1]; r1[0] = o[nt][2]; r1[1] = o[nt][3];
      }
    }
  };
  if (warp < 4) put(red + warp * MQ * D, false);
  __syncthreads();
  if (warp >= 4) put(red + (warp - 4) * MQ * D, true);
  __syncthreads();
  for (int i = threadIdx.x; i < M * D; i += blockDim.x) {
    const float v = red[i] + red[MQ * D + i] + red[2 * MQ * D + i] + red[3 * MQ * D + i];
    O[(size_t)h * M * D + i] = __float2bfloat16_rn(v);
  }
}

constexpr size_t kSmem = (size_t)(MQ * KROW + WARPS * WARP_ELEMS) * 2;
static_assert(kSmem >= 4 * MQ * D * 4 + MQ * KROW * 2, "reduction buffer must fit in the tile region");

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
  FK_CHECK_CUDA(cudaFuncSetAttribute(da1::dattn1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)da1::kSmem));
  da1::dattn1_kernel<<<num_heads, da1::WARPS * 32, da1::kSmem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k),
      static_cast<const __nv_bfloat16*>(v_t), static_cast<__nv_bfloat16*>(out), seq_q, seqlen_kv);
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}
