// KV-cache append for the decode step: write the new token's K and V rows of
// every batch row into the padded cache at position cache_seqlens[b].
//
// Counterpart of the cache write in the reference's fused projection DAttn2
// (python/cutedsl_kernels/decoding_attention/attempt2.py:276-286, which stores
// the new rows at [P-M, P)), here for a ragged cache [B, Lmax, Hkv, D] indexed
// by per-row lengths. The new rows are read straight out of the fused QKV
// projection output (row stride and column offsets given), so no repacking
// kernel runs between the QKV GEMM and attention.
#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace kv {

// One CTA per batch row; 16-byte vector copies.
__global__ void __launch_bounds__(128) append_kernel(const __nv_bfloat16* __restrict__ src, long long src_stride,
                                                     int k_col, int v_col, __nv_bfloat16* __restrict__ kc,
                                                     __nv_bfloat16* __restrict__ vc, const int* seqlens_in,
                                                     int* seqlens_out, int Lmax, int row_elems, PeerWait wait,
                                                     int* err) {
  const int b = blockIdx.x;
  if (wait.counter) {  // src is the output of other GPUs' stage: wait for their signals
    if (threadIdx.x == 0) peer_wait(wait, err);
    __syncthreads();
  }
  const int pos = seqlens_in[b];
  __syncthreads();  // every thread has read the length before it may be overwritten in place
  const bool ok = pos >= 0 && pos < Lmax;
  if (ok) {
    const uint4* ks = reinterpret_cast<const uint4*>(src + (size_t)b * src_stride + k_col);
    const uint4* vs = reinterpret_cast<const uint4*>(src + (size_t)b * src_stride + v_col);
    uint4* kd = reinterpret_cast<uint4*>(kc + ((size_t)b * Lmax + pos) * row_elems);
    uint4* vd = reinterpret_cast<uint4*>(vc + ((size_t)b * Lmax + pos) * row_elems);
    for (int i = threadIdx.x; i < row_elems / 8; i += blockDim.x) {
      kd[i] = ks[i];
      vd[i] = vs[i];
    }
  }
  if (threadIdx.x == 0 && seqlens_out) seqlens_out[b] = ok ? pos + 1 : pos;
}

// Paged form: the row of token pos lives in block block_table[b][pos / bs], row pos % bs.
__global__ void __launch_bounds__(128) append_paged_kernel(const __nv_bfloat16* __restrict__ src,
                                                           long long src_stride, int k_col, int v_col,
                                                           __nv_bfloat16* __restrict__ kp, __nv_bfloat16* __restrict__ vp,
                                                           const int* __restrict__ block_table, int max_blocks, int bs,
                                                           const int* seqlens_in, int* seqlens_out, int row_elems) {
  const int b = blockIdx.x;
  const int pos = seqlens_in[b];
  __syncthreads();
  const bool ok = pos >= 0 && pos < max_blocks * bs;
  if (ok) {
    const int blk = block_table[(size_t)b * max_blocks + pos / bs];
    const size_t row = (size_t)blk * bs + pos % bs;
    const uint4* ks = reinterpret_cast<const uint4*>(src + (size_t)b * src_stride + k_col);
    const uint4* vs = reinterpret_cast<const uint4*>(src + (size_t)b * src_stride + v_col);
    uint4* kd = reinterpret_cast<uint4*>(kp + row * row_elems);
    uint4* vd = reinterpret_cast<uint4*>(vp + row * row_elems);
    for (int i = threadIdx.x; i < row_elems / 8; i += blockDim.x) {
      kd[i] = ks[i];
      vd[i] = vs[i];
    }
  }
  if (threadIdx.x == 0 && seqlens_out) seqlens_out[b] = ok ? pos + 1 : pos;
}

}  // namespace kv
}  // namespace fk

using namespace fk;

extern "C" int fk_kv_append_paged(const void* src, long long src_row_stride, int k_col, int v_col, void* k_pool,
                                  void* v_pool, const int32_t* block_table, const int32_t* cache_seqlens,
                                  int32_t* seqlens_out, int batch, int max_blocks_per_seq, int block_size,
                                  int num_heads_kv, int head_dim, void* stream) {
  FK_CHECK_ARG(src && k_pool && v_pool && block_table && cache_seqlens, "null tensor pointer");
  FK_CHECK_ARG(batch >= 1 && max_blocks_per_seq >= 1 && block_size >= 1 && num_heads_kv >= 1 && head_dim >= 8,
               "sizes must be positive");
  const int row = num_heads_kv * head_dim;
  FK_CHECK_ARG(row % 8 == 0 && src_row_stride % 8 == 0 && k_col % 8 == 0 && v_col % 8 == 0,
               "row length, stride and column offsets must be multiples of 8 elements");
  kv::append_paged_kernel<<<batch, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), src_row_stride, k_col, v_col, static_cast<__nv_bfloat16*>(k_pool),
      static_cast<__nv_bfloat16*>(v_pool), block_table, max_blocks_per_seq, block_size, cache_seqlens, seqlens_out,
      row);
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}

static int kv_append_impl(const void* src, long long src_row_stride, int k_col, int v_col, void* k_cache,
                          void* v_cache, const int32_t* cache_seqlens, int32_t* seqlens_out, int batch,
                          int max_seqlen, int num_heads_kv, int head_dim, void* stream, const PeerWait& wait) {
  FK_CHECK_ARG(src && k_cache && v_cache && cache_seqlens, "null tensor pointer");
  FK_CHECK_ARG(batch >= 1 && max_seqlen >= 1 && num_heads_kv >= 1 && head_dim >= 8, "sizes must be positive");
  const int row = num_heads_kv * head_dim;
  FK_CHECK_ARG(row % 8 == 0 && src_row_stride % 8 == 0 && k_col % 8 == 0 && v_col % 8 == 0,
               "row length, stride and column offsets must be multiples of 8 elements");
  FK_CHECK_ARG(((uintptr_t)src & 15) == 0 && ((uintptr_t)k_cache & 15) == 0 && ((uintptr_t)v_cache & 15) == 0,
               "src and caches must be 16-byte aligned");
  int* err = device_error_word();
  if (!err) return fail(kErrCuda, "device error word unavailable");
  kv::append_kernel<<<batch, 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(src), src_row_stride, k_col, v_col, static_cast<__nv_bfloat16*>(k_cache),
      static_cast<__nv_bfloat16*>(v_cache), cache_seqlens, seqlens_out, max_seqlen, row, wait, err);
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}

extern "C" int fk_kv_append(const void* src, long long src_row_stride, int k_col, int v_col, void* k_cache,
                            void* v_cache, const int32_t* cache_seqlens, int32_t* seqlens_out, int batch,
                            int max_seqlen, int num_heads_kv, int head_dim, void* stream) {
  return kv_append_impl(src, src_row_stride, k_col, v_col, k_cache, v_cache, cache_seqlens, seqlens_out, batch,
                        max_seqlen, num_heads_kv, head_dim, stream, PeerWait{});
}

extern "C" int fk_kv_append_wait(const void* src, long long src_row_stride, int k_col, int v_col, void* k_cache,
                                 void* v_cache, const int32_t* cache_seqlens, int32_t* seqlens_out, int batch,
                                 int max_seqlen, int num_heads_kv, int head_dim, const int32_t* wait_counter,
                                 const int32_t* wait_flags, int rank, int nranks, void* stream) {
  FK_CHECK_ARG(wait_counter && wait_flags, "null wait counter / flags");
  FK_CHECK_ARG(nranks >= 1 && nranks <= kMaxPeers + 1 && rank >= 0 && rank < nranks, "bad rank / nranks");
  const PeerWait pw{wait_counter, wait_flags, rank, nranks};
  return kv_append_impl(src, src_row_stride, k_col, v_col, k_cache, v_cache, cache_seqlens, seqlens_out, batch,
                        max_seqlen, num_heads_kv, head_dim, stream, pw);
}

namespace fk {
namespace kv {

// Head-major scatter of a projection output: dst[h][row0 + m][d] = src[m][h*D + d].
__global__ void __launch_bounds__(128) head_scatter_kernel(const __nv_bfloat16* __restrict__ q_src,
                                                           const __nv_bfloat16* __restrict__ k_src,
                                                           const __nv_bfloat16* __restrict__ v_src,
                                                           __nv_bfloat16* __restrict__ q_out,
                                                           __nv_bfloat16* __restrict__ k_cache,
                                                           __nv_bfloat16* __restrict__ v_cache, int M, int H, int D,
                                                           int P) {
  const int m = blockIdx.x, h = blockIdx.y, which = blockIdx.z;
  const __nv_bfloat16* src = which == 0 ? q_src : which == 1 ? k_src : v_src;
  __nv_bfloat16* dst = which == 0 ? q_out + ((size_t)h * M + m) * D
                                  : (which == 1 ? k_cache : v_cache) + ((size_t)h * P + (P - M) + m) * D;
  const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)m * H * D + (size_t)h * D);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (int i = threadIdx.x; i < D / 8; i += blockDim.x) d4[i] = s[i];
}

}  // namespace kv
}  // namespace fk

extern "C" int fk_qkv_head_scatter(const void* q_src, const void* k_src, const void* v_src, void* q_out,
                                   void* k_cache, void* v_cache, int M, int num_heads, int head_dim, int cache_len,
                                   void* stream) {
  FK_CHECK_ARG(q_src && k_src && v_src && q_out && k_cache && v_cache, "null tensor pointer");
  FK_CHECK_ARG(M >= 1 && num_heads >= 1 && head_dim >= 8 && head_dim % 8 == 0, "bad sizes");
  FK_CHECK_ARG(cache_len >= M, "cache_len must be >= M (new rows go to [cache_len - M, cache_len))");
  kv::head_scatter_kernel<<<dim3(M, num_heads, 3), 128, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(q_src), static_cast<const __nv_bfloat16*>(k_src),
      static_cast<const __nv_bfloat16*>(v_src), static_cast<__nv_bfloat16*>(q_out),
      static_cast<__nv_bfloat16*>(k_cache), static_cast<__nv_bfloat16*>(v_cache), M, num_heads, head_dim,
      cache_len);
  FK_CHECK_CUDA(cudaGetLastError());
  return kOk;
}
