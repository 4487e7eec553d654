// C-ABI entry points of the linear (GEMM) family and their M-based dispatch:
// M <= 16 -> the stream-K weight-streaming kernel (skinny_gemm.cu),
// M  > 16 -> the tcgen05/TMEM kernel (gemm_tc.cu).
#include "common.cuh"
#include "fk_b200.h"

namespace fk {
size_t skinny_workspace_bytes(int N, int G, bool swiglu);
int skinny_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                  const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
                  size_t workspace_bytes, int grid_override, cudaStream_t stream,
                  const LinearExtras* ex = nullptr);
size_t tc_workspace_bytes(int M, int N, int K, bool swiglu);
int tc_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
              const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
              size_t workspace_bytes, cudaStream_t stream, const LinearExtras* ex = nullptr);
}  // namespace fk

using namespace fk;

static int dispatch(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                    const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
                    size_t workspace_bytes, void* stream, const LinearExtras* ex = nullptr) {
  FK_CHECK_ARG(M >= 1, "M must be >= 1");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M <= 16)
    return skinny_linear(x, gamma, w, w_up, up_row_offset, residual, y, M, N, K, eps, workspace,
                         workspace_bytes, 0, st, ex);
  return tc_linear(x, gamma, w, w_up, up_row_offset, residual, y, M, N, K, eps, workspace, workspace_bytes, st,
                   ex);
}

extern "C" {

int fk_linear_workspace_bytes(int M, int N, int K, int flags, size_t* bytes_out) {
  FK_CHECK_ARG(bytes_out != nullptr, "bytes_out is null");
  FK_CHECK_ARG(M >= 1 && N >= 1 && K >= 1, "sizes must be positive");
  const bool sw = (flags & FK_LINEAR_SWIGLU) != 0;
  if (M <= 16)
    *bytes_out = skinny_workspace_bytes(N, num_sms(), sw);
  else
    *bytes_out = tc_workspace_bytes(M, N, K, sw);
  return kOk;
}

int fk_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
              const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
              size_t workspace_bytes, void* stream) {
  return dispatch(x, gamma, w, w_up, up_row_offset, residual, y, M, N, K, eps, workspace, workspace_bytes,
                  stream);
}

int fk_skinny_gemm(const void* x, const void* w, void* y, int M, int N, int K, void* workspace,
                   size_t workspace_bytes, void* stream) {
  return dispatch(x, nullptr, w, nullptr, 0, nullptr, y, M, N, K, 0.f, workspace, workspace_bytes, stream);
}

int fk_rmsnorm_linear(const void* x, const void* gamma, const void* w, void* y, int M, int N, int K,
                      float eps, void* workspace, size_t workspace_bytes, void* stream) {
  FK_CHECK_ARG(gamma != nullptr, "gamma is null");
  return dispatch(x, gamma, w, nullptr, 0, nullptr, y, M, N, K, eps, workspace, workspace_bytes, stream);
}

int fk_swiglu_gemm(const void* x, const void* w_gate_up, void* y, int M, int N, int K, void* workspace,
                   size_t workspace_bytes, void* stream) {
  FK_CHECK_ARG(w_gate_up != nullptr, "w_gate_up is null");
  return dispatch(x, nullptr, w_gate_up, w_gate_up, N, nullptr, y, M, N, K, 0.f, workspace, workspace_bytes,
                  stream);
}

int fk_swiglu_gemm2(const void* x, const void* w_gate, const void* w_up, void* y, int M, int N, int K,
                    void* workspace, size_t workspace_bytes, void* stream) {
  FK_CHECK_ARG(w_gate != nullptr && w_up != nullptr, "null weight");
  return dispatch(x, nullptr, w_gate, w_up, 0, nullptr, y, M, N, K, 0.f, workspace, workspace_bytes, stream);
}

int fk_rmsnorm_swiglu(const void* x, const void* gamma, const void* w_gate_up, void* y, int M, int N, int K,
                      float eps, void* workspace, size_t workspace_bytes, void* stream) {
  FK_CHECK_ARG(gamma != nullptr && w_gate_up != nullptr, "null tensor pointer");
  return dispatch(x, gamma, w_gate_up, w_gate_up, N, nullptr, y, M, N, K, eps, workspace, workspace_bytes,
                  stream);
}

// LoRA linear: y = x . W^T + xA . B^T (+ residual), xA = x . A^T given [M, rank].
// The LoRA product runs as extra k blocks of the same GEMM ([x | xA] . [W | B]^T),
// accumulated in fp32 with the main product before the single bf16 rounding.
int fk_lora_linear(const void* x, const void* w, const void* lora_xa, const void* lora_b, const void* residual,
                   void* y, int M, int N, int K, int rank, void* workspace, size_t workspace_bytes, void* stream) {
  FK_CHECK_ARG(lora_xa != nullptr && lora_b != nullptr, "lora_xa / lora_b is null");
  LinearExtras ex = {};
  ex.lora_xa = lora_xa;
  ex.lora_b = lora_b;
  ex.lora_rank = rank;
  return dispatch(x, nullptr, w, nullptr, 0, residual, y, M, N, K, 0.f, workspace, workspace_bytes, stream, &ex);
}

// Projection with the KV-cache append in its epilogue (gamma null: plain linear).
int fk_linear_kv_append(const void* x, const void* gamma, const void* w, void* y, int M, int N, int K, float eps,
                        void* k_cache, void* v_cache, const int32_t* block_table, const int32_t* cache_seqlens,
                        int32_t* seqlens_next, int k_col, int v_col, int num_heads_kv, int head_dim,
                        int max_seqlen, int block_size, void* workspace, size_t workspace_bytes, void* stream) {
  FK_CHECK_ARG(k_cache && v_cache && cache_seqlens, "null cache / length pointer");
  FK_CHECK_ARG(num_heads_kv >= 1 && head_dim >= 1 && max_seqlen >= 1, "sizes must be positive");
  const long long width = (long long)num_heads_kv * head_dim;
  FK_CHECK_ARG(k_col >= 0 && v_col >= 0 && k_col + width <= N && v_col + width <= N,
               "K / V column ranges must lie inside the N output columns");
  FK_CHECK_ARG(k_col + width <= v_col || v_col + width <= k_col, "K and V column ranges overlap");
  FK_CHECK_ARG(seqlens_next != (int32_t*)cache_seqlens,
               "seqlens_next must not alias cache_seqlens (every CTA reads the lengths)");
  FK_CHECK_ARG(!block_table || (block_size >= 1 && max_seqlen % block_size == 0),
               "paged cache: max_seqlen must be max_blocks_per_seq * block_size");
  LinearExtras ex = {};
  ex.kv.k_cache = static_cast<__nv_bfloat16*>(k_cache);
  ex.kv.v_cache = static_cast<__nv_bfloat16*>(v_cache);
  ex.kv.seqlens_in = cache_seqlens;
  ex.kv.seqlens_next = seqlens_next;
  ex.kv.block_table = block_table;
  ex.kv.k_col = k_col;
  ex.kv.v_col = v_col;
  ex.kv.width = (int)width;
  ex.kv.cap = max_seqlen;
  ex.kv.block_size = block_table ? block_size : max_seqlen;
  ex.kv.max_blocks = block_table ? max_seqlen / block_size : 1;
  return dispatch(x, gamma, w, nullptr, 0, nullptr, y, M, N, K, eps, workspace, workspace_bytes, stream, &ex);
}

// General linear with output placement: y rows ldy apart (>= N), residual rows
// ldr apart, and npeers more copies of y in other GPUs' memory (IPC mappings).
static int linear_ex_impl(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                          const void* residual, int ldr, void* y, int ldy, void* const* peer_y, int npeers, int M,
                          int N, int K, float eps, void* workspace, size_t workspace_bytes, void* stream,
                          const PeerWait& wait) {
  FK_CHECK_ARG(npeers >= 0 && npeers <= kMaxPeers, "npeers must be in [0, 7]");
  FK_CHECK_ARG(ldy == 0 || ldy >= N, "ldy must be 0 (dense) or >= N");
  FK_CHECK_ARG(ldr == 0 || ldr >= N, "ldr must be 0 (dense) or >= N");
  LinearExtras ex = {};
  ex.out.ldy = ldy;
  ex.out.ldr = ldr;
  ex.out.npeers = npeers;
  for (int i = 0; i < npeers; ++i) {
    FK_CHECK_ARG(peer_y && peer_y[i], "null peer output pointer");
    ex.out.peer_y[i] = static_cast<__nv_bfloat16*>(peer_y[i]);
  }
  ex.wait = wait;
  return dispatch(x, gamma, w, w_up, up_row_offset, residual, y, M, N, K, eps, workspace, workspace_bytes, stream,
                  &ex);
}

int fk_linear_ex(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                 const void* residual, int ldr, void* y, int ldy, void* const* peer_y, int npeers, int M, int N,
                 int K, float eps, void* workspace, size_t workspace_bytes, void* stream) {
  return linear_ex_impl(x, gamma, w, w_up, up_row_offset, residual, ldr, y, ldy, peer_y, npeers, M, N, K, eps,
                        workspace, workspace_bytes, stream, PeerWait{});
}

int fk_linear_ex_wait(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                      const void* residual, int ldr, void* y, int ldy, void* const* peer_y, int npeers, int M, int N,
                      int K, float eps, void* workspace, size_t workspace_bytes, const int32_t* wait_counter,
                      const int32_t* wait_flags, int rank, int nranks, void* stream) {
  FK_CHECK_ARG(wait_counter && wait_flags, "null wait counter / flags");
  FK_CHECK_ARG(nranks >= 1 && nranks <= kMaxPeers + 1 && rank >= 0 && rank < nranks, "bad rank / nranks");
  const PeerWait pw{wait_counter, wait_flags, rank, nranks};
  return linear_ex_impl(x, gamma, w, w_up, up_row_offset, residual, ldr, y, ldy, peer_y, npeers, M, N, K, eps,
                        workspace, workspace_bytes, stream, pw);
}

}  // extern "C"
