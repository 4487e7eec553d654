// C-ABI entry points of the linear (GEMM) family and their M-based dispatch:
// M <= 16 -> the stream-K weight-streaming kernel (skinny_gemm.cu),
// M  > 16 -> the tcgen05/TMEM kernel (gemm_tc.cu).
#include "common.cuh"
#include "fk_b200.h"

namespace fk {
size_t skinny_workspace_bytes(int N, int G, bool swiglu);
int skinny_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                  const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
                  size_t workspace_bytes, int grid_override, cudaStream_t stream);
size_t tc_workspace_bytes(int M, int N, int K, bool swiglu);
int tc_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
              const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
              size_t workspace_bytes, cudaStream_t stream);
}  // namespace fk

using namespace fk;

static int dispatch(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                    const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
                    size_t workspace_bytes, void* stream) {
  FK_CHECK_ARG(M >= 1, "M must be >= 1");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (M <= 16)
    return skinny_linear(x, gamma, w, w_up, up_row_offset, residual, y, M, N, K, eps, workspace,
                         workspace_bytes, 0, st);
  return tc_linear(x, gamma, w, w_up, up_row_offset, residual, y, M, N, K, eps, workspace, workspace_bytes, st);
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

}  // extern "C"
