// fk_skinny_gemm_noalloc: the skinny (M <= 16) weight-streaming GEMM with its
// stream-K scratch in a fixed, library-owned device array instead of a
// caller-provided workspace.
//
// Who needs it: code that must not allocate GPU memory while it runs, e.g. a
// host process whose allocator is owned by someone else (a serving runtime
// that pre-plans every byte, an embedding application with its own pool), or
// a caller that cannot reach an allocator at all (plain C through the ABI,
// no torch). Such callers still allocate x, w and y themselves; only the
// split-partial scratch moves here.
//
// The array below is loaded once per GPU with the library and lives until the
// process exits (about 2.7 MB per device). In host code its name is only a
// host-side stand-in, so the entry point looks up its device address with
// cudaGetSymbolAddress on the first call on each device (with that device
// current) and passes that pointer to the kernel. Do that first call before
// any stream capture on the device.
//
// Every call shares the one array, which keeps the previous call's contents:
// each call clears the row-block counters it uses (cudaMemsetAsync on the
// caller's stream, no allocation) before the kernel. Calls that can overlap on
// the GPU (different streams without ordering between them) race on the
// array and give wrong results: order them on one stream.
#include <mutex>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
int skinny_linear(const void* x, const void* gamma, const void* w, const void* w_up, int up_row_offset,
                  const void* residual, void* y, int M, int N, int K, float eps, void* workspace,
                  size_t workspace_bytes, int grid_override, cudaStream_t stream,
                  const LinearExtras* ex = nullptr);
size_t skinny_workspace_bytes(int N, int G, bool swiglu);
}  // namespace fk

namespace {

// Largest persistent grid the array holds partials for (148 SMs on B200).
constexpr int kNoAllocMaxCtas = 160;
// Counter header (4096 row blocks) + two fp32 partial slots of 128 x 16 (+16) per CTA.
constexpr size_t kNoAllocBytes = fk::kCounterBytes + (size_t)2 * kNoAllocMaxCtas * (128 * 16 + 16) * 4;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_address(void** out) {
  int dev = 0;
  FK_CHECK_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fk::fail(fk::kErrUnsupported, "device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return fk::cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return fk::kOk;
}

}  // namespace

extern "C" int fk_skinny_gemm_noalloc(const void* x, const void* w, void* y, int M, int N, int K,
                                      void* stream) {
  FK_CHECK_ARG(M >= 1 && M <= 16, "fk_skinny_gemm_noalloc takes 1 <= M <= 16");
  FK_CHECK_ARG(N >= 1 && (N + 127) / 128 <= fk::kMaxRowBlocks,
               "fk_skinny_gemm_noalloc takes 1 <= N <= 524288");
  int G = fk::num_sms();
  if (G > kNoAllocMaxCtas) G = kNoAllocMaxCtas;
  if (fk::skinny_workspace_bytes(N, G, false) > kNoAllocBytes)
    return fk::fail(fk::kErrInvalidArgument, "problem needs more scratch than the static array holds");
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t counter_bytes = (size_t)((N + 127) / 128) * sizeof(int);
  FK_CHECK_CUDA(cudaMemsetAsync(scratch, 0, counter_bytes, st));
  return fk::skinny_linear(x, nullptr, w, nullptr, 0, nullptr, y, M, N, K, 0.f, scratch, kNoAllocBytes, G, st);
}
