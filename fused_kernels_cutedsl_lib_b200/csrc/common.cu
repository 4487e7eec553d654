// Host-side plumbing shared by every entry point: the thread-local last-error
// message, the device error word, SM counts and TMA descriptor encoding.
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {

static thread_local std::string t_last_error;

void set_last_error(const std::string& msg) { t_last_error = msg; }

int fail(int code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  t_last_error = std::string(what) + ": " + cudaGetErrorString(e);
  return kErrCuda;
}

// One error block per device: the module-scope variable below has one instance
// on every device that loads this library. [0] is the error word kernels write;
// [2..3] hold the wait bound in ns (0: the built-in 1 s), see wait_limit_ns.
__device__ __align__(16) int g_fk_device_error[4] = {0, 0, 0, 0};

static constexpr int kMaxDevices = 64;

int* device_error_word() {
  static std::mutex mu;
  static int* ptrs[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_fk_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

int num_sms() {
  static std::mutex mu;
  static int counts[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lock(mu);
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode_tma(CUtensorMap* map, CUtensorMapDataType dtype, int rank, void* gaddr,
               const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
               CUtensorMapSwizzle swizzle, CUtensorMapL2promotion promo) {
  auto fn = get_encode_fn();
  if (!fn) return fail(kErrCuda, "cuTensorMapEncodeTiled entry point unavailable");
  cuuint64_t gdim[5], gstride[4];
  cuuint32_t bdim[5], estride[5];
  for (int i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = strides_bytes[i];
  CUresult r = fn(map, dtype, rank, gaddr, gdim, gstride, bdim, estride,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(kErrCuda, "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return kOk;
}

}  // namespace fk

extern "C" {

const char* fk_last_error(void) { return fk::t_last_error.c_str(); }

int fk_version(void) { return FK_B200_ABI_VERSION; }

int fk_get_device_error(int* code_out, int clear) {
  if (!code_out) return fk::fail(fk::kErrInvalidArgument, "code_out is null");
  int* w = fk::device_error_word();
  if (!w) return fk::fail(fk::kErrCuda, "device error word unavailable");
  int v = 0;
  FK_CHECK_CUDA(cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost));
  if (clear && v != 0) {
    int z = 0;
    FK_CHECK_CUDA(cudaMemcpy(w, &z, sizeof(int), cudaMemcpyHostToDevice));
  }
  *code_out = v;
  return fk::kOk;
}

int fk_set_wait_limit_ns(unsigned long long ns) {
  int* w = fk::device_error_word();
  if (!w) return fk::fail(fk::kErrCuda, "device error word unavailable");
  FK_CHECK_CUDA(cudaMemcpy(w + 2, &ns, sizeof(ns), cudaMemcpyHostToDevice));
  return fk::kOk;
}

int fk_num_sms(void) { return fk::num_sms(); }

int fk_use_device(int device) {
  FK_CHECK_CUDA(cudaSetDevice(device));
  return fk::kOk;
}

}  // extern "C"
