// Shared device/host helpers for the sm_100a kernels of this library.
//
// Everything here is hand-written inline PTX over documented instructions
// (mbarrier, cp.async.bulk.tensor, ldmatrix, mma.sync, tcgen05) plus the
// host-side C-ABI error plumbing. Every spin-wait is bounded: when a wait runs
// out, the waiting thread records an error code in the library's device error
// word (passed to every kernel as `int* err`) and the kernel returns, so a
// broken pipeline never hangs the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace fk {

// ---------------------------------------------------------------------------
// Error plumbing (host)
// ---------------------------------------------------------------------------
enum Status : int {
  kOk = 0,
  kErrInvalidArgument = -1,  // bad shape / dtype / alignment (Python: ValueError)
  kErrUnsupported = -2,      // a shape outside what the kernels implement
  kErrCuda = -3,             // a CUDA runtime / driver call failed
  kErrDevice = -4,           // a device-side bounded wait ran out
};

void set_last_error(const std::string& msg);
int fail(int code, const std::string& msg);
int cuda_fail(cudaError_t e, const char* what);

#define FK_CHECK_ARG(cond, msg)                                        \
  do {                                                                 \
    if (!(cond)) return ::fk::fail(::fk::kErrInvalidArgument, (msg)); \
  } while (0)
#define FK_CHECK_CUDA(expr)                                \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return ::fk::cuda_fail(_e, #expr); \
  } while (0)

// Number of SMs of the current device (cached per device id).
int num_sms();
// Encode a tiled TMA descriptor through the driver entry point (no -lcuda).
int encode_tma(CUtensorMap* map, CUtensorMapDataType dtype, int rank,
               void* gaddr, const uint64_t* dims, const uint64_t* strides_bytes,
               const uint32_t* box, CUtensorMapSwizzle swizzle,
               CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B);

// Stream-K workspace header: a fixed block of per-row-block counters at the
// start of every linear-family workspace, whatever the call's shape, so that
// fp32 partials of one call can never land on the counters of another call
// sharing the workspace. Supports up to kMaxRowBlocks row blocks (N <= 512K).
constexpr int kMaxRowBlocks = 4096;
constexpr size_t kCounterBytes = kMaxRowBlocks * sizeof(int);  // 16 KB

// Device address of this library's error word on the current device (set up
// once per device). Kernels take it as `int* err`.
int* device_error_word();

// ---------------------------------------------------------------------------
// Device-side error codes (bounded waits report here)
// ---------------------------------------------------------------------------
enum DeviceError : int {
  kDevErrNone = 0,
  kDevErrFullWait = 1,    // consumer waited too long for a TMA stage
  kDevErrEmptyWait = 2,   // producer waited too long for a free stage
  kDevErrMmaWait = 3,     // waited too long for a tensor-core commit
  kDevErrFlagWait = 4,    // waited too long on a global flag
};

// Bound on any single wait, in nanoseconds of %globaltimer: far above any
// legitimate wait inside these kernels (microseconds), far below a watchdog.
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

// The device error block is four ints: [0] the error code, [1] spare,
// [2..3] a uint64 wait bound in ns set from the host (0: kWaitLimitNs). Tests
// shorten the bound to make a withheld pipeline stage time out quickly.
__device__ __forceinline__ uint64_t wait_limit_ns(const int* err) {
  const uint64_t v = *reinterpret_cast<const volatile unsigned long long*>(err + 2);
  return v ? v : kWaitLimitNs;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_device_error(int* err, int code) {
  atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity to complete.
// Returns false (and records `err`) when the bound runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  const uint64_t lim = wait_limit_ns(err);
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - t0 > lim) break;
  }
  record_device_error(err, code);
  return false;
}

// Bounded wait for a group of warps that must leave together: besides its own
// time bound, the wait gives up as soon as any warp of the group has set the
// shared abort flag, and a warp whose bound runs out sets it. Every warp of the
// group therefore stops waiting within one bound of the first time-out, so
// the group still meets at its next named barrier instead of hanging there.
// Warp-uniform: call with all lanes of a warp.
__device__ __forceinline__ bool mbar_wait_group(uint64_t* bar, uint32_t parity, int* err, int code,
                                                volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  const uint64_t lim = wait_limit_ns(err);
  bool ok = false;
  while (true) {
    if (mbar_try_wait(bar, parity)) {
      ok = true;
      break;
    }
    if (*abort_flag) break;
    if (global_timer_ns() - t0 > lim) {
      record_device_error(err, code);
      *abort_flag = 1;
      break;
    }
  }
  // Lanes may leave on different iterations; agree on one answer per warp.
  return __all_sync(0xffffffffu, ok);
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), no multicast anywhere in this library.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)),
      "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// ---------------------------------------------------------------------------
// Warp-level tensor-core helpers (ldmatrix + mma.sync m16n8k16 bf16)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1,
                                          uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(addr));
}
// D += A(16x16, row) * B(16x8, col), bf16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Named barrier among `nthreads` threads (id 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// 128B-swizzle address of the 16-byte chunk `chunk` (0..7) of row `row` in a
// tile whose rows are 128 bytes and whose base is 1024-byte aligned: the TMA
// SWIZZLE_128B pattern XORs the chunk index with the row index modulo 8.
__device__ __forceinline__ uint32_t swz128(uint32_t base, int row, int chunk) {
  return base + row * 128 + (((chunk ^ row) & 7) << 4);
}

// ---- optional epilogue / operand extensions of the linear family -------------

// KV-cache append fused into a projection's epilogue: output columns
// [k_col, k_col + width) of token m are also written to row seqlens_in[m] of the
// K cache, [v_col, v_col + width) to the V cache, and seqlens_next[m] receives
// the advanced length (out of place: the lengths are read by every CTA).
// Contiguous cache [M, cap, width] when block_table is null, else a block pool
// [*, block_size, width] addressed through block_table[m, pos / block_size].
struct KvAppend {
  __nv_bfloat16* k_cache;  // null: no append
  __nv_bfloat16* v_cache;
  const int* seqlens_in;
  int* seqlens_next;       // may be null
  const int* block_table;
  int k_col, v_col, width, cap, max_blocks, block_size;
  int m_base;              // token index of the launch's first row (token-tiled launches)
};

__device__ __forceinline__ void kv_append_store(const KvAppend& a, int m_local, int col, __nv_bfloat16 v) {
  if (a.k_cache == nullptr) return;
  const int m = a.m_base + m_local;
  __nv_bfloat16* base;
  int rel;
  if (col >= a.k_col && col < a.k_col + a.width) {
    base = a.k_cache;
    rel = col - a.k_col;
  } else if (col >= a.v_col && col < a.v_col + a.width) {
    base = a.v_cache;
    rel = col - a.v_col;
  } else {
    return;
  }
  const int pos = __ldg(a.seqlens_in + m);
  const bool ok = pos >= 0 && pos < a.cap;
  if (base == a.k_cache && rel == 0 && a.seqlens_next) a.seqlens_next[m] = ok ? pos + 1 : pos;
  if (!ok) return;
  const size_t row = a.block_table
                         ? (size_t)__ldg(a.block_table + (size_t)m * a.max_blocks + pos / a.block_size) *
                                   a.block_size + pos % a.block_size
                         : (size_t)m * a.cap + pos;
  base[row * a.width + rel] = v;
}

// Output placement of a linear call: y and residual rows `ldy` / `ldr` elements
// apart (0: N, dense), and up to kMaxPeers more copies of y written with plain
// stores into other GPUs' memory (CUDA IPC mappings of their buffers) at the same
// offsets: the GEMM's epilogue performs the all-gather of a column-parallel layer.
constexpr int kMaxPeers = 7;
struct OutPlace {
  int ldy, ldr;
  int npeers;
  __nv_bfloat16* peer_y[kMaxPeers];
};

__device__ __forceinline__ void store_out_all(const OutPlace& o, __nv_bfloat16* y, size_t off, __nv_bfloat16 v) {
  y[off] = v;
#pragma unroll
  for (int i = 0; i < kMaxPeers; ++i)  // constant indices: the pointers stay in the parameter bank
    if (i < o.npeers) o.peer_y[i][off] = v;
}

// The wait half of a cross-GPU stage barrier, done by the kernel that consumes
// the stage (fk_peer_signal did the other half): seq = *counter (advanced by
// the signal kernel, which completed before this kernel passed
// griddepcontrol.wait), then until flags[r] >= seq for every peer r. One
// thread, bounded; counter null: no wait.
struct PeerWait {
  const int* counter;
  const int* flags;
  int rank, nranks;
};

__device__ __forceinline__ void peer_wait(const PeerWait& w, int* err) {
  if (w.counter == nullptr) return;
  const int seq = *reinterpret_cast<const volatile int*>(w.counter);
  const uint64_t t0 = global_timer_ns();
  const uint64_t lim = wait_limit_ns(err);
  for (int r = 0; r < w.nranks; ++r) {
    if (r == w.rank) continue;
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(w.flags + r) : "memory");
      if (v - seq >= 0) break;
      if (global_timer_ns() - t0 > lim) {
        record_device_error(err, kDevErrFlagWait);
        return;
      }
    }
  }
}

// Extensions a linear call may carry besides its main operands.
struct LinearExtras {
  KvAppend kv;                 // kv.k_cache null: none
  const void* lora_xa;         // [M, rank] bf16: x . A^T (null: no LoRA)
  const void* lora_b;          // [N, rank] bf16
  int lora_rank;               // multiple of 8
  OutPlace out;                // ldy = ldr = 0, npeers = 0: dense local output
  PeerWait wait;               // counter null: no cross-GPU wait before reading x
};

}  // namespace fk
