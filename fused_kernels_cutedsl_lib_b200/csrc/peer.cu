// Peer memory for the tensor-parallel decode step: buffers shared between the
// GPUs of one node through CUDA IPC, and a cross-GPU stage barrier.
//
// A column-parallel GEMM of the layer writes its output block into the full
// activation buffer of every rank directly from its epilogue (OutPlace peers,
// plain stores over NVLink); the barrier then orders "every rank's block has
// landed" before the next stage reads the buffer. It replaces the all-gather
// (plus the [P, B, n/P] -> [B, n] re-layout copy) of an NCCL-based layer.
//
// Barrier protocol (one thread, after griddepcontrol.wait: the kernel is a
// programmatic dependent of the producer): seq = ++counter (a per-rank device counter, so
// CUDA-graph replays advance it); system-scope fence, so the stores of the
// preceding kernels on this stream - including their stores into peer memory -
// are ordered before the flag; store seq into flags[rank] of every peer; wait
// until every peer's flag in the local array has reached seq. Flags only grow,
// so a peer already one barrier ahead also satisfies the wait. The wait is
// bounded (1 s): on timeout the device error word is set and the kernel
// returns, leaving the context usable.
#include <cstring>

#include "common.cuh"
#include "fk_b200.h"

namespace fk {
namespace peer {

constexpr int kMaxRanks = kMaxPeers + 1;

struct BarrierArgs {
  int* counter;                 // local [1]
  int* local_flags;             // local [P]: written by the peers
  int* peer_flags[kMaxRanks];   // peer r's flags array (index rank is ours); entry `rank` unused
  int rank, nranks;
  int wait;                     // 0: signal only (the next kernel waits, see PeerWait)
  int* err;
};

__global__ void barrier_kernel(BarrierArgs a) {
  // Launched as a programmatic dependent: let the next kernel launch (a GEMM
  // starts streaming its weights; it waits for this grid before reading x),
  // then wait for the producing kernels on this stream to complete.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x != 0) return;
  const int seq = *a.counter + 1;
  *a.counter = seq;
  // One release fence at system scope orders every earlier write of this
  // stream (the stage's peer stores included) before the flag stores below,
  // which are then plain relaxed stores: the fence + relaxed store pattern is a
  // release, without a full sequentially consistent fence per peer.
  asm volatile("fence.acq_rel.sys;" ::: "memory");
#pragma unroll
  for (int r = 0; r < kMaxRanks; ++r) {
    if (r >= a.nranks || r == a.rank) continue;
    asm volatile("st.relaxed.sys.global.b32 [%0], %1;" ::"l"(a.peer_flags[r] + a.rank), "r"(seq) : "memory");
  }
  if (!a.wait) return;
  const uint64_t t0 = global_timer_ns();
  const uint64_t lim = wait_limit_ns(a.err);
  for (int r = 0; r < a.nranks; ++r) {
    if (r == a.rank) continue;
    while (true) {
      int v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(a.local_flags + r) : "memory");
      if (v - seq >= 0) break;
      if (global_timer_ns() - t0 > lim) {
        record_device_error(a.err, kDevErrFlagWait);
        return;
      }
    }
  }
  // The acquire loads above order this thread after every peer's release; the
  // next kernel on the stream starts after this grid completes.
}

}  // namespace peer
}  // namespace fk

using namespace fk;

extern "C" {

int fk_peer_alloc(size_t bytes, void** ptr_out) {
  FK_CHECK_ARG(ptr_out != nullptr && bytes > 0, "bad arguments");
  void* p = nullptr;
  FK_CHECK_CUDA(cudaMalloc(&p, bytes));
  FK_CHECK_CUDA(cudaMemset(p, 0, bytes));
  FK_CHECK_CUDA(cudaDeviceSynchronize());
  *ptr_out = p;
  return kOk;
}

int fk_peer_free(void* ptr) {
  if (ptr) FK_CHECK_CUDA(cudaFree(ptr));
  return kOk;
}

int fk_ipc_handle_bytes(void) { return (int)sizeof(cudaIpcMemHandle_t); }

int fk_ipc_get_handle(void* ptr, void* handle_out) {
  FK_CHECK_ARG(ptr && handle_out, "null pointer");
  cudaIpcMemHandle_t h;
  FK_CHECK_CUDA(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle_out, &h, sizeof(h));
  return kOk;
}

int fk_ipc_open(const void* handle, void** ptr_out) {
  FK_CHECK_ARG(handle && ptr_out, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  FK_CHECK_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr_out = p;
  return kOk;
}

int fk_ipc_close(void* ptr) {
  if (ptr) FK_CHECK_CUDA(cudaIpcCloseMemHandle(ptr));
  return kOk;
}

static int barrier_impl(int32_t* counter, int32_t* local_flags, int32_t* const* peer_flags, int rank, int nranks,
                        void* stream, int wait) {
  FK_CHECK_ARG(counter && (local_flags || !wait) && peer_flags, "null pointer");
  FK_CHECK_ARG(nranks >= 1 && nranks <= peer::kMaxRanks && rank >= 0 && rank < nranks, "bad rank / nranks");
  int* err = device_error_word();
  if (!err) return fail(kErrCuda, "device error word unavailable");
  peer::BarrierArgs a = {};
  a.counter = counter;
  a.local_flags = local_flags;
  for (int r = 0; r < nranks; ++r) {
    FK_CHECK_ARG(r == rank || peer_flags[r], "null peer flags pointer");
    a.peer_flags[r] = peer_flags[r];
  }
  a.rank = rank;
  a.nranks = nranks;
  a.wait = wait;
  a.err = err;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(32, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FK_CHECK_CUDA(cudaLaunchKernelEx(&cfg, peer::barrier_kernel, a));
  return kOk;
}

int fk_peer_barrier(int32_t* counter, int32_t* local_flags, int32_t* const* peer_flags, int rank, int nranks,
                    void* stream) {
  return barrier_impl(counter, local_flags, peer_flags, rank, nranks, stream, 1);
}

int fk_peer_signal(int32_t* counter, int32_t* const* peer_flags, int rank, int nranks, void* stream) {
  return barrier_impl(counter, nullptr, peer_flags, rank, nranks, stream, 0);
}

}  // extern "C"
