// Peer-memory exchange for Ulysses sequence parallelism over NVLink.
//
// Replaces the two NCCL all-to-alls of DistributedSequenceRank
// (models/adapters/eraserdit/nccl_sequence.py:43-103, collective in
// distributed/communication_op.py:97-137): the prologue stores each head group
// straight into the owning rank's receive buffer and the attention epilogue
// stores each output row into the token owner's return buffer, both through
// CUDA IPC mappings of the peers' buffers (plain st.global over NVLink; no
// multicast).  This file holds the plumbing around those stores:
//   - allocation and IPC handles of the exchanged buffers;
//   - erd_peer_signal: after a phase's stores, a system-scope fence and one
//     release store of the call's epoch into every rank's flag slot for us;
//   - erd_peer_wait: acquire loads of our flags until every rank's epoch has
//     arrived, bounded in time; a timeout sets a status bit and returns, and a
//     negative epoch (a rank whose phase failed) sets another and returns.
#include <cuda_runtime.h>
#include <cstdint>
#include <cstring>

#include "host_common.h"
#include "sm100_ptx.cuh"

namespace erd {
namespace {

constexpr int kMaxPeers = 16;

struct PeerFlags {
  int32_t* slot[kMaxPeers];  // rank p's flag for this rank (peer memory)
};

__global__ void peer_signal_kernel(PeerFlags f, int npeers, int32_t epoch) {
  const int p = threadIdx.x;
  // Every store of this stream's earlier kernels is visible system-wide
  // before any flag is (kernel boundaries order them; the fence orders this
  // thread's view for the release below).
  asm volatile("fence.sc.sys;" ::: "memory");
  if (p < npeers) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f.slot[p]), "r"(epoch) : "memory");
  }
}

__global__ void peer_wait_kernel(const int32_t* flags, int n, int32_t epoch, long long timeout_ns,
                                 int* status) {
  const int i = threadIdx.x;
  if (i < n) {
    const unsigned long long t0 = global_timer_ns();
    while (true) {
      int32_t v;
      asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(flags + i) : "memory");
      if (v == epoch) break;
      if (v == -epoch) {  // that rank's phase failed; it still signalled
        if (status != nullptr) atomicOr(status, kStatusPeerFailed);
        break;
      }
      if (static_cast<long long>(global_timer_ns() - t0) > timeout_ns) {
        if (status != nullptr) atomicOr(status, kStatusTimeoutPeer);
        break;
      }
      __nanosleep(200);
    }
  }
  __syncthreads();
}

}  // namespace
}  // namespace erd

using namespace erd;

extern "C" int erd_peer_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return kErrBadShape;
  if (int rc = check_device_sm100()) return rc;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  return static_cast<int>(cudaMemset(*ptr, 0, bytes));
}

extern "C" int erd_peer_free(void* ptr) { return static_cast<int>(cudaFree(ptr)); }

extern "C" int erd_peer_ipc_handle(void* ptr, void* handle64) {
  if (ptr == nullptr || handle64 == nullptr) return kErrNullPointer;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return static_cast<int>(e);
  static_assert(sizeof(h) == 64, "IPC handle size");
  std::memcpy(handle64, &h, sizeof(h));
  return kErrOk;
}

extern "C" int erd_peer_ipc_open(const void* handle64, void** ptr) {
  if (ptr == nullptr || handle64 == nullptr) return kErrNullPointer;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle64, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

extern "C" int erd_peer_ipc_close(void* ptr) {
  return static_cast<int>(cudaIpcCloseMemHandle(ptr));
}

extern "C" int erd_peer_signal(int32_t* const* peer_slots, int npeers, int32_t epoch,
                               void* stream) {
  if (peer_slots == nullptr) return kErrNullPointer;
  if (npeers <= 0 || npeers > kMaxPeers) return kErrBadShape;
  PeerFlags f;
  for (int p = 0; p < kMaxPeers; ++p) {
    f.slot[p] = p < npeers ? peer_slots[p] : nullptr;
    if (p < npeers && (f.slot[p] == nullptr || (reinterpret_cast<uintptr_t>(f.slot[p]) & 3)))
      return kErrMisaligned;
  }
  peer_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(f, npeers, epoch);
  return static_cast<int>(cudaGetLastError());
}

extern "C" int erd_peer_wait(const int32_t* flags, int n, int32_t epoch, int64_t timeout_ns,
                             int* status, void* stream) {
  if (flags == nullptr) return kErrNullPointer;
  if (n <= 0 || n > kMaxPeers || timeout_ns <= 0) return kErrBadShape;
  peer_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, n, epoch, timeout_ns,
                                                                    status);
  return static_cast<int>(cudaGetLastError());
}
