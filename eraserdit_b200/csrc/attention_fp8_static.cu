// FP8 attention whose workspace is a fixed array in the library's own device
// memory, so that the call allocates nothing.
//
// erd_attn_fwd_fp8 quantises Q, K and V^T into a workspace the caller lends
// it.  Some callers have no device memory to lend at that point: a C or C++
// host that drives the library only through the C ABI and has no caching
// allocator of its own (every cudaMalloc there would synchronise the device
// and stall the other streams), or a serving process that fixed its HBM
// budget when it started and must not grow it per request.  This entry point
// serves them: its workspace is `g_fp8_scratch`, a file-scope __device__ array
// the CUDA module holds for the life of the process.  Inside the call there is
// no cudaMalloc, no cudaFree and no allocating library routine.
//
// Limits and rules:
//   - shapes whose FP8 workspace exceeds ERD_FP8_STATIC_SCRATCH_BYTES (64 MiB)
//     are rejected with kErrTooLarge before anything is enqueued;
//   - the first call on each device looks the array's address up with
//     cudaGetSymbolAddress (with that device current) and keeps it together
//     with the device's current context; make that first call before any
//     stream capture.  A later call under a different context (the primary
//     context was reset and re-created, e.g. after cudaDeviceReset) looks the
//     address up again in that context;
//   - the array is part of the library's CUDA module: each device holds its
//     64 MiB from the moment the module is loaded there until the context
//     ends (at the first kernel launch or symbol lookup of this library with
//     lazy module loading, CUDA's default; at context creation with
//     CUDA_MODULE_LOADING=EAGER), whether or not this entry point is called;
//   - every call on a device uses the same array: calls that can overlap in
//     time (on different streams, or from host threads without ordering
//     between them) race on it;
//   - nothing in the array has to start at zero: each call writes every byte
//     it later reads (partial K sums and V maxima, the scales, the E4M3 tiles
//     with their zero padding) before reading it.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <mutex>

#include "eraserdit_b200.h"
#include "host_common.h"

namespace {

// erd_attn_fwd_fp8 wants a 1024-byte aligned workspace; the array carries the
// slack to round its 256-byte aligned start up to that.
constexpr size_t kWorkspaceAlign = 1024;
constexpr size_t kCapacity = ERD_FP8_STATIC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;
constexpr int64_t kTileBytes = 3 * 128 * 64;  // Q, K and V^T bytes per 128-token tile

std::mutex g_lookup;
void* g_base[kMaxDevices];       // per device: 1024-aligned address inside g_fp8_scratch
CUcontext g_ctx[kMaxDevices];    // the context g_base[device] was looked up in

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// cuCtxGetCurrent through the runtime's driver entry point (the library does
// not link libcuda).
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}

}  // namespace

static __device__ __align__(256) uint8_t g_fp8_scratch[kCapacity + kWorkspaceAlign];

namespace {

int scratch_base(void** base) {
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (device < 0 || device >= kMaxDevices) return erd::kErrUnsupportedDevice;
  CtxGetCurrentFn get_ctx = ctx_get_current();
  if (get_ctx == nullptr) return erd::kErrUnsupportedDevice;
  // No context may be current yet on this host thread (the runtime makes the
  // primary context current lazily); the lookup below then makes it current.
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  std::lock_guard<std::mutex> lock(g_lookup);
  if (g_base[device] == nullptr || ctx == nullptr || g_ctx[device] != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fp8_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr) return erd::kErrUnsupportedDevice;
    const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + kWorkspaceAlign - 1) &
                        ~static_cast<uintptr_t>(kWorkspaceAlign - 1);
    g_base[device] = reinterpret_cast<void*>(a);
    g_ctx[device] = ctx;
  }
  *base = g_base[device];
  return erd::kErrOk;
}

}  // namespace

extern "C" int erd_attn_fwd_fp8_static_scratch(
    const void* q, const void* k, const void* v, int64_t q_token_stride, int64_t q_head_stride,
    int64_t q_batch_stride, int64_t q_seg_stride, int64_t k_token_stride, int64_t k_head_stride,
    int64_t k_batch_stride, int64_t k_seg_stride, int64_t v_token_stride, int64_t v_head_stride,
    int64_t v_batch_stride, int64_t v_seg_stride, int batch, int heads, int seg_len, int nseg,
    const int32_t* seg_lens, int head_dim, float softmax_scale, void* out,
    int64_t o_token_stride, int64_t o_head_stride, int64_t o_batch_stride, int64_t o_seg_stride,
    int* status, void* stream) {
  if (batch <= 0 || heads <= 0 || seg_len <= 0 || nseg <= 0 || nseg > 16)
    return erd::kErrBadShape;
  // Lower bound of the workspace in 64-bit arithmetic first, so that no shape
  // overflows the exact size computation below.
  const int64_t tiles = (static_cast<int64_t>(seg_len) + 127) / 128 * nseg;
  if (static_cast<int64_t>(batch) * heads * tiles * kTileBytes > static_cast<int64_t>(kCapacity))
    return erd::kErrTooLarge;
  const size_t need = erd_attn_fp8_workspace_bytes(batch, heads, seg_len, nseg);
  if (need == 0) return erd::kErrBadShape;
  if (need > kCapacity) return erd::kErrTooLarge;
  void* scratch = nullptr;
  if (int rc = scratch_base(&scratch)) return rc;
  return erd_attn_fwd_fp8(q, k, v, q_token_stride, q_head_stride, q_batch_stride, q_seg_stride,
                          k_token_stride, k_head_stride, k_batch_stride, k_seg_stride,
                          v_token_stride, v_head_stride, v_batch_stride, v_seg_stride, batch,
                          heads, seg_len, nseg, seg_lens, head_dim, softmax_scale, out,
                          o_token_stride, o_head_stride, o_batch_stride, o_seg_stride, scratch,
                          kCapacity, status, stream);
}
