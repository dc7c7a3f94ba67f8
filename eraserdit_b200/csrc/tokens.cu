// Token gather for the block-sparse attention's tile order.
//
// dst[b][t][:] = src[b][index[t]][:], rows of BF16.  One 256-thread block per
// (token, batch) row moves the row in 16-byte words; the copy is HBM-bound
// (one read and one write of every row).
#include <cuda_runtime.h>
#include <cstdint>

#include "host_common.h"

namespace erd {
namespace {

__global__ void __launch_bounds__(256) gather_tokens_kernel(
    const uint4* __restrict__ src, long long src_ts, long long src_bs, int src_tokens,
    uint4* __restrict__ dst, long long dst_ts, long long dst_bs, const int* __restrict__ index,
    int words) {
  const int t = blockIdx.x;
  const int b = blockIdx.y;
  const int from = __ldg(index + t);
  if (from < 0 || from >= src_tokens) return;  // out-of-range index: row left as is
  const uint4* s = src + b * src_bs + from * src_ts;
  uint4* d = dst + b * dst_bs + static_cast<long long>(t) * dst_ts;
  for (int i = threadIdx.x; i < words; i += blockDim.x) d[i] = __ldg(s + i);
}

}  // namespace
}  // namespace erd

using namespace erd;

extern "C" int erd_gather_tokens(const void* src, int64_t src_token_stride,
                                 int64_t src_batch_stride, int src_tokens, void* dst,
                                 int64_t dst_token_stride, int64_t dst_batch_stride,
                                 const int32_t* index, int batch, int tokens, int row_elems,
                                 void* stream) {
  if (src == nullptr || dst == nullptr || index == nullptr) return kErrNullPointer;
  if (batch < 0 || tokens < 0 || src_tokens <= 0 || row_elems <= 0 || (row_elems & 7) ||
      batch > 65535)
    return kErrBadShape;
  if (!aligned16(src) || !aligned16(dst) ||
      ((src_token_stride | src_batch_stride | dst_token_stride | dst_batch_stride) & 7) ||
      src_token_stride < 0 || src_batch_stride < 0 || dst_token_stride < 0 || dst_batch_stride < 0)
    return kErrMisaligned;
  if (batch == 0 || tokens == 0) return kErrOk;
  if (int rc = check_device_sm100()) return rc;
  // strides and row length in 16-byte words
  gather_tokens_kernel<<<dim3(static_cast<unsigned>(tokens), static_cast<unsigned>(batch)), 256, 0,
                         static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), src_token_stride / 8, src_batch_stride / 8, src_tokens,
      static_cast<uint4*>(dst), dst_token_stride / 8, dst_batch_stride / 8, index, row_elems / 8);
  return static_cast<int>(cudaGetLastError());
}
