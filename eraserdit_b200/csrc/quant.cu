// Static-scale E4M3 quantisation of BF16 activations for the FP8 QKV projection.
//
// Replaces the activation quantiser of SharedQKV (layers/quantization/qkv_fp8.py:52-55,
// kernel _quant_fp8_tensor in layers/quantization/eraserdit_fp8.py:60-69):
// q = E4M3_RN(clamp(x / s, -448, 448)) with an IEEE division by the static
// scale s.  Memory-bound: 16 BF16 per thread per step, 128-bit loads, 128-bit stores.
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "host_common.h"

namespace erd {
namespace {

__device__ __forceinline__ uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ float q_in(uint32_t bits_half, float scale) {
  const float x = __uint_as_float(bits_half);
  return fminf(448.f, fmaxf(-448.f, __fdiv_rn(x, scale)));
}

__global__ void __launch_bounds__(256) quantize_e4m3_kernel(const uint4* __restrict__ x,
                                                            uint4* __restrict__ out,
                                                            long long n16, float scale) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n16;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const uint4 a = __ldg(x + 2 * i), b = __ldg(x + 2 * i + 1);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t u0 = w[2 * j], u1 = w[2 * j + 1];
      const uint32_t lo = e4m3x2(q_in(u0 << 16, scale), q_in(u0 & 0xFFFF0000u, scale));
      const uint32_t hi = e4m3x2(q_in(u1 << 16, scale), q_in(u1 & 0xFFFF0000u, scale));
      o[j] = lo | (hi << 16);
    }
    out[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

}  // namespace
}  // namespace erd

using namespace erd;

extern "C" int erd_quantize_e4m3(const void* x, void* out, int64_t n, float scale, void* stream) {
  if (x == nullptr || out == nullptr) return kErrNullPointer;
  if (n < 0 || (n & 15) || !(scale > 0.f)) return kErrBadShape;
  if (!aligned16(x) || !aligned16(out)) return kErrMisaligned;
  if (n == 0) return kErrOk;
  if (int rc = check_device_sm100()) return rc;
  const long long n16 = n / 16;
  const long long blocks = (n16 + 255) / 256;
  const unsigned grid = static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16);
  quantize_e4m3_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(x), static_cast<uint4*>(out), n16, scale);
  return static_cast<int>(cudaGetLastError());
}
