// Host-side helpers shared by the C-ABI entry points: return codes, argument
// checks, device capability probe and the driver's tensor-map encoder.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace erd {

// C-ABI return codes.  0 is success, positive values are cudaError_t values
// from the launch, negative values are argument errors detected on the host
// before anything is enqueued.
enum : int {
  kErrOk = 0,
  kErrNullPointer = -1,
  kErrBadShape = -2,
  kErrMisaligned = -3,
  kErrUnsupportedDevice = -4,
  kErrTensorMap = -5,
  kErrTooLarge = -6,
};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// True when the current device is a compute capability 10.0 part (B200).
int check_device_sm100();

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda
// link dependency).  Returns kErrOk or kErrTensorMap.
int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle);

}  // namespace erd
