// Host-side helpers shared by the C-ABI entry points: cached per-device
// properties and TMA tensor-map encoding through the driver entry point (so
// the library needs no link-time libcuda and loads on machines without a GPU).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

namespace moe {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int sm_count;
  int major;
  int minor;
};

// Device that is current on the calling thread and its cached properties.
int current_device_info(int* dev, DeviceInfo* info);

// cuTensorMapEncodeTiled with the given swizzle (128-byte by default), zero OOB
// fill, 256B L2 promotion.  strides_bytes has rank-1 entries (dimension 0 is
// contiguous).
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// MOE_B200_GEMM_KERNEL=1 selects the 1-SM kernels even for grids of two or more
// SMs (read once per process); the default is the CTA-pair kernels.
inline bool force_single_sm_kernel() {
  static const bool v = [] {
    const char* e = std::getenv("MOE_B200_GEMM_KERNEL");
    return e != nullptr && std::atoi(e) == 1;
  }();
  return v;
}

}  // namespace moe
