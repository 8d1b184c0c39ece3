// Allocation-free entry point for the atomic-queue grouped GEMM.
//
// The dynamic tile queue of moe_grouped_gemm needs one 32-bit counter in device
// memory beyond the call's inputs and outputs.  The regular entry point takes it
// from the caller (work_counter), which assumes the caller can allocate device
// memory.  Some callers cannot: code that runs inside a host framework whose
// memory pool owns the GPU's memory and forbids raw cudaMalloc/cudaFree next to
// it, and latency-critical serving loops where cudaMalloc/cudaFree may
// synchronise the whole device.  For them this file keeps the counter in a
// fixed, file-scope device array that lives as long as the library is loaded on
// each GPU, so a call allocates nothing.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "../../include/moe_overlap.h"
#include "host_common.h"

namespace moe {
namespace {

// The whole scratch area of the allocation-free entry point: 64 words (256
// bytes), of which word 0 is the tile counter; the rest is reserved.
constexpr int kNoAllocScratchWords = 64;
static __device__ __align__(256) int32_t g_gemm_noalloc_scratch[kNoAllocScratchWords];

struct NoAllocSlot {
  std::mutex mu;
  int32_t* dev_ptr = nullptr;  // set only once a lookup has succeeded
};
NoAllocSlot g_noalloc[kMaxDevices];

// Device address of the scratch array on the current device.  In host code the
// array's name is only a host-side stand-in, so the real address has to be
// looked up once per device, with that device current.  A failed lookup (for
// instance one attempted during stream capture) is not remembered: the next
// call on that device tries again, and the CUDA error it left is cleared so
// that it is not reported later against an unrelated operation.
int noalloc_scratch(int32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return MOE_ERR_UNSUPPORTED;
  NoAllocSlot& s = g_noalloc[dev];
  std::lock_guard<std::mutex> lock(s.mu);
  if (s.dev_ptr == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_gemm_noalloc_scratch) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return MOE_ERR_CUDA;
    }
    s.dev_ptr = static_cast<int32_t*>(p);
  }
  *out = s.dev_ptr;
  return MOE_OK;
}

}  // namespace
}  // namespace moe

extern "C" int32_t moe_grouped_gemm_noalloc(const void* a, int64_t lda, const void* b,
                                            int64_t b_stride_e, int64_t b_stride_k,
                                            int64_t b_stride_n, void* c, int64_t ldc,
                                            const void* expert_offsets, int32_t offsets_int64,
                                            int64_t m_total, int64_t k, int64_t n,
                                            int32_t num_experts, int32_t dtype,
                                            int32_t activation, int32_t num_sms,
                                            int32_t* status, void* stream) {
  // The 32-bit tile counter ends at (number of tiles + grid size).  Bound the
  // tile count from above (every expert adds at most one partial 128-row tile)
  // and refuse problems whose count could overflow it.
  if (m_total < 0 || n < 0 || num_experts < 0) return MOE_ERR_INVALID_ARG;
  const int64_t row_tiles_max = (m_total + 127) / 128 + num_experts;
  const int64_t col_tiles = (n + 255) / 256;
  if (col_tiles > 0 && row_tiles_max > (int64_t(INT32_MAX) - 4096) / col_tiles)
    return MOE_ERR_CAPACITY;
  int32_t* counter = nullptr;
  if (int rc = moe::noalloc_scratch(&counter); rc != MOE_OK) return rc;
  // moe_grouped_gemm zeroes the counter on `stream` before its launch, so every
  // call starts from a clean queue whatever the previous call left behind.
  return moe_grouped_gemm(a, lda, b, b_stride_e, b_stride_k, b_stride_n, c, ldc, expert_offsets,
                          offsets_int64, m_total, k, n, num_experts, dtype, activation, num_sms,
                          /*use_atomic_queue=*/1, counter, status, stream);
}
