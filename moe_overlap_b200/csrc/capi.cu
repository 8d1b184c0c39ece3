// C-ABI plumbing: status strings, per-device property cache, TMA tensor-map
// encoding, expert_offsets and the tile-list inspection entry point.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "../../include/moe_overlap.h"
#include "host_common.h"
#include "ptx.cuh"
#include "sched.cuh"

namespace moe {

namespace {
struct DevCache {
  std::once_flag once;
  DeviceInfo info{};
  int rc = MOE_OK;
};
DevCache g_dev[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
}  // namespace

int current_device_info(int* dev, DeviceInfo* info) {
  if (cudaGetDevice(dev) != cudaSuccess) return MOE_ERR_CUDA;
  if (*dev < 0 || *dev >= kMaxDevices) return MOE_ERR_UNSUPPORTED;
  DevCache& dc = g_dev[*dev];
  std::call_once(dc.once, [&] {
    int sm = 0, major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, *dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, *dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, *dev) != cudaSuccess) {
      dc.rc = MOE_ERR_CUDA;
      return;
    }
    dc.info = DeviceInfo{sm, major, minor};
  });
  *info = dc.info;
  return dc.rc;
}

int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, int rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (g_encode == nullptr) return MOE_ERR_UNSUPPORTED;
  cuuint64_t d[5];
  cuuint64_t s[4];
  cuuint32_t b[5];
  cuuint32_t es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    es[i] = 1;
    if (i + 1 < rank) s[i] = strides_bytes[i];
  }
  const CUresult r = g_encode(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d,
                              s, b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MOE_OK : MOE_ERR_INVALID_ARG;
}

namespace {

// Counts enter as int32 values (an int64 count is first narrowed to int32, as
// the reference's .to(torch.int32) does); the running sum is 64-bit.
__host__ __device__ inline long long load_count(const void* counts, int is64, int i) {
  return is64 ? static_cast<long long>(static_cast<int>(
                    static_cast<unsigned long long>(static_cast<const long long*>(counts)[i])))
              : static_cast<long long>(static_cast<const int*>(counts)[i]);
}

// One warp: 64-bit running sum over the counts, chunked per lane.
__global__ void expert_offsets_kernel(const void* counts, int counts_int64, int num_experts,
                                      void* offsets, int offsets_int64) {
  const int lane = threadIdx.x;
  const int per = (num_experts + 31) / 32;
  const int beg = min(num_experts, lane * per);
  const int end = min(num_experts, beg + per);
  long long local = 0;
  for (int e = beg; e < end; ++e) local += load_count(counts, counts_int64, e);
  long long incl = local;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const long long v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  long long run = incl - local;
  auto store = [&](int i, long long v) {
    if (offsets_int64)
      static_cast<long long*>(offsets)[i] = v;
    else
      static_cast<int*>(offsets)[i] = static_cast<int>(static_cast<unsigned long long>(v));
  };
  if (lane == 0) store(0, 0);
  for (int e = beg; e < end; ++e) {
    run += load_count(counts, counts_int64, e);
    store(e + 1, run);
  }
}

__global__ void tile_list_kernel(const void* offsets, int is64, int num_experts, long long m_total,
                                 int block_m, int tiles_n, int order, int* out_e, int* out_m,
                                 int* out_n, int max_items, int* out_count, int32_t* status) {
  extern __shared__ int sh[];
  int* prefix = sh;
  int* seg_start = prefix + num_experts + 1;
  int* seg_rows = seg_start + num_experts + 1;
  if (threadIdx.x < 32)
    build_tile_prefix(offsets, is64, num_experts, m_total, block_m, tiles_n, prefix, seg_start,
                      seg_rows, status);
  __syncthreads();
  const int total = prefix[num_experts];
  if (threadIdx.x == 0) *out_count = total;
  for (int t = threadIdx.x; t < total && t < max_items; t += blockDim.x) {
    const TileCoord c =
        decode_tile(t, num_experts, prefix, seg_start, seg_rows, block_m, tiles_n, order);
    out_e[t] = c.expert;
    out_m[t] = c.tile_m;
    out_n[t] = c.tile_n;
  }
}

}  // namespace
}  // namespace moe

using namespace moe;

extern "C" const char* moe_status_string(int32_t code) {
  switch (code) {
    case MOE_OK: return "ok";
    case MOE_ERR_INVALID_ARG: return "invalid argument (shape, dtype, pointer, stride or alignment)";
    case MOE_ERR_CUDA: return "CUDA call failed";
    case MOE_ERR_TIMEOUT: return "bounded device-side wait expired";
    case MOE_ERR_OFFSETS: return "expert_offsets outside [0, m_total]";
    case MOE_ERR_UNSUPPORTED: return "unsupported device or configuration";
    case MOE_ERR_CAPACITY: return "capacity of a fixed-size buffer exceeded";
    default: return "unknown status";
  }
}

extern "C" int32_t moe_abi_version(void) { return MOE_ABI_VERSION; }

extern "C" int32_t moe_expert_offsets(const void* counts, int32_t counts_int64,
                                      int32_t num_experts, void* offsets, int32_t offsets_int64,
                                      void* stream) {
  if (num_experts < 0 || offsets == nullptr || (num_experts > 0 && counts == nullptr))
    return MOE_ERR_INVALID_ARG;
  expert_offsets_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      counts, counts_int64, num_experts, offsets, offsets_int64);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int32_t moe_expert_offsets_host(const void* counts, int32_t counts_int64,
                                           int32_t num_experts, void* offsets,
                                           int32_t offsets_int64) {
  if (num_experts < 0 || offsets == nullptr || (num_experts > 0 && counts == nullptr))
    return MOE_ERR_INVALID_ARG;
  long long run = 0;
  for (int e = 0; e <= num_experts; ++e) {
    if (e > 0) run += load_count(counts, counts_int64, e - 1);
    if (offsets_int64)
      static_cast<long long*>(offsets)[e] = run;
    else
      static_cast<int*>(offsets)[e] = static_cast<int>(static_cast<unsigned long long>(run));
  }
  return MOE_OK;
}

extern "C" int32_t moe_tile_list(const void* expert_offsets, int32_t offsets_int64,
                                 int32_t num_experts, int64_t m_total, int64_t n, int32_t block_m,
                                 int32_t block_n, int32_t order, int32_t* out_expert,
                                 int32_t* out_tile_m, int32_t* out_tile_n, int32_t max_items,
                                 int32_t* out_count, int32_t* status, void* stream) {
  if (expert_offsets == nullptr || num_experts < 0 || num_experts > 1024 || block_m <= 0 ||
      block_n <= 0 || n < 0 || m_total < 0 || max_items < 0 || out_count == nullptr ||
      (order != 0 && order != 1))
    return MOE_ERR_INVALID_ARG;
  if (max_items > 0 && (out_expert == nullptr || out_tile_m == nullptr || out_tile_n == nullptr))
    return MOE_ERR_INVALID_ARG;
  const int64_t tiles_n = (n + block_n - 1) / block_n;
  if (tiles_n > INT32_MAX) return MOE_ERR_INVALID_ARG;
  const size_t smem = size_t(3) * 4 * (num_experts + 1);
  tile_list_kernel<<<1, 256, smem, static_cast<cudaStream_t>(stream)>>>(
      expert_offsets, offsets_int64, num_experts, m_total, block_m, static_cast<int>(tiles_n),
      order, out_expert, out_tile_m, out_tile_n, max_items, out_count, status);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}
