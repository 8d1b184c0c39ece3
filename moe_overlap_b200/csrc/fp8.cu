// FP8 (e4m3) dispatch payload: per-128-column quantisation and its inverse.
//
// DeepEP's dispatch can carry tokens as (e4m3 rows [T, H], float scales
// [T, H/128]) instead of bf16 rows, halving the bytes that cross NVLink
// (thirdParty/DeepEP/deep_ep/buffer.py:338-342).  These kernels make and undo
// that pair exactly as DeepEP's helpers define it (tests/utils.py:50-75):
//   quantise    amax = max(|x|) over each 128-column group, clamped to 1e-4;
//               q = e4m3(x * (rcp(amax) * 448)) rounded to nearest even with
//               saturation; scale = amax / 448
//   dequantise  bf16(float(q) * scale)
// Every arithmetic step is one IEEE float32 operation with round-to-nearest
// (rcp, mul, div), so the results match the reference bit for bit.  Both
// kernels are HBM-bound: 2H bytes read and H + H/32 written per row, and the
// reverse.
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/moe_overlap.h"
#include "host_common.h"

namespace moe {
namespace fp8 {

constexpr int kGroup = 128;
constexpr int kThreads = 256;

// One warp per (row, 128-column group): each lane converts 4 consecutive values.
__global__ void __launch_bounds__(kThreads) quantize_kernel(const __nv_bfloat16* x, int64_t ldx,
                                                            int64_t rows, int hidden, uint8_t* q,
                                                            int64_t ldq, float* scales, int64_t lds) {
  const int lane = threadIdx.x & 31;
  const int groups = hidden / kGroup;
  const int64_t total = rows * groups;
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total; w += warps) {
    const int64_t r = w / groups;
    const int g = static_cast<int>(w % groups);
    const uint2 raw = *reinterpret_cast<const uint2*>(x + r * ldx + g * kGroup + lane * 4);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
    const float2 f01 = __bfloat1622float2(h[0]), f23 = __bfloat1622float2(h[1]);
    const float f[4] = {f01.x, f01.y, f23.x, f23.y};
    float amax = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    amax = fmaxf(amax, 1e-4f);
    const float mult = __fmul_rn(__frcp_rn(amax), 448.0f);
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_fp8_storage_t b = __nv_cvt_float_to_fp8(__fmul_rn(f[i], mult), __NV_SATFINITE, __NV_E4M3);
      packed |= static_cast<uint32_t>(b) << (8 * i);
    }
    *reinterpret_cast<uint32_t*>(q + r * ldq + g * kGroup + lane * 4) = packed;
    if (lane == 0) scales[r * lds + g] = __fdiv_rn(amax, 448.0f);
  }
}

__device__ __forceinline__ float e4m3_to_float(uint32_t byte) {
  const __half_raw hr = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(byte), __NV_E4M3);
  return __half2float(__half(hr));  // every e4m3 value is exact in half and float
}

// 8 values per thread: 8 e4m3 bytes in, one 16-byte bf16 vector out.  Rows at or
// past *rows_dev (when given) are left untouched.
__global__ void __launch_bounds__(kThreads) dequantize_kernel(const uint8_t* q, int64_t ldq,
                                                              const float* scales, int64_t lds,
                                                              const int32_t* rows_dev,
                                                              int64_t rows_max, int hidden,
                                                              __nv_bfloat16* out, int64_t ldo) {
  int64_t rows = rows_max;
  if (rows_dev != nullptr) rows = min(rows_max, max(int64_t(0), static_cast<int64_t>(*rows_dev)));
  const int per_row = hidden / 8;
  const int64_t total = rows * per_row;
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / per_row;
    const int c = static_cast<int>(i % per_row) * 8;
    const uint2 raw = *reinterpret_cast<const uint2*>(q + r * ldq + c);
    const float s = scales[r * lds + c / kGroup];
    uint4 o;
    __nv_bfloat162* ob = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t word = j < 2 ? raw.x : raw.y;
      const int sh = (j & 1) * 16;
      const float a = e4m3_to_float((word >> sh) & 0xFFu);
      const float b = e4m3_to_float((word >> (sh + 8)) & 0xFFu);
      ob[j] = __floats2bfloat162_rn(__fmul_rn(a, s), __fmul_rn(b, s));
    }
    *reinterpret_cast<uint4*>(out + r * ldo + c) = o;
  }
}

static int grid_for(int64_t work, int per_block) {
  const int64_t g = (work + per_block - 1) / per_block;
  return static_cast<int>(g < 1 ? 1 : (g > 148 * 16 ? 148 * 16 : g));
}

}  // namespace fp8
}  // namespace moe

extern "C" int32_t moe_fp8_quantize(const void* x, int64_t ldx, int64_t rows, int32_t hidden,
                                    void* out_fp8, int64_t ld_out, float* out_scales,
                                    int64_t ld_scales, void* stream) {
  using namespace moe::fp8;
  if (rows < 0 || hidden <= 0 || hidden % kGroup != 0 || ldx < hidden || ld_out < hidden ||
      ld_scales < hidden / kGroup || ldx % 4 != 0 || ld_out % 4 != 0)
    return MOE_ERR_INVALID_ARG;
  if (rows == 0) return MOE_OK;
  if (x == nullptr || out_fp8 == nullptr || out_scales == nullptr ||
      reinterpret_cast<uintptr_t>(x) % 8 != 0 || reinterpret_cast<uintptr_t>(out_fp8) % 4 != 0)
    return MOE_ERR_INVALID_ARG;
  const int64_t warps = rows * (hidden / kGroup);
  quantize_kernel<<<grid_for(warps, kThreads / 32), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, rows, hidden, static_cast<uint8_t*>(out_fp8), ld_out,
      out_scales, ld_scales);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int32_t moe_fp8_dequantize(const void* x_fp8, int64_t ldx, const float* scales,
                                      int64_t ld_scales, const int32_t* rows_dev, int64_t rows_max,
                                      int32_t hidden, void* out, int64_t ld_out, void* stream) {
  using namespace moe::fp8;
  if (rows_max < 0 || hidden <= 0 || hidden % kGroup != 0 || ldx < hidden || ld_out < hidden ||
      ld_scales < hidden / kGroup || ldx % 8 != 0 || ld_out % 8 != 0)
    return MOE_ERR_INVALID_ARG;
  if (rows_max == 0) return MOE_OK;
  if (x_fp8 == nullptr || scales == nullptr || out == nullptr || !moe::aligned16(out) ||
      reinterpret_cast<uintptr_t>(x_fp8) % 8 != 0)
    return MOE_ERR_INVALID_ARG;
  dequantize_kernel<<<grid_for(rows_max * (hidden / 8), kThreads), kThreads, 0,
                      static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(x_fp8), ldx, scales, ld_scales, rows_dev, rows_max, hidden,
      static_cast<__nv_bfloat16*>(out), ld_out);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}
