// Pieces shared by the 1-SM and 2-SM grouped GEMM kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "../../include/moe_overlap.h"
#include "ptx.cuh"

namespace moe {
namespace gg {

constexpr int kMaxExperts = 1024;

struct Params {
  void* c;
  int64_t ldc;
  const void* offsets;
  int offsets_int64;
  int m_total;
  int k;
  int n;
  int num_experts;
  int activation;
  int use_atomic;
  int tile_order;
  int* work_counter;
  int32_t* status;
};

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// All lanes of the calling warp wait; the outcome is made warp-uniform so a
// following .sync.aligned tcgen05 instruction is never reached by part of a warp.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, const volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// Epilogue of one 128-row x 256-column fp32 accumulator held in TMEM lanes
// [32*quad, 32*quad+32) of this warp: optional GELU, round, and 16-byte stores of
// rows [0, rows) of the tile starting at global row `row0`, columns n0.. (< n).
template <bool BF16>
__device__ __forceinline__ void store_accumulator(uint32_t t_base, int quad, int lane, int row0,
                                                  int rows, int n0, const Params& p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int row_in_tile = quad * 32 + lane;
  const bool row_ok = row_in_tile < rows;
  T* crow = reinterpret_cast<T*>(p.c) + (int64_t(row0) + row_in_tile) * p.ldc;
#pragma unroll 1
  for (int ch = 0; ch < 256 / 32; ++ch) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_base + ch * 32, r);
    tmem_wait_ld();
    const int col = n0 + ch * 32;
    if (row_ok && col < p.n) {
      uint32_t packed[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        float lo = __uint_as_float(r[2 * j]);
        float hi = __uint_as_float(r[2 * j + 1]);
        if (p.activation == MOE_ACT_GELU) {
          lo = gelu_erf(lo);
          hi = gelu_erf(hi);
        }
        packed[j] = pack2<BF16>(lo, hi);
      }
      uint4* dst = reinterpret_cast<uint4*>(crow + col);
      if (col + 32 <= p.n) {
#pragma unroll
        for (int v = 0; v < 4; ++v)
          dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
      } else {
#pragma unroll
        for (int v = 0; v < 4; ++v)
          if (col + 8 * v + 8 <= p.n)
            dst[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
      }
    }
  }
}

// Zero-fill of the whole output (no expert owns a row), grid-strided.
template <bool BF16>
__device__ __forceinline__ void zero_output(const Params& p, int nthreads) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int64_t chunks_per_row = p.n / 8;
  const int64_t total_chunks = int64_t(p.m_total) * chunks_per_row;
  for (int64_t i = int64_t(blockIdx.x) * nthreads + threadIdx.x; i < total_chunks;
       i += int64_t(gridDim.x) * nthreads) {
    const int64_t r = i / chunks_per_row, cc = i % chunks_per_row;
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.c) + r * p.ldc + cc * 8) = make_uint4(0, 0, 0, 0);
  }
}

// Launches the 2-SM (CTA pair) kernel; grid must be even.  Returns a MOE_* code.
int launch_pair_kernel(bool bf16, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb,
                       const Params& p, int grid, cudaStream_t stream);

}  // namespace gg
}  // namespace moe
