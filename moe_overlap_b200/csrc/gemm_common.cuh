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

// Expert-parallel combine push: instead of C, row r of the result goes to
// peers[src[r].x] + cb + dst[r] * ldc elements (the source rank's combine rows);
// rows with src[r].x < 0 or dst[r] < 0 (alignment padding) are not stored.
struct PushTarget {
  const int2* src;         // [m_total] {source rank, token}; null = ordinary C stores
  const int32_t* dst;      // [m_total] row index in the source rank's combine rows
  uint8_t* const* peers;   // [world] every rank's symmetric buffer, as mapped here
  uint64_t cb;             // byte offset of the combine rows in each buffer
  const CUtensorMap* maps; // [world] TMA store maps of each rank's combine rows, or null
};

// Expert-ordered dispatch: the rows of local expert e are all present once
// arrived[e] >= expected[e] (peers add to arrived[e] as their rows land).
struct ArrivalWait {
  const uint32_t* arrived;  // [num_experts] arrival counters (this GPU's memory)
  const int32_t* expected;  // [num_experts] rows of each expert
  uint64_t wait_ns;         // bound on each wait
};

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
  // optional epilogue operands (all may be null)
  const float* row_scale;  // v = acc * row_scale[row]
  const void* aux_in;      // MOE_ACT_DGELU: C = v * gelu'(aux_in[row, col])
  void* aux_out;           // aux_out[row, col] = v (before the activation)
  int64_t ld_aux;
  int c_tma;               // the CTA-pair kernel may store C through its TMA store map
  int swap_tails;          // the CTA-pair kernel computes tiles of <= 224 rows swapped
  PushTarget push;         // combine push instead of C (push.src != null)
  ArrivalWait arrival;     // arrival.arrived != null: wait for each expert's rows
};

// Producer side of an expert-ordered dispatch: returns once every row of `expert`
// has landed (then visible to the TMA loads that follow), or false after
// p.arrival.wait_ns.  Without arrival counters it returns at once.
__device__ __forceinline__ bool wait_expert_rows(const Params& p, int expert) {
  if (p.arrival.arrived == nullptr) return true;
  const uint32_t need = static_cast<uint32_t>(max(0, p.arrival.expected[expert]));
  const uint32_t* ctr = p.arrival.arrived + expert;
  if (ld_acquire_sys_u32(ctr) < need) {
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_sys_u32(ctr) < need) {
      if (global_timer_ns() - t0 > p.arrival.wait_ns) return false;
      __nanosleep(64);
    }
  }
  fence_proxy_async_global();
  return true;
}

__device__ __forceinline__ float gelu_erf(float x) {
  return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f));
}

// d/dx [x * Phi(x)] = Phi(x) + x * phi(x), with Phi the standard normal CDF.
__device__ __forceinline__ float gelu_erf_grad(float x) {
  const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752440f));
  const float pdf = 0.39894228040143267794f * expf(-0.5f * x * x);
  return cdf + x * pdf;
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if constexpr (BF16) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&v));
  } else {
    return __half22float2(*reinterpret_cast<const __half2*>(&v));
  }
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

// Epilogue of one 128-row fp32 accumulator held in TMEM lanes [32*quad, 32*quad+32)
// of this warp: the 32-column chunks [ch0, ch0 + nch) of the tile, for rows
// [0, rows) of the tile starting at global row `row0`, columns n0.. (< n).
// v = acc (* row_scale), optionally saved to aux_out, then C = act(v) with act
// none, GELU or v * gelu'(aux_in), rounded and written with 16-byte stores.
// aux_in for chunk c+1 is loaded while chunk c is computed, so the epilogue of
// the backward GEMM does not wait a full memory latency per chunk.
//
// With `tmap_c` (a 2-D {N, rows} or, when e3 >= 0, 3-D {N, rows, E} tensor map of C
// with 32x32 boxes and 64-byte swizzle) a warp whose 32 rows may all be written
// stages each bf16 chunk in its 2 KiB of shared memory at `stage` and stores it with
// one TMA bulk store instead of 32 scattered 16-byte stores per instruction.  A warp
// may use it when all its rows belong to the tile (rows >= 32*quad + 32) or, with
// `rows_clipped_by_map`, when the map's row extent is the tile's own bound (rows past
// it are dropped by the TMA unit).  Other warps store directly.  The caller drains
// its bulk stores (bulk_wait_group0) before the CTA exits.
template <bool BF16, bool PUSH = false>
__device__ __forceinline__ void store_accumulator(uint32_t t_base, int quad, int lane, int row0,
                                                  int rows, int n0, const Params& p, int ch0 = 0,
                                                  int nch = 8, const void* tmap_c = nullptr,
                                                  uint32_t stage = 0, bool rows_clipped_by_map = false,
                                                  int e3 = -1) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int row_in_tile = quad * 32 + lane;
  bool row_ok = row_in_tile < rows;
  const int64_t grow = int64_t(row0) + row_in_tile;
  T* crow;
  // TMA store target of this warp's rows: C's map at row0 + 32*quad, or, for a
  // combine push whose 32 rows all go to one source rank's consecutive cb rows,
  // that rank's cb map at the first row (warp-uniform).
  const void* tmap = tmap_c;
  int trow = row0 + quad * 32;
  if constexpr (PUSH) {
    // Combine push: this row's destination on its source rank (peer memory).
    crow = nullptr;
    int2 src = make_int2(-1, -1);
    int32_t dst = -1;
    if (row_ok) {
      src = p.push.src[grow];
      dst = p.push.dst[grow];
      if (src.x >= 0 && dst >= 0)
        crow = reinterpret_cast<T*>(p.push.peers[src.x] + p.push.cb) + int64_t(dst) * p.ldc;
      else
        row_ok = false;
    }
    const int s0 = __shfl_sync(0xffffffffu, src.x, 0);
    const int d0 = __shfl_sync(0xffffffffu, dst, 0);
    const bool run = __all_sync(0xffffffffu, row_ok && src.x == s0 && dst == d0 + lane);
    tmap = (run && p.push.maps != nullptr && stage != 0) ? static_cast<const void*>(p.push.maps + s0)
                                                         : nullptr;
    trow = d0;
  } else {
    crow = reinterpret_cast<T*>(p.c) + grow * p.ldc;
  }
  const float rs = (p.row_scale != nullptr && row_ok) ? p.row_scale[grow] : 1.0f;
  // DGELU and MUL_AUX read aux_in; DGELU maps it through gelu', MUL_AUX uses it as is.
  const bool dgelu = p.activation == MOE_ACT_DGELU || p.activation == MOE_ACT_MUL_AUX;
  const bool aux_is_grad = p.activation == MOE_ACT_MUL_AUX;
  const T* arow = dgelu ? reinterpret_cast<const T*>(p.aux_in) + grow * p.ld_aux : nullptr;
  // 16-byte vectors of chunk c that lie inside the matrix (0 when the row or chunk is outside).
  auto vecs = [&](int c) {
    const int col = n0 + c * 32;
    return (row_ok && col < p.n) ? min(4, (p.n - col) / 8) : 0;
  };
  uint4 anext[4] = {};
  if (dgelu) {
    const int nv = vecs(ch0);
    const uint4* ai = reinterpret_cast<const uint4*>(arow + n0 + ch0 * 32);
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (q < nv) anext[q] = ai[q];
  }
#pragma unroll 1
  for (int ch = ch0; ch < ch0 + nch; ++ch) {
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_base + ch * 32, r);
    uint4 acur[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) acur[q] = anext[q];
    if (dgelu && ch + 1 < ch0 + nch) {
      const int nv = vecs(ch + 1);
      const uint4* ai = reinterpret_cast<const uint4*>(arow + n0 + (ch + 1) * 32);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (q < nv) anext[q] = ai[q];
    }
    tmem_wait_ld();
    const int col = n0 + ch * 32;
    const int nvec = vecs(ch);  // 16-byte vectors inside the matrix
    const bool tma = tmap != nullptr && col < p.n &&
                     (PUSH || (rows_clipped_by_map ? quad * 32 < rows : quad * 32 + 32 <= rows));  // warp-uniform
    if (tma || nvec > 0) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * rs;
      if (p.activation == MOE_ACT_GELU_SAVE_GRAD) {
        // One erf per element: C = v * Phi(v), aux_out = Phi(v) + v * phi(v).
        uint4* ad = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.aux_out) + grow * p.ld_aux + col);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint32_t g[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float gg2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const float x = v[8 * q + 2 * h + u];
              const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752440f));
              gg2[u] = cdf + x * (0.39894228040143267794f * expf(-0.5f * x * x));
              v[8 * q + 2 * h + u] = x * cdf;
            }
            g[h] = pack2<BF16>(gg2[0], gg2[1]);
          }
          if (q < nvec) ad[q] = make_uint4(g[0], g[1], g[2], g[3]);
        }
      } else if (p.aux_out != nullptr && nvec > 0) {
        uint4* ad = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.aux_out) + grow * p.ld_aux + col);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < nvec)
            ad[q] = make_uint4(pack2<BF16>(v[8 * q], v[8 * q + 1]), pack2<BF16>(v[8 * q + 2], v[8 * q + 3]),
                               pack2<BF16>(v[8 * q + 4], v[8 * q + 5]),
                               pack2<BF16>(v[8 * q + 6], v[8 * q + 7]));
      }
      if (p.activation == MOE_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
      } else if (dgelu) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          if (q < nvec) {
            const uint32_t w[4] = {acur[q].x, acur[q].y, acur[q].z, acur[q].w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float2 f = unpack2<BF16>(w[h]);
              v[8 * q + 2 * h] *= aux_is_grad ? f.x : gelu_erf_grad(f.x);
              v[8 * q + 2 * h + 1] *= aux_is_grad ? f.y : gelu_erf_grad(f.y);
            }
          }
        }
      }
      if (tma) {
        if (lane == 0) bulk_wait_group_read0();  // the previous chunk's store has read the buffer
        __syncwarp();
        // Row `lane` is 64 bytes; 16-byte unit q sits at unit q ^ ((lane >> 1) & 3) (64-byte swizzle).
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_shared_v4(stage + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4), pack2<BF16>(v[8 * q], v[8 * q + 1]),
                       pack2<BF16>(v[8 * q + 2], v[8 * q + 3]), pack2<BF16>(v[8 * q + 4], v[8 * q + 5]),
                       pack2<BF16>(v[8 * q + 6], v[8 * q + 7]));
        fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) {
          if (e3 >= 0)
            tma_store_3d(tmap, stage, col, trow, e3);
          else
            tma_store_2d(tmap, stage, col, trow);
          bulk_commit_group();
        }
      } else {
        uint4* dst = reinterpret_cast<uint4*>(crow + col);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (q < nvec)
            dst[q] = make_uint4(pack2<BF16>(v[8 * q], v[8 * q + 1]), pack2<BF16>(v[8 * q + 2], v[8 * q + 3]),
                                pack2<BF16>(v[8 * q + 4], v[8 * q + 5]),
                                pack2<BF16>(v[8 * q + 6], v[8 * q + 7]));
      }
    }
  }
}

// Zero-fill of the whole output (no expert owns a row), grid-strided.
template <bool BF16>
__device__ __forceinline__ void zero_output(const Params& p, int nthreads) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  if (p.push.src != nullptr) return;  // combine push: no expert rows, nothing to push
  const int64_t chunks_per_row = p.n / 8;
  const int64_t total_chunks = int64_t(p.m_total) * chunks_per_row;
  for (int64_t i = int64_t(blockIdx.x) * nthreads + threadIdx.x; i < total_chunks;
       i += int64_t(gridDim.x) * nthreads) {
    const int64_t r = i / chunks_per_row, cc = i % chunks_per_row;
    *reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.c) + r * p.ldc + cc * 8) = make_uint4(0, 0, 0, 0);
  }
}

// The grouped GEMM with the extended epilogue (moe_grouped_gemm_ex's contract) and,
// when push is non-null, the combine push instead of C (c may then be null and ldc
// is the combine row stride).  Returns a MOE_* code.
int grouped_gemm_launch(const void* a, int64_t lda, const void* b, int64_t b_stride_e,
                        int64_t b_stride_k, int64_t b_stride_n, void* c, int64_t ldc,
                        const void* expert_offsets, int32_t offsets_int64, int64_t m_total,
                        int64_t k, int64_t n, int32_t num_experts, int32_t dtype,
                        int32_t activation, int32_t num_sms, int32_t use_atomic_queue,
                        int32_t* work_counter, const float* row_scale, const void* aux_in,
                        void* aux_out, int64_t ld_aux, int32_t* status, cudaStream_t stream,
                        const PushTarget* push, const ArrivalWait* arrival = nullptr);

// Launches the 2-SM (CTA pair) kernel; grid must be even.  `ta_half` is A's map with
// 64-row boxes (the rows a swapped tile of N <= 128 reads per CTA); `tc` is the 2-D {N, m_total}
// store map of C (32x32 boxes, 64-byte swizzle), used when p.c_tma is set.
// Returns a MOE_* code.
int launch_pair_kernel(bool bf16, bool b_mn, const CUtensorMap& ta, const CUtensorMap& ta_half,
                       const CUtensorMap& tb, const CUtensorMap& tc, const Params& p, int grid,
                       cudaStream_t stream);

}  // namespace gg
}  // namespace moe
