// On-device tile scheduler for the grouped GEMM.
//
// The reference builds an (expert, tile_m, tile_n) work list on the host side
// of every call (_build_work_queue, src/triton_grouped_gemm.py:240-297: per-expert
// counts clamped at zero, ceil(count/block_m) row tiles times ceil(n/block_n)
// column tiles, expert-major).  Here each CTA derives the same list from
// expert_offsets in shared memory: per-expert tile counts and their exclusive
// prefix sum, then a binary search maps a linear tile id to its expert.  No
// host synchronisation and nothing to cache.
#pragma once

#include <cstdint>

#include "../../include/moe_overlap.h"
#include "ptx.cuh"

namespace moe {

struct TileCoord {
  int expert;
  int tile_m;
  int tile_n;
  int row0;  // first global row of the tile
  int rows;  // rows of the tile that belong to the expert (1..block_m)
};

__device__ __forceinline__ long long load_offset(const void* offsets, int is64, int i) {
  return is64 ? static_cast<const long long*>(offsets)[i]
              : static_cast<long long>(static_cast<const int*>(offsets)[i]);
}

// Run by one full warp.  Writes tile_prefix[0..E] (exclusive prefix of tiles per
// expert; tile_prefix[E] = total), seg_start[e] and seg_rows[e] (the expert's
// row range clamped to [0, m_total]).  Offsets outside [0, m_total] are
// clamped and reported as MOE_ERR_OFFSETS; a tile count beyond INT32_MAX is
// reported as MOE_ERR_CAPACITY and yields an empty list.
__device__ __forceinline__ void build_tile_prefix(const void* offsets, int is64, int num_experts,
                                                  long long m_total, int block_m, int tiles_n,
                                                  int* tile_prefix, int* seg_start, int* seg_rows,
                                                  int32_t* status) {
  const int lane = lane_id();
  const int per = (num_experts + 31) / 32;
  const int beg = min(num_experts, lane * per);
  const int end = min(num_experts, beg + per);
  long long local = 0;
  bool bad = false;
  for (int e = beg; e < end; ++e) {
    const long long lo = load_offset(offsets, is64, e);
    const long long hi = load_offset(offsets, is64, e + 1);
    const long long clo = lo < 0 ? 0 : (lo > m_total ? m_total : lo);
    const long long chi = hi < 0 ? 0 : (hi > m_total ? m_total : hi);
    bad |= (clo != lo) || (chi != hi);
    const long long rows = chi > clo ? chi - clo : 0;
    seg_start[e] = static_cast<int>(clo);
    seg_rows[e] = static_cast<int>(rows);
    tile_prefix[e] = static_cast<int>(local);  // chunk-local for now
    local += ((rows + block_m - 1) / block_m) * tiles_n;
  }
  long long incl = local;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const long long v = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += v;
  }
  const long long excl = incl - local;
  const long long total = __shfl_sync(0xffffffffu, incl, 31);
  const bool overflow = total > 0x7fffffffll;
  for (int e = beg; e < end; ++e)
    tile_prefix[e] = overflow ? 0 : static_cast<int>(tile_prefix[e] + excl);
  if (lane == 0) {
    tile_prefix[num_experts] = overflow ? 0 : static_cast<int>(total);
    if (overflow) record_status(status, MOE_ERR_CAPACITY);
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) record_status(status, MOE_ERR_OFFSETS);
  __syncwarp();
}

// order 0: expert-major, tile_m, tile_n fastest (the reference list order,
// src/triton_grouped_gemm.py:277-286).  order 1: expert-major, tile_n, tile_m
// fastest, so consecutive tiles share one weight column block.
__device__ __forceinline__ TileCoord decode_tile(int t, int num_experts, const int* tile_prefix,
                                                 const int* seg_start, const int* seg_rows,
                                                 int block_m, int tiles_n, int order) {
  int lo = 0, hi = num_experts;  // invariant: tile_prefix[lo] <= t < tile_prefix[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tile_prefix[mid] <= t)
      lo = mid;
    else
      hi = mid;
  }
  TileCoord c;
  c.expert = lo;
  const int local = t - tile_prefix[lo];
  const int tiles_m = (tile_prefix[lo + 1] - tile_prefix[lo]) / tiles_n;
  if (order == 0) {
    c.tile_m = local / tiles_n;
    c.tile_n = local % tiles_n;
  } else {
    c.tile_n = local / tiles_m;
    c.tile_m = local % tiles_m;
  }
  c.row0 = seg_start[lo] + c.tile_m * block_m;
  const int left = seg_rows[lo] - c.tile_m * block_m;
  c.rows = left < block_m ? left : block_m;
  return c;
}

}  // namespace moe
