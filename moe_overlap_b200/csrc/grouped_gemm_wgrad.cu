// Weight-gradient grouped GEMM on sm_100a: C[e] = A_e^T . B_e over ragged row segments.
//
// For every expert e with rows r in [off[e], off[e+1]):
//   C[e][m][n] = sum_r A[r][m] * B[r][n]       (fp32 accumulation, bf16/fp16 result)
// i.e. dW1[e] = dA_e^T X_e and dW2[e] = dY_e^T H_e of the routed experts' backward,
// which the reference does not have (it runs inference only,
// src/train_moe_baseline.py:524-552).  The contraction runs over the token rows,
// so both operands are MN-major in shared memory, straight from their row-major
// storage: tcgen05 kind::f16 MMAs with A and B MN-major.
//
// Every expert segment must start and end on a multiple of 64 rows (the
// exchange's expert_alignment provides that, with zero padding rows), so a
// 64-row k-block never straddles two experts; a misaligned segment is reported
// as MOE_ERR_OFFSETS.  An expert without rows gets a zero gradient.
//
// Two kernels.  Grids of two or more SMs run wgrad_pair_kernel (CTA pairs,
// cta_group::2, 256x256 tiles, TMA-store epilogue; see its comment below).  The
// 1-SM wgrad_kernel (for num_sms == 1 or MOE_B200_GEMM_KERNEL=1): one CTA per SM,
// 192 threads: warp 0 schedules (striped over a fixed tile grid of
// E x ceil(M/128) x ceil(N/256)) and TMA-loads, warp 1 owns TMEM and issues
// 128x256x16 MMAs, warps 2-5 run the epilogue; two TMEM accumulators overlap the
// epilogue of one tile with the main loop of the next.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "gemm_common.cuh"
#include "host_common.h"
#include "sched.cuh"

namespace moe {
namespace wg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // token rows per k-block
constexpr int UMMA_K = 16;
constexpr int STAGES = 4;
constexpr int QDEPTH = 8;
constexpr int NUM_THREADS = 192;
constexpr int NUM_EPI_WARPS = 4;
constexpr int SLAB_BYTES = BK * 64 * 2;          // 64 k-rows x 64 MN-columns
constexpr int A_STAGE_BYTES = (BM / 64) * SLAB_BYTES;  // 16 KiB
constexpr int B_STAGE_BYTES = (BN / 64) * SLAB_BYTES;  // 32 KiB
constexpr uint32_t TMEM_COLS = 2 * BN;

struct Ctrl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t qfull[QDEPTH];
  uint64_t qempty[QDEPTH];
  uint64_t drain;
  int4 slot[QDEPTH];  // {expert (-1 = end), m0, n0, num_kb}
  int4 slot2[QDEPTH]; // {first row, 0, 0, 0}
  uint32_t tmem_base;
  int abort;
};

struct WParams {
  gg::Params out;  // c, ldc (row stride inside one expert's C), n, activation (none), status
  int64_t c_stride_e;
  const void* offsets;
  int offsets_int64;
  int rows_total;
  int m;
  int n;
  int num_experts;
};

constexpr size_t kSmem = 1024 + size_t(STAGES) * (A_STAGE_BYTES + B_STAGE_BYTES) +
                         ((sizeof(Ctrl) + 15) / 16) * 16;

template <bool BF16>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    wgrad_kernel(const __grid_constant__ CUtensorMap tmap_a,
                 const __grid_constant__ CUtensorMap tmap_b, const WParams wp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(sB + STAGES * B_STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = lane_id();
  const int tiles_m = (wp.m + BM - 1) / BM;
  const int tiles_n = (wp.n + BN - 1) / BN;
  const int total_tiles = wp.num_experts * tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&ctrl->tfull[a]), 1);
      mbar_init(smem_u32(&ctrl->tempty[a]), NUM_EPI_WARPS);
    }
    for (int q = 0; q < QDEPTH; ++q) {
      mbar_init(smem_u32(&ctrl->qfull[q]), 1);
      mbar_init(smem_u32(&ctrl->qempty[q]), 1 + NUM_EPI_WARPS);
    }
    mbar_init(smem_u32(&ctrl->drain), 1);
    ctrl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc(smem_u32(&ctrl->tmem_base), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = ctrl->tmem_base;
  volatile int* abort_flag = &ctrl->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int stage = 0, q = 0;
      uint32_t phase = 0, qphase = 0;
      int issued[STAGES] = {0, 0, 0, 0};
      bool failed = false;
      for (int t = blockIdx.x;; t += gridDim.x) {
        if (!mbar_wait(smem_u32(&ctrl->qempty[q]), qphase ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        if (t >= total_tiles) {
          ctrl->slot[q] = make_int4(-1, 0, 0, 0);
          mbar_arrive(smem_u32(&ctrl->qfull[q]));
          break;
        }
        const int e = t / (tiles_m * tiles_n);
        const int rem = t % (tiles_m * tiles_n);
        const int m0 = (rem / tiles_n) * BM;
        const int n0 = (rem % tiles_n) * BN;
        long long lo = load_offset(wp.offsets, wp.offsets_int64, e);
        long long hi = load_offset(wp.offsets, wp.offsets_int64, e + 1);
        if (lo < 0 || hi > wp.rows_total || lo % BK != 0 || hi % BK != 0) {
          record_status(wp.out.status, MOE_ERR_OFFSETS);
          lo = hi = 0;
        }
        const int num_kb = hi > lo ? static_cast<int>((hi - lo) / BK) : 0;
        ctrl->slot[q] = make_int4(e, m0, n0, num_kb);
        ctrl->slot2[q] = make_int4(static_cast<int>(lo), 0, 0, 0);
        mbar_arrive(smem_u32(&ctrl->qfull[q]));
        if (++q == QDEPTH) {
          q = 0;
          qphase ^= 1;
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&ctrl->empty[stage]), phase ^ 1, abort_flag)) {
            failed = true;
            break;
          }
          const uint32_t fb = smem_u32(&ctrl->full[stage]);
          mbar_arrive_expect_tx(fb, A_STAGE_BYTES + B_STAGE_BYTES);
          const int k0 = static_cast<int>(lo) + kb * BK;
          const uint32_t a_dst = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_dst = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
          for (int j = 0; j < BM / 64; ++j) tma_load_2d(a_dst + j * SLAB_BYTES, &tmap_a, fb, m0 + 64 * j, k0);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j) tma_load_2d(b_dst + j * SLAB_BYTES, &tmap_b, fb, n0 + 64 * j, k0);
          ++issued[stage];
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (failed) break;
      }
      if (failed) {
        record_status(wp.out.status, MOE_ERR_TIMEOUT);
        *abort_flag = 1;
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] > 0)
            mbar_wait(smem_u32(&ctrl->full[s]), uint32_t((issued[s] - 1) & 1), nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BF16, BM, BN, true, true);
      int stage = 0, q = 0, acc = 0;
      uint32_t phase = 0, qphase = 0, aphase = 0;
      bool failed = false, issued_any = false;
      while (true) {
        if (!mbar_wait(smem_u32(&ctrl->qfull[q]), qphase, abort_flag)) {
          failed = true;
          break;
        }
        const int4 s = ctrl->slot[q];
        mbar_arrive(smem_u32(&ctrl->qempty[q]));
        if (++q == QDEPTH) {
          q = 0;
          qphase ^= 1;
        }
        if (s.x < 0) break;
        if (s.w == 0) continue;  // no rows: the epilogue writes zeros, no accumulator used
        if (!mbar_wait(smem_u32(&ctrl->tempty[acc]), aphase ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < s.w; ++kb) {
          if (!mbar_wait(smem_u32(&ctrl->full[stage]), phase, abort_flag)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // Both operands MN-major: 64-column slabs SLAB_BYTES apart (LBO), 8-row
            // k groups 1024 bytes apart (SBO); a 16-row k step is +2048 bytes.
            const uint64_t adesc = smem_desc_sw128(a_base + kk * UMMA_K * 128, SLAB_BYTES, 1024);
            const uint64_t bdesc = smem_desc_sw128(b_base + kk * UMMA_K * 128, SLAB_BYTES, 1024);
            umma_f16(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(smem_u32(&ctrl->empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (failed) break;
        umma_commit(smem_u32(&ctrl->tfull[acc]));
        if (++acc == 2) {
          acc = 0;
          aphase ^= 1;
        }
      }
      if (failed) {
        record_status(wp.out.status, MOE_ERR_TIMEOUT);
        *abort_flag = 1;
        if (issued_any) {
          umma_commit(smem_u32(&ctrl->drain));
          mbar_wait(smem_u32(&ctrl->drain), 0, nullptr);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    const int quad = warp & 3;
    int q = 0, acc = 0;
    uint32_t qphase = 0, aphase = 0;
    bool failed = false;
    while (true) {
      if (!gg::warp_wait(smem_u32(&ctrl->qfull[q]), qphase, abort_flag)) {
        failed = true;
        break;
      }
      const int4 s = ctrl->slot[q];
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->qempty[q]));
      if (++q == QDEPTH) {
        q = 0;
        qphase ^= 1;
      }
      if (s.x < 0) break;
      gg::Params op = wp.out;
      op.c = reinterpret_cast<T*>(wp.out.c) + int64_t(s.x) * wp.c_stride_e;
      const int rows = min(BM, wp.m - s.y);
      if (s.w == 0) {
        const int r = quad * 32 + lane;
        if (r < rows) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(op.c) + int64_t(s.y + r) * op.ldc + s.z);
          for (int v = 0; v < BN / 8 && s.z + 8 * v < wp.n; ++v) dst[v] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      if (!gg::warp_wait(smem_u32(&ctrl->tfull[acc]), aphase, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      gg::store_accumulator<BF16>(tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN), quad,
                                  lane, s.y, rows, s.z, op);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->tempty[acc]));
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1;
      }
    }
    if (failed && lane == 0) {
      record_status(wp.out.status, MOE_ERR_TIMEOUT);
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool BF16>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const WParams& wp, int grid,
                  cudaStream_t stream) {
  auto kern = wgrad_kernel<BF16>;
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MOE_ERR_CUDA;
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev], [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kSmem));
  });
  if (attr_err != cudaSuccess) return MOE_ERR_CUDA;
  kern<<<grid, NUM_THREADS, kSmem, stream>>>(ta, tb, wp);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace wg
}  // namespace moe

namespace moe {
namespace wg {
namespace pair {

// CTA-pair (cta_group::2) variant: 256x256 tiles of C[e], each CTA holding 128
// rows of M (its A half) and loading 128 columns of N (its B half) per 64-row
// k-block, so a stage is 32 KiB per CTA and six stages fit.  The leader takes
// tiles striped over the pairs and posts them to both CTAs' tile rings; warp 1
// of the leader issues tcgen05.mma.cta_group::2 with both operands MN-major; 8
// epilogue warps per CTA split the 256 columns like the forward pair kernel.
// No load uses cluster multicast.
constexpr int BM = 256, BM_CTA = 128, BN = 256, BN_CTA = 128, BK = 64, UMMA_K = 16;
constexpr int STAGES = 6, QDEPTH = 8, NUM_EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int SLAB_BYTES = BK * 64 * 2;
constexpr int A_STAGE_BYTES = (BM_CTA / 64) * SLAB_BYTES;  // 16 KiB
constexpr int B_STAGE_BYTES = (BN_CTA / 64) * SLAB_BYTES;  // 16 KiB
constexpr uint32_t PAIR_TX_BYTES = 2 * (A_STAGE_BYTES + B_STAGE_BYTES);
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr int EPI_STAGE_BYTES = 32 * 32 * 2;  // one 32x32 bf16 chunk per epilogue warp

struct Ctrl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t qfull[QDEPTH];
  uint64_t qempty[QDEPTH];
  uint64_t drain;
  int4 slot[QDEPTH];  // {expert (-1 = end), m0, n0, num_kb}
  int4 slot2[QDEPTH]; // {first row, 0, 0, 0}
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSmem = 1024 + size_t(STAGES) * (A_STAGE_BYTES + B_STAGE_BYTES) +
                         size_t(NUM_EPI_WARPS) * EPI_STAGE_BYTES + ((sizeof(Ctrl) + 15) / 16) * 16;

// 144 registers leave room for a 4-warp exchange block beside this kernel (see
// the forward pair kernel): the backward's combine runs during the weight gradients.
template <bool BF16>
__global__ void __cluster_dims__(2, 1, 1) __maxnreg__(144)
    wgrad_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                      const __grid_constant__ CUtensorMap tmap_b,
                      const __grid_constant__ CUtensorMap tmap_c, const WParams wp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint8_t* sEpi = sB + STAGES * B_STAGE_BYTES;  // 1024-aligned, EPI_STAGE_BYTES per epilogue warp
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(sEpi + NUM_EPI_WARPS * EPI_STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = lane_id();
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int tiles_m = (wp.m + BM - 1) / BM;
  const int tiles_n = (wp.n + BN - 1) / BN;
  const int total_tiles = wp.num_experts * tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&ctrl->tfull[a]), 1);
      mbar_init(smem_u32(&ctrl->tempty[a]), 2 * NUM_EPI_WARPS);
    }
    for (int q = 0; q < QDEPTH; ++q) {
      mbar_init(smem_u32(&ctrl->qfull[q]), 1);
      // leader MMA + follower producer + the epilogue warps of both CTAs
      mbar_init(smem_u32(&ctrl->qempty[q]), 2 + 2 * NUM_EPI_WARPS);
    }
    mbar_init(smem_u32(&ctrl->drain), 1);
    ctrl->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_b);
  }
  if (warp == 1) {
    __syncwarp();
    tmem_alloc_pair(smem_u32(&ctrl->tmem_base), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // barrier inits of both CTAs visible before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = ctrl->tmem_base;
  volatile int* abort_flag = &ctrl->abort;

  if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int stage = 0, q = 0;
      uint32_t phase = 0, qphase = 0;
      bool failed = false;
      const int pair_id = static_cast<int>(cluster_id_x());
      const int npairs = static_cast<int>(nclusters_x());
      for (int iter = 0;; ++iter) {
        int4 s, s2 = make_int4(0, 0, 0, 0);
        if (leader) {
          const int t = pair_id + iter * npairs;
          if (!mbar_wait_cluster(smem_u32(&ctrl->qempty[q]), qphase ^ 1, abort_flag)) {
            failed = true;
            break;
          }
          if (t >= total_tiles) {
            s = make_int4(-1, 0, 0, 0);
          } else {
            const int e = t / (tiles_m * tiles_n);
            const int rem = t % (tiles_m * tiles_n);
            long long lo = load_offset(wp.offsets, wp.offsets_int64, e);
            long long hi = load_offset(wp.offsets, wp.offsets_int64, e + 1);
            if (lo < 0 || hi > wp.rows_total || lo % BK != 0 || hi % BK != 0) {
              record_status(wp.out.status, MOE_ERR_OFFSETS);
              lo = hi = 0;
            }
            s = make_int4(e, (rem / tiles_n) * BM, (rem % tiles_n) * BN,
                          hi > lo ? static_cast<int>((hi - lo) / BK) : 0);
            s2 = make_int4(static_cast<int>(lo), 0, 0, 0);
          }
          ctrl->slot[q] = s;
          ctrl->slot2[q] = s2;
          st_shared_cluster_v4(mapa_shared(smem_u32(&ctrl->slot[q]), 1), s);
          st_shared_cluster_v4(mapa_shared(smem_u32(&ctrl->slot2[q]), 1), s2);
          mbar_arrive(smem_u32(&ctrl->qfull[q]));
          mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->qfull[q]), 1));
        } else {
          if (!mbar_wait_cluster(smem_u32(&ctrl->qfull[q]), qphase, abort_flag)) {
            failed = true;
            break;
          }
          s = ctrl->slot[q];
          s2 = ctrl->slot2[q];
          mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->qempty[q]), 0));
        }
        if (++q == QDEPTH) {
          q = 0;
          qphase ^= 1;
        }
        if (s.x < 0) break;
        const int m_a = s.y + static_cast<int>(crank) * BM_CTA;
        const int n_b = s.z + static_cast<int>(crank) * BN_CTA;
        for (int kb = 0; kb < s.w; ++kb) {
          if (!mbar_wait_cluster(smem_u32(&ctrl->empty[stage]), phase ^ 1, abort_flag)) {
            failed = true;
            break;
          }
          const uint32_t full_local = smem_u32(&ctrl->full[stage]);
          if (leader) mbar_arrive_expect_tx(full_local, PAIR_TX_BYTES);
          const uint32_t full_leader = mapa_shared(full_local, 0);
          const int k0 = s2.x + kb * BK;
          const uint32_t a_dst = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_dst = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
          for (int j = 0; j < BM_CTA / 64; ++j)
            tma_load_2d_pair(a_dst + j * SLAB_BYTES, &tmap_a, full_leader, m_a + 64 * j, k0);
#pragma unroll
          for (int j = 0; j < BN_CTA / 64; ++j)
            tma_load_2d_pair(b_dst + j * SLAB_BYTES, &tmap_b, full_leader, n_b + 64 * j, k0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (failed) break;
      }
      if (failed) {
        record_status(wp.out.status, MOE_ERR_TIMEOUT);
        *abort_flag = 1;
        // Give loads already issued time to land before this CTA can leave.
        const long long t0 = clock64();
        while (clock64() - t0 < (1ll << 22)) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA (leader only) --
    if (leader && lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BF16, BM, BN, true, true);
      int stage = 0, q = 0, acc = 0;
      uint32_t phase = 0, qphase = 0, aphase = 0;
      bool failed = false, issued_any = false;
      while (true) {
        if (!mbar_wait_cluster(smem_u32(&ctrl->qfull[q]), qphase, abort_flag)) {
          failed = true;
          break;
        }
        const int4 s = ctrl->slot[q];
        mbar_arrive(smem_u32(&ctrl->qempty[q]));
        if (++q == QDEPTH) {
          q = 0;
          qphase ^= 1;
        }
        if (s.x < 0) break;
        if (s.w == 0) continue;  // no rows: both epilogues write zeros, no accumulator used
        if (!mbar_wait_cluster(smem_u32(&ctrl->tempty[acc]), aphase ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < s.w; ++kb) {
          if (!mbar_wait_cluster(smem_u32(&ctrl->full[stage]), phase, abort_flag)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // Both operands MN-major: 64-column slabs SLAB_BYTES apart (LBO), 8-row
            // k groups 1024 bytes apart (SBO); a 16-row k step is +2048 bytes.
            const uint64_t adesc = smem_desc_sw128(a_base + kk * UMMA_K * 128, SLAB_BYTES, 1024);
            const uint64_t bdesc = smem_desc_sw128(b_base + kk * UMMA_K * 128, SLAB_BYTES, 1024);
            umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          issued_any = true;
          const uint32_t e_local = smem_u32(&ctrl->empty[stage]);
          umma_commit_pair(e_local);
          umma_commit_pair(mapa_shared(e_local, 1));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (failed) break;
        const uint32_t tf_local = smem_u32(&ctrl->tfull[acc]);
        umma_commit_pair(tf_local);
        umma_commit_pair(mapa_shared(tf_local, 1));
        if (++acc == 2) {
          acc = 0;
          aphase ^= 1;
        }
      }
      if (failed) {
        record_status(wp.out.status, MOE_ERR_TIMEOUT);
        *abort_flag = 1;
        if (issued_any) {
          umma_commit_pair(smem_u32(&ctrl->drain));
          mbar_wait(smem_u32(&ctrl->drain), 0, nullptr);
        }
      }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue --
    using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
    const int quad = warp & 3;
    const int col_half = (warp - 2) >> 2;
    int q = 0, acc = 0;
    uint32_t qphase = 0, aphase = 0;
    bool failed = false;
    while (true) {
      const bool ok = mbar_wait_cluster(smem_u32(&ctrl->qfull[q]), qphase, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        failed = true;
        break;
      }
      const int4 s = ctrl->slot[q];
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->qempty[q]), 0));
      if (++q == QDEPTH) {
        q = 0;
        qphase ^= 1;
      }
      if (s.x < 0) break;
      gg::Params op = wp.out;
      op.c = reinterpret_cast<T*>(wp.out.c) + int64_t(s.x) * wp.c_stride_e;
      const int row0 = s.y + static_cast<int>(crank) * BM_CTA;
      const int rows = min(BM_CTA, max(0, wp.m - row0));
      if (s.w == 0) {
        const int r = quad * 32 + lane;
        if (r < rows) {
          const int c0 = s.z + col_half * (BN / 2);
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(op.c) + int64_t(row0 + r) * op.ldc + c0);
          for (int v = 0; v < BN / 16 && c0 + 8 * v < wp.n; ++v) dst[v] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const bool ok2 = mbar_wait_cluster(smem_u32(&ctrl->tfull[acc]), aphase, abort_flag);
      if (!__all_sync(0xffffffffu, ok2)) {
        failed = true;
        break;
      }
      tc_fence_after();
      // C[e] is stored through the 3-D {N, M, E} map, whose row extent M clips the
      // last tile's rows.
      gg::store_accumulator<BF16>(tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN), quad,
                                  lane, row0, rows, s.z, op, col_half * 4, 4,
                                  wp.out.c_tma ? &tmap_c : nullptr,
                                  smem_u32(sEpi + (warp - 2) * EPI_STAGE_BYTES), true, s.x);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->tempty[acc]), 0));
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1;
      }
    }
    if (failed && lane == 0) {
      record_status(wp.out.status, MOE_ERR_TIMEOUT);
      *abort_flag = 1;
    }
    if (lane == 0) bulk_wait_group0();  // this warp's C stores are complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // neither CTA leaves while the pair still uses its memory
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

template <bool BF16>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                  const WParams& wp, int grid, cudaStream_t stream) {
  auto kern = wgrad_pair_kernel<BF16>;
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MOE_ERR_CUDA;
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev], [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(kSmem));
  });
  if (attr_err != cudaSuccess) return MOE_ERR_CUDA;
  kern<<<grid, NUM_THREADS, kSmem, stream>>>(ta, tb, tc, wp);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace pair
}  // namespace wg
}  // namespace moe

extern "C" int32_t moe_grouped_gemm_wgrad(const void* a, int64_t lda, const void* b, int64_t ldb,
                                          void* c, int64_t ldc, int64_t c_stride_e,
                                          const void* expert_offsets, int32_t offsets_int64,
                                          int64_t rows_total, int64_t m, int64_t n,
                                          int32_t num_experts, int32_t dtype, int32_t num_sms,
                                          int32_t* status, void* stream_) {
  using namespace moe;
  using namespace moe::wg;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_F16) return MOE_ERR_INVALID_ARG;
  if (rows_total < 0 || m < 0 || n < 0 || num_experts < 0 || rows_total > INT32_MAX ||
      m > INT32_MAX || n > INT32_MAX || expert_offsets == nullptr)
    return MOE_ERR_INVALID_ARG;
  if (num_experts == 0 || m == 0 || n == 0) return MOE_OK;
  if (c == nullptr || !aligned16(c) || ldc < n || ldc % 8 != 0 || n % 8 != 0 || m % 8 != 0 ||
      c_stride_e < m * ldc || c_stride_e % 8 != 0)
    return MOE_ERR_INVALID_ARG;
  if (int64_t(num_experts) * ((m + BM - 1) / BM) * ((n + BN - 1) / BN) > INT32_MAX)
    return MOE_ERR_CAPACITY;
  if (rows_total == 0) {
    // Every expert is empty: all gradients are zero.
    return cudaMemset2DAsync(c, size_t(ldc) * 2, 0, size_t(n) * 2, size_t(m) * num_experts,
                             stream) == cudaSuccess
               ? MOE_OK
               : MOE_ERR_CUDA;
  }
  if (a == nullptr || b == nullptr || !aligned16(a) || !aligned16(b) || lda < m || ldb < n ||
      lda % 8 != 0 || ldb % 8 != 0)
    return MOE_ERR_INVALID_ARG;
  int dev = 0;
  DeviceInfo info;
  if (int rc = current_device_info(&dev, &info); rc != MOE_OK) return rc;
  if (info.major != 10) return MOE_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt =
      dtype == MOE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {uint64_t(m), uint64_t(rows_total)};
    const uint64_t strides[1] = {uint64_t(lda) * 2};
    const uint32_t box[2] = {64, BK};
    if (int rc = encode_tiled(&ta, dt, 2, a, dims, strides, box); rc != MOE_OK) return rc;
  }
  {
    const uint64_t dims[2] = {uint64_t(n), uint64_t(rows_total)};
    const uint64_t strides[1] = {uint64_t(ldb) * 2};
    const uint32_t box[2] = {64, BK};
    if (int rc = encode_tiled(&tb, dt, 2, b, dims, strides, box); rc != MOE_OK) return rc;
  }
  WParams wp{};
  wp.out.c = c;
  wp.out.ldc = ldc;
  wp.out.n = static_cast<int>(n);
  wp.out.activation = MOE_ACT_NONE;
  wp.out.status = status;
  wp.c_stride_e = c_stride_e;
  wp.offsets = expert_offsets;
  wp.offsets_int64 = offsets_int64 ? 1 : 0;
  wp.rows_total = static_cast<int>(rows_total);
  wp.m = static_cast<int>(m);
  wp.n = static_cast<int>(n);
  wp.num_experts = num_experts;
  const int grid = std::max(1, std::min<int>(num_sms > 0 ? num_sms : info.sm_count, info.sm_count));
  if (grid >= 2 && !force_single_sm_kernel()) {
    // CTA pairs: an even grid of (2,1,1) clusters; C[e] stored through a 3-D
    // {N, M, E} map in 32x32 boxes with 64-byte swizzle.
    CUtensorMap tc;
    const uint64_t dims[3] = {uint64_t(n), uint64_t(m), uint64_t(num_experts)};
    const uint64_t strides[2] = {uint64_t(ldc) * 2, uint64_t(c_stride_e) * 2};
    const uint32_t box[3] = {32, 32, 1};
    if (int rc = encode_tiled(&tc, dt, 3, c, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B); rc != MOE_OK)
      return rc;
    wp.out.c_tma = 1;
    const int pgrid = grid & ~1;
    return dtype == MOE_DTYPE_BF16 ? pair::launch<true>(ta, tb, tc, wp, pgrid, stream)
                                   : pair::launch<false>(ta, tb, tc, wp, pgrid, stream);
  }
  return dtype == MOE_DTYPE_BF16 ? launch<true>(ta, tb, wp, grid, stream)
                                 : launch<false>(ta, tb, wp, grid, stream);
}
