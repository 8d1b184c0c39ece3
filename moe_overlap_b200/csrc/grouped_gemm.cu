// Persistent grouped GEMM for MoE experts on sm_100a (tcgen05 + TMEM + TMA).
//
// Computes, for every expert e, C[off[e]:off[e+1]] = act(A[off[e]:off[e+1]] @ B[e])
// with an fp32 accumulator, the operation of persistent_grouped_gemm and its
// _gemm_tile device function (src/triton_grouped_gemm.py:36-98, 326-443).
//
// One CTA per SM, 192 threads, warp-specialised:
//   warp 0      tile scheduler + TMA producer (one lane): takes the next tile
//               (striped over the grid, or from a global atomic counter), posts
//               it to a small shared-memory ring, then streams the tile's A and
//               B k-blocks into a STAGES-deep ring of 128B-swizzled buffers.
//   warp 1      TMEM owner + MMA issuer (one lane): tcgen05.mma 128x256x16 into
//               one of two TMEM accumulators; tcgen05.commit frees smem stages
//               and hands a finished accumulator to the epilogue.
//   warps 2..5  epilogue: tcgen05.ld TMEM -> registers, optional exact GELU,
//               round to bf16/fp16, masked 16-byte stores of the rows that
//               belong to the tile's expert.  Two accumulators let the epilogue
//               of tile i overlap the main loop of tile i+1.
//
// The tile list is built on the device from expert_offsets (per-expert tile
// counts + prefix sum in shared memory, binary search per tile), so there is no
// host synchronisation and no host-built work queue as in _build_work_queue
// (src/triton_grouped_gemm.py:240-297).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <cstdlib>
#include <mutex>

#include "../../include/moe_overlap.h"
#include "gemm_common.cuh"
#include "host_common.h"
#include "ptx.cuh"
#include "sched.cuh"

namespace moe {
namespace gg {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one 128B swizzle row
constexpr int UMMA_K = 16;
constexpr int STAGES = 4;
constexpr int QDEPTH = 8;
constexpr int NUM_THREADS = 192;
constexpr int NUM_EPI_WARPS = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;    // 16 KiB
constexpr int B_STAGE_BYTES = BK * BN * 2;    // 32 KiB
constexpr int B_NCHUNK_BYTES = BK * 64 * 2;   // one 64-column slab of an N-major B stage
constexpr uint32_t TMEM_COLS = 2 * BN;        // two fp32 accumulators of 128 x 256
constexpr int MAX_EXPERTS = kMaxExperts;

struct Ctrl {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t qfull[QDEPTH];
  uint64_t qempty[QDEPTH];
  uint64_t drain;
  int4 slot[QDEPTH];  // {row0, valid_rows, n0 (-1 = no more tiles), expert}
  uint32_t tmem_base;
  int abort;
};

__host__ __device__ constexpr size_t smem_bytes(int num_experts) {
  return 1024 /* alignment slack */ + size_t(STAGES) * (A_STAGE_BYTES + B_STAGE_BYTES) +
         ((sizeof(Ctrl) + 15) / 16) * 16 + size_t(3) * 4 * (num_experts + 1);
}

template <bool BF16, bool B_MN_MAJOR>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(sB + STAGES * B_STAGE_BYTES);
  int* tile_prefix = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ctrl) +
                                            ((sizeof(Ctrl) + 15) / 16) * 16);
  int* seg_start = tile_prefix + (p.num_experts + 1);
  int* seg_rows = seg_start + (p.num_experts + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = lane_id();
  const int tiles_n = (p.n + BN - 1) / BN;

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
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_b);
    }
    build_tile_prefix(p.offsets, p.offsets_int64, p.num_experts, p.m_total, BM, tiles_n,
                      tile_prefix, seg_start, seg_rows, p.status);
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
  const int total_tiles = tile_prefix[p.num_experts];
  const int num_kb = (p.k + BK - 1) / BK;
  volatile int* abort_flag = &ctrl->abort;

  if (total_tiles == 0) {
    // No expert owns a row: the result is all zeros (src/triton_grouped_gemm.py:369-371).
    zero_output<BF16>(p, NUM_THREADS);
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int q = 0;
      uint32_t qphase = 0;
      int issued[STAGES] = {0, 0, 0, 0};
      int ready_expert = -1;  // rows of this expert are known to have landed
      bool failed = false;
      for (int iter = 0;; ++iter) {
        const int t = p.use_atomic ? atomicAdd(p.work_counter, 1)
                                   : static_cast<int>(blockIdx.x) + iter * static_cast<int>(gridDim.x);
        if (!mbar_wait(smem_u32(&ctrl->qempty[q]), qphase ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        if (t >= total_tiles || t < 0) {
          ctrl->slot[q] = make_int4(0, 0, -1, 0);
          mbar_arrive(smem_u32(&ctrl->qfull[q]));
          break;
        }
        TileCoord tc = decode_tile(t, p.num_experts, tile_prefix, seg_start, seg_rows, BM, tiles_n,
                                   p.tile_order);
        const int n0 = tc.tile_n * BN;
        ctrl->slot[q] = make_int4(tc.row0, tc.rows, n0, tc.expert);
        mbar_arrive(smem_u32(&ctrl->qfull[q]));
        if (++q == QDEPTH) {
          q = 0;
          qphase ^= 1;
        }
        if (tc.expert != ready_expert) {
          if (!wait_expert_rows(p, tc.expert)) {
            failed = true;
            break;
          }
          ready_expert = tc.expert;
        }
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&ctrl->empty[stage]), phase ^ 1, abort_flag)) {
            failed = true;
            break;
          }
          const uint32_t fb = smem_u32(&ctrl->full[stage]);
          mbar_arrive_expect_tx(fb, A_STAGE_BYTES + B_STAGE_BYTES);
          tma_load_2d(smem_u32(sA + stage * A_STAGE_BYTES), &tmap_a, fb, kb * BK, tc.row0);
          const uint32_t b_dst = smem_u32(sB + stage * B_STAGE_BYTES);
          if constexpr (B_MN_MAJOR) {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(b_dst + j * B_NCHUNK_BYTES, &tmap_b, fb, n0 + 64 * j, kb * BK, tc.expert);
          } else {
            tma_load_3d(b_dst, &tmap_b, fb, kb * BK, n0, tc.expert);
          }
          ++issued[stage];
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (failed) break;
      }
      if (failed) {
        record_status(p.status, MOE_ERR_TIMEOUT);
        *abort_flag = 1;
        // Let every TMA load this CTA issued land before the CTA exits.
        for (int s = 0; s < STAGES; ++s)
          if (issued[s] > 0)
            mbar_wait(smem_u32(&ctrl->full[s]), uint32_t((issued[s] - 1) & 1), nullptr);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer --
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(BF16, BM, BN, false, B_MN_MAJOR);
      int stage = 0;
      uint32_t phase = 0;
      int q = 0;
      uint32_t qphase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool failed = false;
      bool issued_any = false;
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
        if (s.z < 0) break;
        if (!mbar_wait(smem_u32(&ctrl->tempty[acc]), aphase ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(smem_u32(&ctrl->full[stage]), phase, abort_flag)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            // A: K-major, 128B swizzle; a 16-element k step is +32 bytes inside the swizzle row.
            const uint64_t adesc = smem_desc_sw128(a_base + kk * UMMA_K * 2, 16, 1024);
            uint64_t bdesc;
            if constexpr (B_MN_MAJOR) {
              // B: N-major; 64-column slabs BK*128 bytes apart (LBO), 8-row k groups
              // 1024 bytes apart (SBO); a 16-row k step is +2048 bytes.
              bdesc = smem_desc_sw128(b_base + kk * UMMA_K * 128, B_NCHUNK_BYTES, 1024);
            } else {
              bdesc = smem_desc_sw128(b_base + kk * UMMA_K * 2, 16, 1024);
            }
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
        record_status(p.status, MOE_ERR_TIMEOUT);
        *abort_flag = 1;
        if (issued_any) {
          // Wait for every MMA this thread issued before TMEM is released.
          umma_commit(smem_u32(&ctrl->drain));
          mbar_wait(smem_u32(&ctrl->drain), 0, nullptr);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    const int quad = warp & 3;  // TMEM lanes this warp may read: [32*quad, 32*quad+32)
    int q = 0;
    uint32_t qphase = 0;
    int acc = 0;
    uint32_t aphase = 0;
    bool failed = false;
    while (true) {
      if (!warp_wait(smem_u32(&ctrl->qfull[q]), qphase, abort_flag)) {
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
      if (s.z < 0) break;
      if (!warp_wait(smem_u32(&ctrl->tfull[acc]), aphase, abort_flag)) {
        failed = true;
        break;
      }
      tc_fence_after();
      if (p.push.src != nullptr)
        store_accumulator<BF16, true>(tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN),
                                      quad, lane, s.x, s.y, s.z, p);
      else
        store_accumulator<BF16>(tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN), quad,
                                lane, s.x, s.y, s.z, p);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->tempty[acc]));
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1;
      }
    }
    if (failed && lane == 0) {
      record_status(p.status, MOE_ERR_TIMEOUT);
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

// ------------------------------------------------------------------- host --
// MOE_B200_GEMM_KERNEL=1 forces the 1-SM kernel, =2 (default) the CTA-pair kernel.
static int gemm_kernel_choice() {
  static const int v = [] {
    const char* e = std::getenv("MOE_B200_GEMM_KERNEL");
    return e ? std::atoi(e) : 2;
  }();
  return v;
}

// MOE_B200_GEMM_TMA_STORE=0 makes the pair kernel write C with direct 16-byte
// stores instead of staged TMA bulk stores (default 1).
static bool gemm_tma_store() {
  static const bool v = [] {
    const char* e = std::getenv("MOE_B200_GEMM_TMA_STORE");
    return e == nullptr || std::atoi(e) != 0;
  }();
  return v;
}

// MOE_B200_GEMM_SWAP=0 computes every tile of the CTA-pair kernel as 256 rows
// (default 1: tiles of at most 224 rows run swapped, see grouped_gemm_pair.cu).
static bool gemm_swap_tails() {
  static const bool v = [] {
    const char* e = std::getenv("MOE_B200_GEMM_SWAP");
    return e == nullptr || std::atoi(e) != 0;
  }();
  return v;
}

// Tile walk order: 0 (default) = the reference's expert, tile_m, tile_n fastest
// (measured ~1 % faster on BASELINE configs 2/3 than 1 = expert, tile_n, tile_m
// fastest).  MOE_B200_GEMM_ORDER overrides.
static int gemm_tile_order() {
  static const int v = [] {
    const char* e = std::getenv("MOE_B200_GEMM_ORDER");
    return (e && std::atoi(e) == 1) ? 1 : 0;
  }();
  return v;
}

template <bool BF16, bool B_MN>
static int launch(const CUtensorMap& ta, const CUtensorMap& tb, const Params& p, int grid,
                  cudaStream_t stream) {
  auto kern = grouped_gemm_kernel<BF16, B_MN>;
  const size_t smem = smem_bytes(p.num_experts);
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MOE_ERR_CUDA;
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev], [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem_bytes(MAX_EXPERTS)));
  });
  if (attr_err != cudaSuccess) return MOE_ERR_CUDA;
  kern<<<grid, NUM_THREADS, smem, stream>>>(ta, tb, p);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace gg
}  // namespace moe

using namespace moe;

int moe::gg::grouped_gemm_launch(const void* a, int64_t lda, const void* b, int64_t b_stride_e,
                                 int64_t b_stride_k, int64_t b_stride_n, void* c, int64_t ldc,
                                 const void* expert_offsets, int32_t offsets_int64, int64_t m_total,
                                 int64_t k, int64_t n, int32_t num_experts, int32_t dtype,
                                 int32_t activation, int32_t num_sms, int32_t use_atomic_queue,
                                 int32_t* work_counter, const float* row_scale, const void* aux_in,
                                 void* aux_out, int64_t ld_aux, int32_t* status, cudaStream_t stream,
                                 const PushTarget* push, const ArrivalWait* arrival) {
  using namespace moe::gg;
  const bool pushing = push != nullptr && push->src != nullptr;
  if (dtype != MOE_DTYPE_BF16 && dtype != MOE_DTYPE_F16) return MOE_ERR_INVALID_ARG;
  if (activation < MOE_ACT_NONE || activation > MOE_ACT_MUL_AUX) return MOE_ERR_INVALID_ARG;
  if ((activation == MOE_ACT_DGELU || activation == MOE_ACT_MUL_AUX) && aux_in == nullptr)
    return MOE_ERR_INVALID_ARG;
  if (activation == MOE_ACT_GELU_SAVE_GRAD && aux_out == nullptr) return MOE_ERR_INVALID_ARG;
  if ((aux_in != nullptr || aux_out != nullptr) &&
      (ld_aux < n || ld_aux % 8 != 0 || (aux_in && !aligned16(aux_in)) ||
       (aux_out && !aligned16(aux_out))))
    return MOE_ERR_INVALID_ARG;
  if (m_total < 0 || k < 0 || n < 0 || num_experts < 0) return MOE_ERR_INVALID_ARG;
  if (m_total > INT32_MAX || k > INT32_MAX || n > INT32_MAX) return MOE_ERR_INVALID_ARG;
  if (num_experts > MAX_EXPERTS) return MOE_ERR_UNSUPPORTED;
  if (expert_offsets == nullptr) return MOE_ERR_INVALID_ARG;
  if (m_total == 0 || n == 0) return MOE_OK;
  if (pushing) {
    // Combine push: rows go to the source ranks' combine rows (stride ldc), not C.
    if (push->dst == nullptr || push->peers == nullptr || ldc < n || ldc % 8 != 0 ||
        n % 8 != 0 || k == 0 || num_experts == 0 || aux_out != nullptr ||
        activation == MOE_ACT_GELU_SAVE_GRAD)
      return MOE_ERR_INVALID_ARG;
  } else if (c == nullptr || !aligned16(c) || ldc < n || ldc % 8 != 0 || n % 8 != 0) {
    return MOE_ERR_INVALID_ARG;
  }
  if (k == 0 || num_experts == 0) {
    // Empty contraction or no experts: every computed row is zero, and with no
    // experts at all the reference zero-fills the whole output.
    return cudaMemset2DAsync(c, size_t(ldc) * 2, 0, size_t(n) * 2, size_t(m_total), stream) ==
                   cudaSuccess
               ? MOE_OK
               : MOE_ERR_CUDA;
  }
  if (a == nullptr || b == nullptr || !aligned16(a) || !aligned16(b)) return MOE_ERR_INVALID_ARG;
  if (k % 8 != 0 || lda < k || lda % 8 != 0) return MOE_ERR_INVALID_ARG;
  const bool b_mn = (b_stride_n == 1);
  const bool b_kmaj = (!b_mn && b_stride_k == 1);
  if (!b_mn && !b_kmaj) return MOE_ERR_INVALID_ARG;
  const int64_t b_inner_stride = b_mn ? b_stride_k : b_stride_n;
  if (b_inner_stride % 8 != 0 || b_inner_stride <= 0) return MOE_ERR_INVALID_ARG;
  if (num_experts > 1 && (b_stride_e % 8 != 0 || b_stride_e <= 0)) return MOE_ERR_INVALID_ARG;
  if (use_atomic_queue && work_counter == nullptr) return MOE_ERR_INVALID_ARG;

  int dev = 0;
  DeviceInfo info;
  if (int rc = current_device_info(&dev, &info); rc != MOE_OK) return rc;
  if (info.major != 10) return MOE_ERR_UNSUPPORTED;

  // Grids of two or more SMs run the CTA-pair kernel (256x256 tiles, grid
  // rounded down to even); a single SM runs the 1-SM kernel (128x256 tiles).
  int grid = std::max(1, std::min<int>(num_sms > 0 ? num_sms : info.sm_count, info.sm_count));
  const bool use_pair = grid >= 2 && gemm_kernel_choice() != 1;
  if (use_pair) grid &= ~1;
  const CUtensorMapDataType dt =
      dtype == MOE_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ta, ta_half, tb;
  {
    const uint64_t dims[2] = {uint64_t(k), uint64_t(m_total)};
    const uint64_t strides[1] = {uint64_t(lda) * 2};
    const uint32_t box[2] = {BK, BM};
    if (int rc = encode_tiled(&ta, dt, 2, a, dims, strides, box); rc != MOE_OK) return rc;
    const uint32_t box_half[2] = {BK, BM / 2};  // the <= 64 rows a swapped tile of N <= 128 reads per CTA
    if (int rc = encode_tiled(&ta_half, dt, 2, a, dims, strides, box_half); rc != MOE_OK) return rc;
  }
  {
    const int64_t se = num_experts > 1 ? b_stride_e : b_inner_stride * (b_mn ? k : n);
    if (b_mn) {
      const uint64_t dims[3] = {uint64_t(n), uint64_t(k), uint64_t(num_experts)};
      const uint64_t strides[2] = {uint64_t(b_stride_k) * 2, uint64_t(se) * 2};
      const uint32_t box[3] = {64, BK, 1};
      if (int rc = encode_tiled(&tb, dt, 3, b, dims, strides, box); rc != MOE_OK) return rc;
    } else {
      const uint64_t dims[3] = {uint64_t(k), uint64_t(n), uint64_t(num_experts)};
      const uint64_t strides[2] = {uint64_t(b_stride_n) * 2, uint64_t(se) * 2};
      const uint32_t box[3] = {BK, use_pair ? uint32_t(BN / 2) : uint32_t(BN), 1};
      if (int rc = encode_tiled(&tb, dt, 3, b, dims, strides, box); rc != MOE_OK) return rc;
    }
  }

  Params p;
  p.c = c;
  p.ldc = ldc;
  p.offsets = expert_offsets;
  p.offsets_int64 = offsets_int64 ? 1 : 0;
  p.m_total = static_cast<int>(m_total);
  p.k = static_cast<int>(k);
  p.n = static_cast<int>(n);
  p.num_experts = num_experts;
  p.activation = activation;
  p.use_atomic = use_atomic_queue ? 1 : 0;
  p.tile_order = gemm_tile_order();
  p.work_counter = work_counter;
  p.status = status;
  p.row_scale = row_scale;
  p.aux_in = aux_in;
  p.aux_out = aux_out;
  p.ld_aux = ld_aux;
  p.push = pushing ? *push : PushTarget{nullptr, nullptr, nullptr, 0, nullptr};
  p.arrival = arrival != nullptr ? *arrival : ArrivalWait{nullptr, nullptr, 0};
  // Tiles of at most 224 rows (an expert's tail) run swapped on the CTA pair with
  // every epilogue but the combine push, whose rows go to their source ranks.
  p.swap_tails = use_pair && gemm_swap_tails() && !pushing;

  // The pair kernel stores C through a {N, m_total} map in 32x32 boxes (64-byte swizzle).
  CUtensorMap tc;
  std::memset(&tc, 0, sizeof(tc));
  p.c_tma = 0;
  if (use_pair && gemm_tma_store() && !pushing) {
    const uint64_t dims[2] = {uint64_t(n), uint64_t(m_total)};
    const uint64_t strides[1] = {uint64_t(ldc) * 2};
    const uint32_t box[2] = {32, 32};
    if (int rc = encode_tiled(&tc, dt, 2, c, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_64B); rc != MOE_OK)
      return rc;
    p.c_tma = 1;
  }

  if (p.use_atomic &&
      cudaMemsetAsync(work_counter, 0, sizeof(int32_t), stream) != cudaSuccess)
    return MOE_ERR_CUDA;
  const bool bf16 = dtype == MOE_DTYPE_BF16;
  if (use_pair) return launch_pair_kernel(bf16, b_mn, ta, ta_half, tb, tc, p, grid, stream);
  if (bf16 && b_mn) return launch<true, true>(ta, tb, p, grid, stream);
  if (bf16 && !b_mn) return launch<true, false>(ta, tb, p, grid, stream);
  if (!bf16 && b_mn) return launch<false, true>(ta, tb, p, grid, stream);
  return launch<false, false>(ta, tb, p, grid, stream);
}

extern "C" int32_t moe_grouped_gemm_ex(const void* a, int64_t lda, const void* b,
                                       int64_t b_stride_e, int64_t b_stride_k, int64_t b_stride_n,
                                       void* c, int64_t ldc, const void* expert_offsets,
                                       int32_t offsets_int64, int64_t m_total, int64_t k,
                                       int64_t n, int32_t num_experts, int32_t dtype,
                                       int32_t activation, int32_t num_sms,
                                       int32_t use_atomic_queue, int32_t* work_counter,
                                       const float* row_scale, const void* aux_in, void* aux_out,
                                       int64_t ld_aux, int32_t* status, void* stream) {
  return moe::gg::grouped_gemm_launch(a, lda, b, b_stride_e, b_stride_k, b_stride_n, c, ldc,
                                      expert_offsets, offsets_int64, m_total, k, n, num_experts,
                                      dtype, activation, num_sms, use_atomic_queue, work_counter,
                                      row_scale, aux_in, aux_out, ld_aux, status,
                                      static_cast<cudaStream_t>(stream), nullptr);
}

extern "C" int32_t moe_grouped_gemm(const void* a, int64_t lda, const void* b, int64_t b_stride_e,
                                    int64_t b_stride_k, int64_t b_stride_n, void* c, int64_t ldc,
                                    const void* expert_offsets, int32_t offsets_int64,
                                    int64_t m_total, int64_t k, int64_t n, int32_t num_experts,
                                    int32_t dtype, int32_t activation, int32_t num_sms,
                                    int32_t use_atomic_queue, int32_t* work_counter,
                                    int32_t* status, void* stream) {
  // the activations with auxiliary operands need moe_grouped_gemm_ex
  if (activation != MOE_ACT_NONE && activation != MOE_ACT_GELU) return MOE_ERR_INVALID_ARG;
  return moe_grouped_gemm_ex(a, lda, b, b_stride_e, b_stride_k, b_stride_n, c, ldc,
                             expert_offsets, offsets_int64, m_total, k, n, num_experts, dtype,
                             activation, num_sms, use_atomic_queue, work_counter, nullptr,
                             nullptr, nullptr, 0, status, stream);
}
