// Grouped GEMM on CTA pairs (tcgen05 cta_group::2): 256x256 output tiles.
//
// Same contract as the 1-SM kernel in grouped_gemm.cu (C[off[e]:off[e+1]] =
// act(A[off[e]:off[e+1]] @ B[e]), fp32 accumulation), for grids of two or more
// SMs.  A (2,1,1) cluster is one CTA pair; the even CTA ("leader") owns the
// schedule and issues tcgen05.mma.cta_group::2 with M=256, N=256.  Each CTA
// TMA-loads its own 128 rows of A and its own 128 columns of B per k-block
// (32 KB per SM instead of the 48 KB a 1-SM 128x256 tile needs for the same
// tensor work), so six stages fit in shared memory, and each CTA receives its
// 128 rows of the accumulator in its own TMEM.
//
// Roles per CTA (320 threads):
//   warp 0   producer.  Leader: takes the next tile (striped over the pairs, or
//            from the global atomic counter), posts it to both CTAs' tile rings,
//            loads its halves.  Follower: reads the posted tile, loads its halves.
//            Both CTAs' loads complete on the leader's stage barrier.
//   warp 1   TMEM (both CTAs allocate the pair's 512 columns); in the leader it
//            also issues the MMAs and commits stage/accumulator completion to the
//            barriers of both CTAs.
//   warps 2-9 epilogue of this CTA's 128 rows (see store_accumulator): warp w
//            reads TMEM lanes 32*(w%4).. (the lanes its warp slot may access) and
//            columns 128*((w-2)/4).. of the tile, so two warps share each lane
//            quadrant and every SM sub-partition runs two epilogue warps.  Each
//            warp stages 32x32 bf16 chunks in its own 2 KiB of shared memory and
//            writes them with TMA bulk stores (rows inside the tile's expert only).
// Swapped tails: a tile of at most 224 rows (an expert's last rows) would leave part
// of a 256-row MMA empty.  With swap_tails such a tile is computed transposed
// instead: the 256 weight columns take the MMA's M side (128 per CTA, the same B
// stage as usual, now the MMA's A operand) and the tile's rows its N side, N the
// rows rounded up to 16 (N/2 rows from each CTA, through a 64-row map when N <= 128),
// so the tensor work follows the rows.  Each CTA's TMEM then holds its 128 output
// columns in its lanes and the tile's rows in N accumulator columns; the epilogue
// stores them transposed (plain or GELU epilogues only).
// No load uses cluster multicast; the pair exchanges only barrier arrivals and
// the tile ring entries through shared::cluster addresses.
#include <algorithm>
#include <cstdint>
#include <mutex>

#include "gemm_common.cuh"
#include "host_common.h"
#include "sched.cuh"

namespace moe {
namespace gg {
namespace pair {

constexpr int BM = 256;      // rows per pair tile
constexpr int BM_CTA = 128;  // rows per CTA
constexpr int BN = 256;
constexpr int BN_CTA = 128;  // B columns held by each CTA
constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr int STAGES = 6;
constexpr int QDEPTH = 8;
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_THREADS = 64 + 32 * NUM_EPI_WARPS;
constexpr int kMaxRegs = 144;
constexpr int A_STAGE_BYTES = BM_CTA * BK * 2;  // 16 KiB
constexpr int B_STAGE_BYTES = BK * BN_CTA * 2;  // 16 KiB
constexpr int B_SLAB_BYTES = BK * 64 * 2;       // one 64-column slab of an N-major B stage
constexpr uint32_t PAIR_TX_BYTES = 2 * (A_STAGE_BYTES + B_STAGE_BYTES);
// A swapped tile of at most 128 rows loads only the 64 rows per CTA that its MMA can read.
constexpr uint32_t PAIR_TX_BYTES_SWAPPED = 2 * (A_STAGE_BYTES / 2 + B_STAGE_BYTES);
// Tiles of at most this many rows run swapped (above it the N side would be within 32
// rows of a full tile's tensor work and its epilogue is the slower one).
constexpr int SWAP_MAX_ROWS = 224;
constexpr int EPI_STAGE_BYTES = 32 * 32 * 2;  // one 32x32 bf16 chunk per epilogue warp
constexpr uint32_t TMEM_COLS = 2 * BN;

struct Ctrl {
  uint64_t full[STAGES];   // leader: both CTAs' loads of a stage landed
  uint64_t empty[STAGES];  // each CTA: its stage buffers are free again
  uint64_t tfull[2];       // each CTA: accumulator ready
  uint64_t tempty[2];      // leader: both CTAs' epilogues drained the accumulator
  uint64_t qfull[QDEPTH];  // each CTA: tile ring entry posted
  uint64_t qempty[QDEPTH]; // leader: entry read by every consumer of both CTAs
  uint64_t drain;
  int4 slot[QDEPTH];       // {row0, rows (1..256), n0 (-1 = end), expert}
  uint32_t tmem_base;
  int abort;
};

__host__ __device__ constexpr size_t smem_bytes(int num_experts) {
  return 1024 + size_t(STAGES) * (A_STAGE_BYTES + B_STAGE_BYTES) + size_t(NUM_EPI_WARPS) * EPI_STAGE_BYTES +
         ((sizeof(Ctrl) + 15) / 16) * 16 + size_t(3) * 4 * (num_experts + 1);
}

// A tile of at most SWAP_MAX_ROWS rows (an expert's last rows) is computed swapped:
// the 256 weight columns take the MMA's M side and the tile's rows its N side, N the
// rows rounded up to 16 (the N granularity with M = 256), so the tensor work follows
// the rows.  Returns that N, or 0 for a tile computed the usual way.
__device__ __forceinline__ int swapped_n(const Params& p, int rows) {
  return (p.swap_tails && rows <= SWAP_MAX_ROWS) ? (rows + 15) & ~15 : 0;
}

// Epilogue of a swapped tile: TMEM lane (32*quad + lane) of this CTA holds output
// column n_cta + 32*quad + lane, accumulator column j the tile's row j.  The warp
// covers rows [r_first, r_end) in 32-row chunks and applies, per element, the same
// float operations in the same order as store_accumulator (row scale, derivative or
// pre-activation to aux_out, GELU or the multiply by aux_in), so a swapped tile's
// outputs equal an unswapped one's bit for bit.  Lane pairs swap values so that each
// thread stores two adjacent columns of one row (4 bytes) of C and of aux_out, and
// the 32 lanes of a warp store 64 contiguous bytes of a row per instruction.
template <bool BF16>
__device__ __forceinline__ void store_swapped(uint32_t t_lane_base, int lane, int quad, int row0,
                                              int rows, int r_first, int r_end, int n_cta,
                                              const Params& p) {
  using T = typename std::conditional<BF16, __nv_bfloat16, __half>::type;
  const int col = n_cta + quad * 32 + lane;
  const bool odd = (lane & 1) != 0;
  const int pair_col = col - (odd ? 1 : 0);  // first column of the pair this thread stores
  const bool col_ok = pair_col < p.n;        // n is a multiple of 8: col + 1 < n as well
  const int act = p.activation;
  const bool save_grad = act == MOE_ACT_GELU_SAVE_GRAD;
  const bool pre_out = !save_grad && p.aux_out != nullptr;  // aux_out = pre-activation
  const bool with_aux_out = save_grad || pre_out;
  const bool dgelu = act == MOE_ACT_DGELU || act == MOE_ACT_MUL_AUX;
  const bool aux_is_grad = act == MOE_ACT_MUL_AUX;
#pragma unroll 1
  for (int rbase = r_first; rbase < r_end && rbase < rows; rbase += 32) {  // warp-uniform
    uint32_t r[32];
    tmem_ld_32x32b_x32(t_lane_base + uint32_t(rbase), r);
    // This chunk's row scales, one row per lane, broadcast to every lane below.
    const float rs_lane = (p.row_scale != nullptr && rbase + lane < rows)
                              ? p.row_scale[int64_t(row0) + rbase + lane]
                              : 1.0f;
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      float v[2], g[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int rr_u = rbase + j + u;
        float x = __uint_as_float(r[j + u]) * __shfl_sync(0xffffffffu, rs_lane, j + u);
        g[u] = 0.0f;
        if (save_grad) {
          const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752440f));
          g[u] = cdf + x * (0.39894228040143267794f * expf(-0.5f * x * x));
          x = x * cdf;
        } else if (pre_out) {
          g[u] = x;
        }
        if (act == MOE_ACT_GELU) {
          x = gelu_erf(x);
        } else if (dgelu) {
          float f = 0.0f;
          if (col < p.n && rr_u < rows) {
            const T h = reinterpret_cast<const T*>(p.aux_in)[(int64_t(row0) + rr_u) * p.ld_aux + col];
            if constexpr (BF16)
              f = __bfloat162float(h);
            else
              f = __half2float(h);
          }
          x *= aux_is_grad ? f : gelu_erf_grad(f);
        }
        v[u] = x;
      }
      // even lane: row j, columns (col, col+1); odd lane: row j+1, columns (col-1, col)
      const int rr = rbase + j + (odd ? 1 : 0);
      const bool store = col_ok && rr < rows;
      const float theirs = __shfl_xor_sync(0xffffffffu, odd ? v[0] : v[1], 1);
      const uint32_t packed = odd ? pack2<BF16>(theirs, v[1]) : pack2<BF16>(v[0], theirs);
      if (store)
        *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.c) + (int64_t(row0) + rr) * p.ldc +
                                     pair_col) = packed;
      if (with_aux_out) {  // warp-uniform
        const float gtheirs = __shfl_xor_sync(0xffffffffu, odd ? g[0] : g[1], 1);
        const uint32_t gpacked = odd ? pack2<BF16>(gtheirs, g[1]) : pack2<BF16>(g[0], gtheirs);
        if (store)
          *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.aux_out) + (int64_t(row0) + rr) * p.ld_aux +
                                       pair_col) = gpacked;
      }
    }
  }
}

// The MMA issuer's k-block loop for one tile (leader CTA, one thread): waits for
// each stage's data, issues its four 16-deep MMAs into the accumulator at d_tmem
// and commits the stage back to both CTAs' producers.  SWAPPED issues the swapped
// form (B stage as the MMA's A operand with M = 256, the A stage's first N/2 rows
// as its B operand, N and the operand layouts in idesc_sw).  Returns false when a
// wait gave up.
template <bool BF16, bool B_MN_MAJOR, bool SWAPPED>
__device__ __forceinline__ bool issue_tile(Ctrl* ctrl, uint8_t* sA, uint8_t* sB, uint32_t d_tmem,
                                           int num_kb, int& stage, uint32_t& phase,
                                           const volatile int* abort_flag, bool& issued_any,
                                           uint32_t idesc_sw) {
  const uint32_t idesc = SWAPPED ? idesc_sw : idesc_f16(BF16, BM, BN, false, B_MN_MAJOR);
  // This thread's loop is on the critical path and shares its SM sub-partition with
  // two epilogue warps, so every per-stage quantity is formed once per tile and
  // advanced by constants: the descriptors of stage s differ from stage 0's only in
  // the start address (bits 0-13, in 16-byte units), the stage barriers are 8 bytes
  // apart, and mapa keeps offsets within the peer CTA's shared window.  The four
  // 16-deep steps of a stage add +32 bytes along a K-major row, or +16 rows of 128
  // bytes down an MN-major slab.  Shared memory ends below 2^18 bytes, so the
  // start-address field never carries into the next one.
  const uint64_t adesc_s0 = smem_desc_sw128(smem_u32(sA), 16, 1024);
  const uint64_t bdesc_s0 = B_MN_MAJOR ? smem_desc_sw128(smem_u32(sB), B_SLAB_BYTES, 1024)
                                       : smem_desc_sw128(smem_u32(sB), 16, 1024);
  const uint32_t full_s0 = smem_u32(&ctrl->full[0]);
  const uint32_t empty_s0 = smem_u32(&ctrl->empty[0]);
  const uint32_t empty_peer_s0 = mapa_shared(empty_s0, 1);
  for (int kb = 0; kb < num_kb; ++kb) {
    if (!mbar_wait_cluster(full_s0 + 8u * uint32_t(stage), phase, abort_flag)) return false;
    tc_fence_after();
    const uint64_t adesc0 = adesc_s0 + uint64_t(uint32_t(stage) * (A_STAGE_BYTES >> 4));
    const uint64_t bdesc0 = bdesc_s0 + uint64_t(uint32_t(stage) * (B_STAGE_BYTES >> 4));
#pragma unroll
    for (int kk = 0; kk < BK / UMMA_K; ++kk) {
      const uint64_t adesc = adesc0 + uint64_t(kk * (UMMA_K * 2 / 16));
      const uint64_t bdesc = bdesc0 + uint64_t(B_MN_MAJOR ? kk * (UMMA_K * 128 / 16) : kk * (UMMA_K * 2 / 16));
      if constexpr (SWAPPED)
        umma_f16_pair(d_tmem, bdesc, adesc, idesc, (kb | kk) != 0 ? 1u : 0u);
      else
        umma_f16_pair(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
    }
    issued_any = true;
    umma_commit_pair(empty_s0 + 8u * uint32_t(stage));
    umma_commit_pair(empty_peer_s0 + 8u * uint32_t(stage));
    if (++stage == STAGES) {
      stage = 0;
      phase ^= 1;
    }
  }
  return true;
}

// 144 registers: with 10 warps, SM sub-partitions 0 and 1 hold three of them
// (3 x 32 x 144 = 13,824 of their 16,384 registers), which leaves room for one
// warp per sub-partition of a 4-warp exchange block at <= 80 registers, so the
// dispatch/combine kernels run beside this persistent kernel.  PUSH compiles the
// expert-parallel combine push into the epilogue (rows go to their source ranks).
template <bool BF16, bool B_MN_MAJOR, bool PUSH>
__global__ void __cluster_dims__(2, 1, 1) __maxnreg__(kMaxRegs)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmap_a,
                             const __grid_constant__ CUtensorMap tmap_a_half,
                             const __grid_constant__ CUtensorMap tmap_b,
                             const __grid_constant__ CUtensorMap tmap_c, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint8_t* sEpi = sB + STAGES * B_STAGE_BYTES;  // 1024-aligned, EPI_STAGE_BYTES per epilogue warp
  Ctrl* ctrl = reinterpret_cast<Ctrl*>(sEpi + NUM_EPI_WARPS * EPI_STAGE_BYTES);
  int* tile_prefix = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(ctrl) +
                                            ((sizeof(Ctrl) + 15) / 16) * 16);
  int* seg_start = tile_prefix + (p.num_experts + 1);
  int* seg_rows = seg_start + (p.num_experts + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = lane_id();
  const uint32_t crank = cluster_ctarank();
  const bool leader = crank == 0;
  const int tiles_n = (p.n + BN - 1) / BN;

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
  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_a);
      tma_prefetch_desc(&tmap_a_half);
      tma_prefetch_desc(&tmap_b);
    }
    build_tile_prefix(p.offsets, p.offsets_int64, p.num_experts, p.m_total, BM, tiles_n,
                      tile_prefix, seg_start, seg_rows, leader ? p.status : nullptr);
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
  const int total_tiles = tile_prefix[p.num_experts];
  const int num_kb = (p.k + BK - 1) / BK;
  volatile int* abort_flag = &ctrl->abort;

  if (total_tiles == 0) {
    zero_output<BF16>(p, NUM_THREADS);
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer --
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int q = 0;
      uint32_t qphase = 0;
      int ready_expert = -1;
      bool failed = false;
      const int pair_id = static_cast<int>(cluster_id_x());
      const int npairs = static_cast<int>(nclusters_x());
      for (int iter = 0;; ++iter) {
        int4 s;
        if (leader) {
          const int t = p.use_atomic ? atomicAdd(p.work_counter, 1) : pair_id + iter * npairs;
          if (!mbar_wait_cluster(smem_u32(&ctrl->qempty[q]), qphase ^ 1, abort_flag)) {
            failed = true;
            break;
          }
          if (t >= total_tiles || t < 0) {
            s = make_int4(0, 0, -1, 0);
          } else {
            const TileCoord tc = decode_tile(t, p.num_experts, tile_prefix, seg_start, seg_rows,
                                             BM, tiles_n, p.tile_order);
            s = make_int4(tc.row0, tc.rows, tc.tile_n * BN, tc.expert);
          }
          ctrl->slot[q] = s;
          st_shared_cluster_v4(mapa_shared(smem_u32(&ctrl->slot[q]), 1), s);
          mbar_arrive(smem_u32(&ctrl->qfull[q]));
          mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->qfull[q]), 1));
        } else {
          if (!mbar_wait_cluster(smem_u32(&ctrl->qfull[q]), qphase, abort_flag)) {
            failed = true;
            break;
          }
          s = ctrl->slot[q];
          mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->qempty[q]), 0));
        }
        if (++q == QDEPTH) {
          q = 0;
          qphase ^= 1;
        }
        if (s.z < 0) break;
        if (s.w != ready_expert) {  // expert-ordered dispatch: this expert's rows have landed
          if (!wait_expert_rows(p, s.w)) {
            failed = true;
            break;
          }
          ready_expert = s.w;
        }
        // A swapped tile of N rows takes N/2 of them from each CTA (the MMA's N side),
        // CTA c from row c*N/2, through the 64-row map into the first half of the A
        // stage when N/2 <= 64, else through the usual 128-row map; the MMA reads only
        // the first N/2 rows of each stage.
        const int n_sw = swapped_n(p, s.y);
        const bool half_box = n_sw > 0 && n_sw <= BM_CTA;
        const int row_a = s.x + static_cast<int>(crank) * (n_sw > 0 ? n_sw / 2 : BM_CTA);
        const CUtensorMap* map_a = half_box ? &tmap_a_half : &tmap_a;
        const uint32_t stage_tx = half_box ? PAIR_TX_BYTES_SWAPPED : PAIR_TX_BYTES;
        const int n_b = s.z + static_cast<int>(crank) * BN_CTA;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait_cluster(smem_u32(&ctrl->empty[stage]), phase ^ 1, abort_flag)) {
            failed = true;
            break;
          }
          const uint32_t full_local = smem_u32(&ctrl->full[stage]);
          if (leader) mbar_arrive_expect_tx(full_local, stage_tx);
          const uint32_t full_leader = mapa_shared(full_local, 0);
          tma_load_2d_pair(smem_u32(sA + stage * A_STAGE_BYTES), map_a, full_leader, kb * BK, row_a);
          const uint32_t b_dst = smem_u32(sB + stage * B_STAGE_BYTES);
          if constexpr (B_MN_MAJOR) {
#pragma unroll
            for (int j = 0; j < BN_CTA / 64; ++j)
              tma_load_3d_pair(b_dst + j * B_SLAB_BYTES, &tmap_b, full_leader, n_b + 64 * j, kb * BK,
                               s.w);
          } else {
            tma_load_3d_pair(b_dst, &tmap_b, full_leader, kb * BK, n_b, s.w);
          }
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
        // Give loads already issued time to land before this CTA can leave.
        const long long t0 = clock64();
        while (clock64() - t0 < (1ll << 22)) {
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------- MMA (leader only) --
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int q = 0;
      uint32_t qphase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool failed = false;
      bool issued_any = false;
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
        if (s.z < 0) break;
        if (!mbar_wait_cluster(smem_u32(&ctrl->tempty[acc]), aphase ^ 1, abort_flag)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + uint32_t(acc * BN);
        const int n_sw = swapped_n(p, s.y);
        // Two instantiations of the k-block loop, so that the usual tile's loop
        // carries no per-MMA choice between the two operand arrangements.
        const bool ok =
            n_sw > 0 ? issue_tile<BF16, B_MN_MAJOR, true>(ctrl, sA, sB, d_tmem, num_kb, stage, phase,
                                                          abort_flag, issued_any,
                                                          idesc_f16(BF16, BM, n_sw, B_MN_MAJOR, false))
                     : issue_tile<BF16, B_MN_MAJOR, false>(ctrl, sA, sB, d_tmem, num_kb, stage, phase,
                                                           abort_flag, issued_any, 0u);
        if (!ok) failed = true;
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
        record_status(p.status, MOE_ERR_TIMEOUT);
        *abort_flag = 1;
        if (issued_any) {
          umma_commit_pair(smem_u32(&ctrl->drain));
          mbar_wait(smem_u32(&ctrl->drain), 0, nullptr);
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue --
    const int quad = warp & 3;
    const int col_half = (warp - 2) >> 2;  // 0 or 1: which 128 columns of the tile
    int q = 0;
    uint32_t qphase = 0;
    int acc = 0;
    uint32_t aphase = 0;
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
      if (s.z < 0) break;
      const bool ok2 = mbar_wait_cluster(smem_u32(&ctrl->tfull[acc]), aphase, abort_flag);
      if (!__all_sync(0xffffffffu, ok2)) {
        failed = true;
        break;
      }
      tc_fence_after();
      const int n_sw = PUSH ? 0 : swapped_n(p, s.y);
      if (n_sw > 0) {
        // The two warps of a lane quadrant split the tile's rows in 32-row chunks.
        const int half = ((n_sw / 2) + 31) & ~31;
        store_swapped<BF16>(tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN), lane, quad,
                            s.x, s.y, col_half * half, col_half * half + half,
                            s.z + static_cast<int>(crank) * BN_CTA, p);
      } else {
      const int rows_here = min(int(BM_CTA), max(0, s.y - static_cast<int>(crank) * int(BM_CTA)));
      store_accumulator<BF16, PUSH>(tmem_base + (uint32_t(quad * 32) << 16) + uint32_t(acc * BN), quad,
                              lane, s.x + static_cast<int>(crank) * BM_CTA, rows_here, s.z, p,
                              col_half * 4, 4, p.c_tma ? &tmap_c : nullptr,
                              smem_u32(sEpi + (warp - 2) * EPI_STAGE_BYTES));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->tempty[acc]), 0));
      if (++acc == 2) {
        acc = 0;
        aphase ^= 1;
      }
    }
    if (failed && lane == 0) {
      record_status(p.status, MOE_ERR_TIMEOUT);
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

template <bool BF16, bool B_MN, bool PUSH = false>
int launch(const CUtensorMap& ta, const CUtensorMap& ta_half, const CUtensorMap& tb,
           const CUtensorMap& tc, const Params& p, int grid, cudaStream_t stream) {
  auto kern = grouped_gemm_pair_kernel<BF16, B_MN, PUSH>;
  static std::once_flag once[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MOE_ERR_CUDA;
  cudaError_t attr_err = cudaSuccess;
  std::call_once(once[dev], [&] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem_bytes(kMaxExperts)));
  });
  if (attr_err != cudaSuccess) return MOE_ERR_CUDA;
  kern<<<grid, NUM_THREADS, smem_bytes(p.num_experts), stream>>>(ta, ta_half, tb, tc, p);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

}  // namespace pair

int launch_pair_kernel(bool bf16, bool b_mn, const CUtensorMap& ta, const CUtensorMap& ta_half,
                       const CUtensorMap& tb, const CUtensorMap& tc, const Params& p, int grid,
                       cudaStream_t stream) {
  if (grid < 2 || grid % 2 != 0) return MOE_ERR_INVALID_ARG;
  if (p.push.src != nullptr) {  // combine push (bf16 only)
    if (!bf16) return MOE_ERR_INVALID_ARG;
    return b_mn ? pair::launch<true, true, true>(ta, ta_half, tb, tc, p, grid, stream)
                : pair::launch<true, false, true>(ta, ta_half, tb, tc, p, grid, stream);
  }
  if (bf16 && b_mn) return pair::launch<true, true>(ta, ta_half, tb, tc, p, grid, stream);
  if (bf16 && !b_mn) return pair::launch<true, false>(ta, ta_half, tb, tc, p, grid, stream);
  if (!bf16 && b_mn) return pair::launch<false, true>(ta, ta_half, tb, tc, p, grid, stream);
  return pair::launch<false, false>(ta, ta_half, tb, tc, p, grid, stream);
}

}  // namespace gg
}  // namespace moe
