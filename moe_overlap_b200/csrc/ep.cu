// Expert-parallel token exchange over NVLink peer memory (sm_100a).
//
// Replaces the intranode dispatch/combine that src/deep_ep_comm.py:69-115 drives
// through DeepEP (thirdParty/DeepEP/csrc/kernels/layout.cu, intranode.cu,
// deep_ep.cpp:397-914), with a layout built for the grouped GEMM that follows:
//
//   dispatch  every (token, selected expert) pair becomes one bf16 row pushed
//             straight into the owning rank's receive buffer, at its place in
//             that rank's expert-ordered layout (local expert, then source rank,
//             then token/slot order).  The receiver gets expert_offsets on the
//             device, so recv_x feeds the grouped GEMM with no permutation and no
//             host synchronisation.
//   combine   the source rank pulls, for each of its tokens, the rows the owners
//             produced (plain loads through peer pointers) and reduces them in
//             fp32, optionally weighted by its own top-k weights, into one bf16 row.
//
// Phases (separate launches, all on one stream):
//   dispatch_begin   layout (stable per-expert ranks) + push this rank's per-expert
//                    counts into every peer + count flag            (no waiting)
//   dispatch_scatter wait for every peer's counts, derive row bases, push rows and
//                    metadata, last block raises the data flag in every peer
//   dispatch_end     wait until every peer's rows have landed here
//   combine_begin    raise "my expert outputs are ready" in every peer (no waiting)
//   combine_end      wait for every peer's ready flag, pull + reduce
// Waits are bounded (globaltimer); on expiry a kernel records MOE_ERR_TIMEOUT in the
// status word and returns.  Flags carry a monotonically increasing epoch, so they
// are never reset.  Two slots alternate between consecutive dispatches, which lets
// the next chunk's dispatch run while the previous chunk is being computed.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>

#include "../../include/moe_overlap.h"
#include "gemm_common.cuh"
#include "host_common.h"

namespace moe {
namespace ep {

constexpr int kMaxRanks = MOE_EP_MAX_RANKS;
// Experts per layer the exchange supports: its per-expert tables live in the
// scatter's shared memory, which must stay small enough to run beside the GEMM.
constexpr int kMaxExperts = 512;
constexpr int kAssignPerLayoutBlock = 2048;  // 8 warps x 8 chunks x 32 lanes
constexpr int kLayoutThreads = 256;
// The scatter and pull blocks are sized to run beside a resident CTA of the
// CTA-pair grouped GEMM (320 threads x 168 registers, ~215 KB shared memory),
// which leaves ~11.7K registers and ~17 KB of shared memory per SM: 128 threads
// at <= 64 registers and the 12 KB CountView fit, so the exchange runs during the
// expert GEMMs instead of waiting for their persistent CTAs to exit.
constexpr int kCommThreads = 128;
constexpr int kPullThreads = 128;
constexpr int kCommMinBlocks = 8;  // __launch_bounds__ minimum: caps registers at 64

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void record_status(int32_t* status, int32_t code) {
  if (status != nullptr) {
    volatile int32_t* s = status;
    if (*s == 0) *s = code;
  }
}

// Per-slot regions of the symmetric buffer, byte offsets from its base.
struct SlotLayout {
  uint64_t recv_x;     // [cap][hidden] bf16
  uint64_t y;          // [cap][hidden] bf16 (expert outputs read by combine)
  uint64_t topk_idx;   // [cap][max_topk] int64
  uint64_t topk_w;     // [cap][max_topk] float
  uint64_t src;        // [cap] int2 {src_rank, src_token}
  uint64_t dst;        // [cap] int32: the row's index in its source rank's cb (-1: padding)
  uint64_t counts;     // [world][num_experts] int32
  uint64_t cb;         // [max_tokens * max_topk][hidden] bf16: this rank's tokens' expert
                       // outputs, pushed here by their owners' GEMM epilogue, in blocks
                       // ordered by global expert, each in (token, slot) order - the
                       // order of the same rows on the owner, so runs of received rows
                       // land on consecutive cb rows
};

struct SymLayout {
  SlotLayout slot[2];
  uint64_t count_flag;  // [2][world] uint64
  uint64_t data_flag;   // [2][world] uint64
  uint64_t ready_flag;  // [2][world] uint64
  uint64_t arrived;     // [2][num_experts / world] uint32: rows of each local expert that
                        // have landed here in an expert-ordered dispatch (peers add to it)
  uint64_t bytes;
};

struct Endpoint {
  int rank, world, num_experts, per_rank, hidden, max_tokens, max_topk;
  int64_t cap_rows;
  SymLayout lay;
  uint8_t* sym = nullptr;          // this rank's symmetric buffer
  uint8_t* peers[kMaxRanks] = {};  // every rank's buffer as mapped here
  // local scratch
  uint8_t* scratch = nullptr;
  uint8_t** d_peers = nullptr;      // [world]
  int32_t* block_hist = nullptr;    // [max_blocks][E] -> exclusive block base after count
  int32_t* rank_in_block = nullptr; // [max_tokens*max_topk]
  int32_t* send_pos[2] = {};        // [max_tokens*max_topk]
  int32_t* cb_pos[2] = {};          // [max_tokens*max_topk] row of each (token, slot) in cb
  CUtensorMap* d_cb_maps = nullptr; // [2][world] TMA store maps of every rank's cb (per slot)
  int32_t* offsets[2] = {};         // [per_rank+1] receiver expert offsets
  int32_t* my_counts = nullptr;     // [E]
  int32_t* order = nullptr;         // [max_tokens] tokens in the expert-ordered sending order
  int32_t* token_key = nullptr;     // [max_tokens] sending key of each token
  int32_t* key_count = nullptr;     // [E+1] tokens per sending key
  int32_t* key_cursor = nullptr;    // [E+1] tokens placed per key
  int32_t ordered_tokens[2] = {-1, -1};  // tokens of the slot's last ordered begin, else -1
  int32_t* expected[2] = {};        // [per_rank] rows of each local expert (before alignment)
  unsigned int* done_ctr = nullptr; // blocks finished in the current scatter
  uint64_t* epoch_ctr = nullptr;    // device-side epoch counter (epoch 0 = use it)
  uint64_t* slot_epoch = nullptr;   // [2] epoch the last dispatch into each slot drew
  int max_blocks = 0;
  int64_t* host_info = nullptr;     // mapped pinned: [2][2] {epoch, total rows}
  int device = 0;
};

struct Params {
  uint8_t** peers;
  SymLayout lay;
  int rank, world, num_experts, per_rank, hidden, max_topk;
  int64_t cap_rows;
  int slot;
  uint64_t epoch;
  uint64_t wait_ns;
  int32_t* status;
  // dispatch
  const __nv_bfloat16* x;
  // FP8 payload (fp8 != 0): e4m3 rows [T, hidden] and float scales [T, hidden/128]
  // instead of x; each receive row then holds hidden bytes at recv_x + row * hidden
  // and its scales at recv_x + cap_rows * hidden + row * hidden / 32 bytes.
  const uint8_t* x8;
  const float* x_scales;
  int fp8;
  const int64_t* topk_idx;
  const float* topk_w;
  int num_tokens, topk;
  int32_t* block_hist;
  int32_t* rank_in_block;
  int32_t* send_pos;
  int32_t* cb_pos;
  int32_t* offsets_out;
  int32_t* my_counts;
  int32_t* order;        // expert-ordered dispatch: this rank's tokens in sending order
  int32_t* token_key;    // expert-ordered dispatch: sending key of each token
  int32_t* key_count;    // [E + 1] tokens per key, then
  int32_t* key_cursor;   // [E + 1] tokens placed per key
  int32_t* expected_out; // expert-ordered dispatch: rows of each local expert, for the GEMM
  int ordered;           // count phase: also build `order` and clear the arrival counters
  unsigned int* done_ctr;
  uint64_t* epoch_ctr;
  uint64_t* slot_epoch;
  int num_layout_blocks;
  int pad_rows;  // fill recv_topk_idx rows past the received count with -1
  int align;     // receive segments of each local expert rounded up to this many rows
  int scale_rows;  // multiply each pushed row by its slot's weight (bf16 result)
  int64_t* host_info;
  // cached re-dispatch: the slot whose layout the rows follow
  int src_slot;
  const int32_t* src_send_pos;
  const int32_t* src_cb_pos;
  const int32_t* src_offsets;
  // combine
  __nv_bfloat16* out;
  int weighted;
  int pushed;  // combine reads the rows the owners pushed here instead of pulling them
};

template <typename T>
__device__ __forceinline__ T* at(uint8_t* base, uint64_t off) {
  return reinterpret_cast<T*>(base + off);
}

// The kernel's slot layout, selected with constant indices (a dynamic index into
// the parameter struct would copy it to local memory).
__device__ __forceinline__ SlotLayout slot_of(const Params& p) {
  return p.slot ? p.lay.slot[1] : p.lay.slot[0];
}

// The epoch of the dispatch a kernel belongs to: the host's, or with host epoch 0
// the one that dispatch's count kernel drew from this endpoint's device counter,
// so that a captured CUDA graph replays with fresh epochs.
__device__ __forceinline__ uint64_t kernel_epoch(const Params& p) {
  return p.epoch != 0 ? p.epoch : *reinterpret_cast<const volatile uint64_t*>(p.slot_epoch + p.slot);
}

// Bounded wait until flag >= epoch.  Returns false on timeout.
__device__ __forceinline__ bool wait_flag(const uint64_t* flag, uint64_t epoch, uint64_t wait_ns) {
  if (ld_acquire_sys(flag) >= epoch) return true;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_sys(flag) < epoch) {
    if (globaltimer_ns() - t0 > wait_ns) return false;
    __nanosleep(64);
  }
  return true;
}

// ------------------------------------------------------------ layout phase --
// Per block of 2048 (token, slot) assignments: per-expert counts, and each
// assignment's rank among the block's assignments to the same expert, in
// assignment order (stable).
__global__ void __launch_bounds__(kLayoutThreads) layout_kernel(Params p) {
  extern __shared__ int warp_hist[];  // [8][E]
  const int E = p.num_experts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = p.num_tokens * p.topk;
  for (int i = threadIdx.x; i < 8 * E; i += blockDim.x) warp_hist[i] = 0;
  __syncthreads();
  const int a0 = blockIdx.x * kAssignPerLayoutBlock + warp * 256;
  int* hist = warp_hist + warp * E;
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int c = 0; c < 8; ++c) {
    const int a = a0 + c * 32 + lane;
    int e = -1;
    if (a < total) {
      const int64_t v = p.topk_idx[a];
      e = (v >= 0 && v < E) ? static_cast<int>(v) : -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int before = (e >= 0) ? hist[e] : 0;
    __syncwarp();
    if (e >= 0) {
      p.rank_in_block[a] = before + __popc(peers & lt_mask);
      if ((__ffs(peers) - 1) == lane) hist[e] = before + __popc(peers);
    }
    __syncwarp();
  }
  __syncthreads();
  int32_t* out_hist = p.block_hist + static_cast<int64_t>(blockIdx.x) * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < 8; ++w) {
      const int v = warp_hist[w * E + e];
      warp_hist[w * E + e] = run;
      run += v;
    }
    out_hist[e] = run;
  }
  __syncthreads();
  for (int c = 0; c < 8; ++c) {
    const int a = a0 + c * 32 + lane;
    if (a < total) {
      const int64_t v = p.topk_idx[a];
      if (v >= 0 && v < E) p.rank_in_block[a] += hist[v];
    }
  }
}

// One block: turn block histograms into exclusive per-block bases, total the
// per-expert counts, and publish them to every rank (row `rank` of each peer's
// count matrix for this slot), then raise this rank's count flag there.
__global__ void count_kernel(Params p) {
  const int E = p.num_experts;
  __shared__ uint64_t epoch_sh;
  if (threadIdx.x == 0) {
    uint64_t e = p.epoch;
    if (e == 0) {  // draw this dispatch's epoch on the device
      e = *p.epoch_ctr + 1;
      *p.epoch_ctr = e;
      p.slot_epoch[p.slot] = e;
    }
    epoch_sh = e;
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < p.num_layout_blocks; ++b) {
      int32_t* h = p.block_hist + static_cast<int64_t>(b) * E + e;
      const int v = *h;
      *h = run;
      run += v;
    }
    p.my_counts[e] = run;
  }
  __syncthreads();
  if (p.ordered) {
    // Expert-ordered dispatch: this rank's arrival counters for the slot start again
    // from zero, before any peer can see the count flag raised below.
    uint32_t* arrived = at<uint32_t>(p.peers[p.rank], p.lay.arrived) + p.slot * p.per_rank;
    for (int le = threadIdx.x; le < p.per_rank; le += blockDim.x) arrived[le] = 0;
    for (int i = threadIdx.x; i <= E; i += blockDim.x) {
      p.key_count[i] = 0;
      p.key_cursor[i] = 0;
    }
  }
  for (int d = 0; d < p.world; ++d) {
    int32_t* dst = at<int32_t>(p.peers[d], slot_of(p).counts) + p.rank * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) dst[e] = p.my_counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.world) {
    uint64_t* f = at<uint64_t>(p.peers[threadIdx.x], p.lay.count_flag) + p.slot * p.world + p.rank;
    st_release_sys(f, epoch_sh);
  }
}

// Expert-ordered dispatch, sending order.  A token's key is the earliest position,
// in the walk (local expert index first, then owner: e -> (e % per_rank) * W + e / per_rank),
// of the experts it was routed to; the scatter sends tokens by increasing key, so
// every token of the walk's first expert goes first, and an expert's rows are all
// sent once the tokens of its key (and of the keys before it) are.  Tokens with no
// expert get key E.  One thread per token; the per-key counts are atomics into
// arrays the count phase zeroed.
__device__ __forceinline__ int walk_key(const Params& p, int t) {
  int key = p.num_experts;
  for (int j = 0; j < p.topk; ++j) {
    const int64_t v = p.topk_idx[static_cast<int64_t>(t) * p.topk + j];
    if (v < 0 || v >= p.num_experts) continue;
    const int e = static_cast<int>(v);
    key = min(key, (e % p.per_rank) * p.world + e / p.per_rank);
  }
  return key;
}

__global__ void __launch_bounds__(256) token_key_kernel(Params p) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.num_tokens) return;
  const int key = walk_key(p, t);
  p.token_key[t] = key;
  atomicAdd(p.key_count + key, 1);
}

// Places each token at (first position of its key) + (its arrival among the key's
// tokens); the order within a key is free (it changes only when rows are sent, not
// where they land).  Each block forms the exclusive prefix of the E + 1 key counts.
__global__ void __launch_bounds__(256) token_order_kernel(Params p) {
  __shared__ int base_sh[kMaxExperts + 1];
  const int n = p.num_experts + 1;
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const int per = (n + 31) / 32;
    const int beg = min(n, lane * per), end = min(n, beg + per);
    int local = 0;
    for (int i = beg; i < end; ++i) local += p.key_count[i];
    int incl = local;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += v;
    }
    int run = incl - local;
    for (int i = beg; i < end; ++i) {
      base_sh[i] = run;
      run += p.key_count[i];
    }
  }
  __syncthreads();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.num_tokens) return;
  const int key = p.token_key[t];
  p.order[base_sh[key] + atomicAdd(p.key_cursor + key, 1)] = t;
}

__device__ __forceinline__ uint4 scale_bf16x8(const uint4& v, float s) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
  uint4 o;
  __nv_bfloat162* r = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    r[i] = __floats2bfloat162_rn(__fmul_rn(f.x, s), __fmul_rn(f.y, s));
  }
  return o;
}

// Shared state every scatter/combine block derives from the count matrix.
struct CountView {
  int exp_base[kMaxExperts];  // first row of expert e on its owner
  int my_prefix[kMaxExperts]; // rows of expert e from ranks before this one
  int exp_count[kMaxExperts]; // rows of expert e from all ranks (before alignment)
  int my_base[kMaxExperts];   // first cb row of expert e's block (this rank's rows)
  int recv_total;             // rows this rank receives
  int overflow;               // some owner would exceed its capacity
  int fail;
};

__device__ void build_count_view(const Params& p, CountView& cv) {
  const int E = p.num_experts;
  const int32_t* M = at<int32_t>(p.peers[p.rank], slot_of(p).counts);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int col = 0, before = 0;
    for (int q = 0; q < p.world; ++q) {
      const int v = M[q * E + e];
      if (q < p.rank) before += v;
      col += v;
    }
    cv.exp_base[e] = col;  // column sums for now
    cv.my_prefix[e] = before;
  }
  __syncthreads();
  if (threadIdx.x < p.world) {
    const int d = threadIdx.x;
    int run = 0;
    for (int le = 0; le < p.per_rank; ++le) {
      const int e = d * p.per_rank + le;
      const int v = cv.exp_base[e];
      cv.exp_base[e] = run;
      cv.exp_count[e] = v;
      run += (v + p.align - 1) / p.align * p.align;
    }
    if (run > p.cap_rows) atomicOr(&cv.overflow, 1);
    if (d == p.rank) cv.recv_total = run;
  }
  if (threadIdx.x == 32) {
    // This rank's cb blocks: its own rows per global expert, in expert order.
    int run = 0;
    for (int e = 0; e < E; ++e) {
      cv.my_base[e] = run;
      run += M[p.rank * E + e];
    }
  }
  __syncthreads();
}

__device__ __forceinline__ bool wait_all_flags(const Params& p, uint64_t off, int* fail) {
  if (threadIdx.x < p.world) {
    const uint64_t* f = at<uint64_t>(p.peers[p.rank], off) + p.slot * p.world + threadIdx.x;
    if (!wait_flag(f, kernel_epoch(p), p.wait_ns)) atomicOr(fail, 1);
  }
  __syncthreads();
  return *fail == 0;
}

__global__ void __launch_bounds__(kCommThreads, kCommMinBlocks) scatter_kernel(Params p) {
  __shared__ CountView cv;
  if (threadIdx.x == 0) {
    cv.overflow = 0;
    cv.fail = 0;
    cv.recv_total = 0;
  }
  __syncthreads();
  if (!wait_all_flags(p, p.lay.count_flag, &cv.fail)) {
    if (threadIdx.x == 0) record_status(p.status, MOE_ERR_TIMEOUT);
    return;
  }
  build_count_view(p, cv);
  const bool overflow = cv.overflow != 0;
  if (blockIdx.x == 0 && threadIdx.x == 0 && overflow) record_status(p.status, MOE_ERR_CAPACITY);

  const int E = p.num_experts;
  if (blockIdx.x == 0) {
    for (int le = threadIdx.x; le <= p.per_rank; le += blockDim.x) {
      const int e = p.rank * p.per_rank + le;
      p.offsets_out[le] = overflow ? 0 : (le < p.per_rank ? cv.exp_base[e] : cv.recv_total);
    }
    if (threadIdx.x == 0 && p.host_info != nullptr) {
      volatile int64_t* hi = p.host_info + 2 * p.slot;
      hi[1] = overflow ? -1 : cv.recv_total;
      __threadfence_system();
      hi[0] = static_cast<int64_t>(kernel_epoch(p));
    }
  }

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (kCommThreads / 32);
  const int nvec = p.hidden / 8;  // 16-byte vectors per row
  const SlotLayout sl = slot_of(p);
  if (!overflow) {
    for (int t = blockIdx.x * (kCommThreads / 32) + warp; t < p.num_tokens; t += warps_total) {
      const uint4* src = p.fp8 ? reinterpret_cast<const uint4*>(p.x8 + static_cast<int64_t>(t) * p.hidden)
                               : reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(t) * p.hidden);
      uint4* dst[8];
      float* dsc[8];  // FP8 payload: the row's scales on the owner
      float dscale[8];
      int nd = 0;
      for (int j = 0; j < p.topk; ++j) {
        const int a = t * p.topk + j;
        const int64_t ev = p.topk_idx[a];
        if (ev < 0 || ev >= E) {
          if (lane == 0) p.send_pos[a] = -1;
          continue;
        }
        const int e = static_cast<int>(ev);
        const int d = e / p.per_rank;
        const int blk = a / kAssignPerLayoutBlock;
        const int row = cv.exp_base[e] + cv.my_prefix[e] + p.block_hist[blk * E + e] +
                        p.rank_in_block[a];
        uint8_t* peer = p.peers[d];
        dscale[nd] = p.topk_w[a];
        if (p.fp8) {
          dsc[nd] = at<float>(peer, sl.recv_x + static_cast<uint64_t>(p.cap_rows) * p.hidden) +
                    static_cast<int64_t>(row) * (p.hidden / 128);
          dst[nd++] = at<uint4>(peer, sl.recv_x) + static_cast<int64_t>(row) * (p.hidden / 16);
        } else {
          dsc[nd] = nullptr;
          dst[nd++] = at<uint4>(peer, sl.recv_x) + static_cast<int64_t>(row) * nvec;
        }
        if (lane < p.topk) {
          at<int64_t>(peer, sl.topk_idx)[static_cast<int64_t>(row) * p.max_topk + lane] =
              (lane == j) ? static_cast<int64_t>(e - d * p.per_rank) : -1;
          at<float>(peer, sl.topk_w)[static_cast<int64_t>(row) * p.max_topk + lane] =
              (lane == j) ? p.topk_w[a] : 0.0f;
        }
        if (lane == 0) {
          // Row in this rank's cb: its block (global expert e, blocks in expert order,
          // sized by this rank's counts) plus its rank among this rank's rows for e.
          const int cb_row = cv.my_base[e] + p.block_hist[blk * E + e] + p.rank_in_block[a];
          at<int2>(peer, sl.src)[row] = make_int2(p.rank, t);
          at<int32_t>(peer, sl.dst)[row] = cb_row;
          p.send_pos[a] = row;
          p.cb_pos[a] = cb_row;
        }
      }
      if (p.fp8) {
        // e4m3 row (hidden bytes) and its hidden/128 scales, copied unchanged.
        const int nsc = p.hidden / 128;
        for (int i = lane; i < nsc; i += 32) {
          const float sc = p.x_scales[static_cast<int64_t>(t) * nsc + i];
          for (int q = 0; q < nd; ++q) dsc[q][i] = sc;
        }
      }
      const int nv_row = p.fp8 ? p.hidden / 16 : nvec;  // 16-byte vectors per payload row
      // Each lane loads 4 x 16 B per pass (2 KB of a row per warp)
      // before storing anything, so every load of the pass is in flight at once.
      constexpr int U = 4;
      for (int base = 0; base < nv_row; base += 32 * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * 32 + lane;
          if (i < nv_row) v[u] = __ldg(src + i);
        }
        for (int q = 0; q < nd; ++q) {
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int i = base + u * 32 + lane;
            if (i < nv_row) dst[q][i] = p.scale_rows ? scale_bf16x8(v[u], dscale[q]) : v[u];
          }
        }
      }
    }
    if (p.align > 1) {
      // Alignment padding inside this rank's expert segments: zero rows, no slot.
      uint8_t* me = p.peers[p.rank];
      for (int le = 0; le < p.per_rank; ++le) {
        const int e = p.rank * p.per_rank + le;
        const int64_t first = cv.exp_base[e] + cv.exp_count[e];
        const int64_t npad = (cv.exp_count[e] + p.align - 1) / p.align * p.align - cv.exp_count[e];
        for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
             i < npad * nvec; i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
          const int64_t r = first + i / nvec;
          at<uint4>(me, sl.recv_x)[r * nvec + i % nvec] = make_uint4(0, 0, 0, 0);
          if (i % nvec == 0) {
            for (int j = 0; j < p.max_topk; ++j) {
              at<int64_t>(me, sl.topk_idx)[r * p.max_topk + j] = -1;
              at<float>(me, sl.topk_w)[r * p.max_topk + j] = 0.0f;
            }
            at<int2>(me, sl.src)[r] = make_int2(-1, -1);
            at<int32_t>(me, sl.dst)[r] = -1;
          }
        }
      }
    }
    if (p.pad_rows) {
      // Rows of this rank's own receive area past the received count: no slot.
      uint8_t* me = p.peers[p.rank];
      const int64_t first = cv.recv_total;
      const int64_t n = (p.cap_rows - first) * p.max_topk;
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
           i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        at<int64_t>(me, sl.topk_idx)[first * p.max_topk + i] = -1;
        at<float>(me, sl.topk_w)[first * p.max_topk + i] = 0.0f;
      }
    }
  } else {
    for (int a = blockIdx.x * blockDim.x + threadIdx.x; a < p.num_tokens * p.topk;
         a += gridDim.x * blockDim.x)
      p.send_pos[a] = -1;
  }

  // Last block to finish tells every rank that this rank's rows have landed.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(p.done_ctr, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < p.world; ++d)
        st_release_sys(at<uint64_t>(p.peers[d], p.lay.data_flag) + p.slot * p.world + p.rank,
                       kernel_epoch(p));
    }
  }
}

// ------------------------------------------------------ expert-ordered scatter --
// The same rows, receive layout and metadata as scatter_kernel, sent in an order
// that finishes experts early, so that an owner can start multiplying an expert's
// rows as soon as they have all landed while later experts are still in flight.
// Tokens go by increasing walk key (token_key_kernel), in batches of up to 64
// tokens dealt round-robin to the blocks; a warp pushes one token's rows to all its
// owners from one load of the row, as the token-order scatter does; after each
// batch the block fences once and adds, per expert, the rows it delivered to the
// owner's arrival counter of that local expert (system-scope atomics over NVLink).  The owner's GEMM waits until a
// counter reaches that expert's row count (moe_ep_expert_gemm).
constexpr int kOrderedBatch = 64;  // tokens per lookup / fence batch of a block

__global__ void __launch_bounds__(kCommThreads, kCommMinBlocks) scatter_ordered_kernel(Params p) {
  __shared__ CountView cv;
  __shared__ int batch_tok[kOrderedBatch];
  __shared__ int batch_cnt[kMaxExperts];  // rows of each expert sent in this batch
  if (threadIdx.x == 0) {
    cv.overflow = 0;
    cv.fail = 0;
    cv.recv_total = 0;
  }
  const int E = p.num_experts;
  for (int e = threadIdx.x; e < E; e += blockDim.x) batch_cnt[e] = 0;
  __syncthreads();
  if (!wait_all_flags(p, p.lay.count_flag, &cv.fail)) {
    if (threadIdx.x == 0) record_status(p.status, MOE_ERR_TIMEOUT);
    return;
  }
  build_count_view(p, cv);
  const bool overflow = cv.overflow != 0;
  if (blockIdx.x == 0 && threadIdx.x == 0 && overflow) record_status(p.status, MOE_ERR_CAPACITY);
  if (blockIdx.x == 0) {
    for (int le = threadIdx.x; le <= p.per_rank; le += blockDim.x) {
      const int e = p.rank * p.per_rank + le;
      p.offsets_out[le] = overflow ? 0 : (le < p.per_rank ? cv.exp_base[e] : cv.recv_total);
      if (le < p.per_rank) p.expected_out[le] = overflow ? 0 : cv.exp_count[e];
    }
    if (threadIdx.x == 0 && p.host_info != nullptr) {
      volatile int64_t* hi = p.host_info + 2 * p.slot;
      hi[1] = overflow ? -1 : cv.recv_total;
      __threadfence_system();
      hi[0] = static_cast<int64_t>(kernel_epoch(p));
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = p.hidden / 8;
  const SlotLayout sl = slot_of(p);
  if (!overflow) {
    // Batches are dealt round-robin, so the grid as a whole sweeps the sending order
    // front to back and the walk's first experts complete first.  A batch is a
    // multiple of the block's warps, just large enough for every block to have one.
    constexpr int kWarps = kCommThreads / 32;
    const int per_warp = (p.num_tokens + gridDim.x * kWarps - 1) / (gridDim.x * kWarps);
    const int batch = min(kOrderedBatch, kWarps * max(1, per_warp));
    for (int tb = blockIdx.x * batch; tb < p.num_tokens; tb += gridDim.x * batch) {
      const int n = min(batch, p.num_tokens - tb);
      if (threadIdx.x < n) batch_tok[threadIdx.x] = p.order[tb + threadIdx.x];
      __syncthreads();
      for (int r = warp; r < n; r += kWarps) {
        const int t = batch_tok[r];
        if (t < 0 || t >= p.num_tokens) continue;  // the order array is the begin's, for these tokens
        const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(t) * p.hidden);
        uint4* dst[8];
        int nd = 0;
        for (int j = 0; j < p.topk; ++j) {
          const int a = t * p.topk + j;
          const int64_t ev = p.topk_idx[a];
          if (ev < 0 || ev >= E) {
            if (lane == 0) p.send_pos[a] = -1;
            continue;
          }
          const int e = static_cast<int>(ev);
          const int d = e / p.per_rank;
          const int blk = a / kAssignPerLayoutBlock;
          const int row = cv.exp_base[e] + cv.my_prefix[e] + p.block_hist[blk * E + e] +
                          p.rank_in_block[a];
          uint8_t* peer = p.peers[d];
          dst[nd++] = at<uint4>(peer, sl.recv_x) + static_cast<int64_t>(row) * nvec;
          if (lane < p.topk) {
            at<int64_t>(peer, sl.topk_idx)[static_cast<int64_t>(row) * p.max_topk + lane] =
                (lane == j) ? static_cast<int64_t>(e - d * p.per_rank) : -1;
            at<float>(peer, sl.topk_w)[static_cast<int64_t>(row) * p.max_topk + lane] =
                (lane == j) ? p.topk_w[a] : 0.0f;
          }
          if (lane == 0) {
            const int cb_row = cv.my_base[e] + p.block_hist[blk * E + e] + p.rank_in_block[a];
            at<int2>(peer, sl.src)[row] = make_int2(p.rank, t);
            at<int32_t>(peer, sl.dst)[row] = cb_row;
            p.send_pos[a] = row;
            p.cb_pos[a] = cb_row;
            atomicAdd_block(batch_cnt + e, 1);
          }
        }
        constexpr int U = 4;
        for (int base = 0; base < nvec; base += 32 * U) {
          uint4 v[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const int i = base + u * 32 + lane;
            if (i < nvec) v[u] = __ldg(src + i);
          }
          for (int q = 0; q < nd; ++q) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
              const int i = base + u * 32 + lane;
              if (i < nvec) dst[q][i] = v[u];
            }
          }
        }
      }
      // The batch's rows are visible everywhere before their owners count them.
      __threadfence_system();
      __syncthreads();
      for (int e = threadIdx.x; e < E; e += blockDim.x) {
        const int c = batch_cnt[e];
        if (c > 0) {
          const int d = e / p.per_rank;
          __threadfence_system();
          atomicAdd_system(at<unsigned int>(p.peers[d], p.lay.arrived) + p.slot * p.per_rank +
                               (e - d * p.per_rank),
                           static_cast<unsigned int>(c));
          batch_cnt[e] = 0;
        }
      }
      __syncthreads();  // the next batch reuses batch_tok and batch_cnt
    }
    if (p.pad_rows) {
      uint8_t* me = p.peers[p.rank];
      const int64_t first = cv.recv_total;
      const int64_t n = (p.cap_rows - first) * p.max_topk;
      for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
           i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        at<int64_t>(me, sl.topk_idx)[first * p.max_topk + i] = -1;
        at<float>(me, sl.topk_w)[first * p.max_topk + i] = 0.0f;
      }
    }
  } else {
    for (int a = blockIdx.x * blockDim.x + threadIdx.x; a < p.num_tokens * p.topk;
         a += gridDim.x * blockDim.x)
      p.send_pos[a] = -1;
  }
  // Last block to finish tells every rank that this rank's rows have landed.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(p.done_ctr, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < p.world; ++d)
        st_release_sys(at<uint64_t>(p.peers[d], p.lay.data_flag) + p.slot * p.world + p.rank,
                       kernel_epoch(p));
    }
  }
}

__global__ void wait_data_kernel(Params p) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!wait_all_flags(p, p.lay.data_flag, &fail) && threadIdx.x == 0)
    record_status(p.status, MOE_ERR_TIMEOUT);
}

// ------------------------------------------------------ cached re-dispatch --
// New rows for the tokens and top-k choices of the dispatch into src_slot, pushed
// to the places that dispatch gave them (its send_pos), so neither the layout nor
// the count phase runs.  What stays is the handshake that makes a slot reusable:
// a rank writes into another rank's slot only after that rank has raised its
// count flag for the new epoch, i.e. has finished everything it enqueued before.
__device__ __forceinline__ SlotLayout src_slot_of(const Params& p) {
  return p.src_slot ? p.lay.slot[1] : p.lay.slot[0];
}

__global__ void cached_begin_kernel(Params p) {
  __shared__ uint64_t epoch_sh;
  if (threadIdx.x == 0) {
    uint64_t e = p.epoch;
    if (e == 0) {  // draw this dispatch's epoch on the device
      e = *p.epoch_ctr + 1;
      *p.epoch_ctr = e;
      p.slot_epoch[p.slot] = e;
    }
    epoch_sh = e;
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.world) {
    uint64_t* f = at<uint64_t>(p.peers[threadIdx.x], p.lay.count_flag) + p.slot * p.world + p.rank;
    st_release_sys(f, epoch_sh);
  }
}

__global__ void __launch_bounds__(kCommThreads, kCommMinBlocks) cached_scatter_kernel(Params p) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!wait_all_flags(p, p.lay.count_flag, &fail)) {
    if (threadIdx.x == 0) record_status(p.status, MOE_ERR_TIMEOUT);
    return;
  }
  const SlotLayout sl = slot_of(p);
  const SlotLayout ss = src_slot_of(p);
  // This rank's receive layout is the source slot's (written by an earlier scatter
  // whose data flags this stream has already waited for).
  const int64_t recv_total =
      max(static_cast<int64_t>(0), min(static_cast<int64_t>(p.src_offsets[p.per_rank]), p.cap_rows));
  if (blockIdx.x == 0) {
    for (int le = threadIdx.x; le <= p.per_rank; le += blockDim.x) p.offsets_out[le] = p.src_offsets[le];
    if (threadIdx.x == 0 && p.host_info != nullptr) {
      const int64_t src_rows = reinterpret_cast<const volatile int64_t*>(p.host_info)[2 * p.src_slot + 1];
      volatile int64_t* hi = p.host_info + 2 * p.slot;
      hi[1] = src_rows < 0 ? -1 : recv_total;
      __threadfence_system();
      hi[0] = static_cast<int64_t>(kernel_epoch(p));
    }
  }

  const int E = p.num_experts;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (kCommThreads / 32);
  const int gwarp = blockIdx.x * (kCommThreads / 32) + warp;
  const int nvec = p.hidden / 8;
  for (int t = gwarp; t < p.num_tokens; t += warps_total) {
    const uint4* src = reinterpret_cast<const uint4*>(p.x + static_cast<int64_t>(t) * p.hidden);
    uint4* dst[8];
    float dscale[8];
    int nd = 0;
    for (int j = 0; j < p.topk; ++j) {
      const int a = t * p.topk + j;
      const int row = p.src_send_pos[a];
      const int64_t ev = p.topk_idx[a];
      if (row < 0 || row >= p.cap_rows || ev < 0 || ev >= E) {
        if (lane == 0) p.send_pos[a] = -1;
        continue;
      }
      const int d = static_cast<int>(ev) / p.per_rank;
      dscale[nd] = p.topk_w[a];
      dst[nd++] = at<uint4>(p.peers[d], sl.recv_x) + static_cast<int64_t>(row) * nvec;
      if (lane == 0) {
        p.send_pos[a] = row;
        p.cb_pos[a] = p.src_cb_pos[a];
      }
    }
    constexpr int U = 4;
    for (int base = 0; base < nvec; base += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * 32 + lane;
        if (i < nvec) v[u] = __ldg(src + i);
      }
      for (int q = 0; q < nd; ++q) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * 32 + lane;
          if (i < nvec) dst[q][i] = p.scale_rows ? scale_bf16x8(v[u], dscale[q]) : v[u];
        }
      }
    }
  }

  // This rank's receive rows: metadata from the source slot (one warp per row);
  // alignment padding rows (no source token) are zeroed in the new slot.
  uint8_t* me = p.peers[p.rank];
  for (int64_t r = gwarp; r < recv_total; r += warps_total) {
    const int2 s = at<const int2>(me, ss.src)[r];
    if (lane < p.max_topk) {
      at<int64_t>(me, sl.topk_idx)[r * p.max_topk + lane] = at<const int64_t>(me, ss.topk_idx)[r * p.max_topk + lane];
      at<float>(me, sl.topk_w)[r * p.max_topk + lane] = at<const float>(me, ss.topk_w)[r * p.max_topk + lane];
    }
    if (lane == 0) {
      at<int2>(me, sl.src)[r] = s;
      at<int32_t>(me, sl.dst)[r] = at<const int32_t>(me, ss.dst)[r];
    }
    if (s.x < 0) {
      uint4* row = at<uint4>(me, sl.recv_x) + r * nvec;
      for (int i = lane; i < nvec; i += 32) row[i] = make_uint4(0, 0, 0, 0);
    }
  }
  if (p.pad_rows) {
    const int64_t n = (p.cap_rows - recv_total) * p.max_topk;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      at<int64_t>(me, sl.topk_idx)[recv_total * p.max_topk + i] = -1;
      at<float>(me, sl.topk_w)[recv_total * p.max_topk + i] = 0.0f;
    }
  }

  // Last block to finish tells every rank that this rank's rows have landed.
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(p.done_ctr, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int d = 0; d < p.world; ++d)
        st_release_sys(at<uint64_t>(p.peers[d], p.lay.data_flag) + p.slot * p.world + p.rank,
                       kernel_epoch(p));
    }
  }
}

// ----------------------------------------------------------------- combine --
__global__ void ready_kernel(Params p) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < p.world)
    st_release_sys(at<uint64_t>(p.peers[threadIdx.x], p.lay.ready_flag) + p.slot * p.world + p.rank,
                   kernel_epoch(p));
}

__device__ __forceinline__ void acc_bf16x8(float (&acc)[8], const uint4& v, float s) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(s, f.x));
    acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(s, f.y));
  }
}

// Reduces one token: every lane first loads its U 16-byte vectors of each of
// the token's ns source rows (up to MAXR), then sums them in fp32 in slot order.
template <int U, int MAXR>
__device__ __forceinline__ void pull_token(const uint4* const* srcs, const float* scale, int ns,
                                           uint4* dst, int nvec, int lane) {
  for (int base = 0; base < nvec; base += 32 * U) {
    uint4 v[MAXR][U];
#pragma unroll
    for (int q = 0; q < MAXR; ++q) {
      if (q < ns) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * 32 + lane;
          if (i < nvec) v[q][u] = srcs[q][i];
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * 32 + lane;
      if (i >= nvec) continue;
      float acc[8];
#pragma unroll
      for (int w = 0; w < 8; ++w) acc[w] = 0.0f;
#pragma unroll
      for (int q = 0; q < MAXR; ++q)
        if (q < ns) acc_bf16x8(acc, v[q][u], scale[q]);
      uint4 o;
      __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
      for (int w = 0; w < 4; ++w) h[w] = __floats2bfloat162_rn(acc[2 * w], acc[2 * w + 1]);
      dst[i] = o;
    }
  }
}

template <int U, int MAXR>
__global__ void __launch_bounds__(kPullThreads, kCommMinBlocks) pull_kernel(Params p) {
  __shared__ int fail;
  if (threadIdx.x == 0) fail = 0;
  __syncthreads();
  if (!wait_all_flags(p, p.lay.ready_flag, &fail)) {
    if (threadIdx.x == 0) record_status(p.status, MOE_ERR_TIMEOUT);
    return;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (kPullThreads / 32);
  const int nvec = p.hidden / 8;
  const SlotLayout sl = slot_of(p);
  for (int t = blockIdx.x * (kPullThreads / 32) + warp; t < p.num_tokens; t += warps_total) {
    const uint4* srcs[MAXR];
    float scale[MAXR];
    int ns = 0;
    for (int j = 0; j < p.topk; ++j) {
      const int a = t * p.topk + j;
      const int row = p.send_pos[a];
      if (row < 0) continue;
      if (p.pushed) {
        // The owner's GEMM pushed this (token, slot) row into our combine rows.
        srcs[ns] = at<const uint4>(p.peers[p.rank], sl.cb) + static_cast<int64_t>(p.cb_pos[a]) * nvec;
      } else {
        const int64_t ev = p.topk_idx[a];
        if (ev < 0 || ev >= p.num_experts) continue;  // not the dispatch's ids: nothing to pull
        const int d = static_cast<int>(ev) / p.per_rank;
        srcs[ns] = at<const uint4>(p.peers[d], sl.y) + static_cast<int64_t>(row) * nvec;
      }
      scale[ns] = p.weighted ? p.topk_w[a] : 1.0f;
      ++ns;
    }
    uint4* dst = reinterpret_cast<uint4*>(p.out + static_cast<int64_t>(t) * p.hidden);
    pull_token<U, MAXR>(srcs, scale, ns, dst, nvec, lane);
  }
}

// d loss / d w[t][j] = <grad_out[t], y(t, j)>: the row the owner returned for
// (token t, slot j) in `slot`'s expert outputs, read through the peer pointers.
// One warp per (token, slot); fp32 dot product.
__global__ void __launch_bounds__(256) topk_weight_grad_kernel(Params p, const __nv_bfloat16* grad_out,
                                                             float* out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int warps_total = gridDim.x * (blockDim.x / 32);
  const int nvec = p.hidden / 8;
  const SlotLayout sl = slot_of(p);
  for (int a = blockIdx.x * (blockDim.x / 32) + warp; a < p.num_tokens * p.topk; a += warps_total) {
    const int t = a / p.topk;
    const int row = p.send_pos[a];
    float acc = 0.0f;
    const int64_t ev = p.topk_idx[a];
    if (row >= 0 && ev >= 0 && ev < p.num_experts) {
      const int d = static_cast<int>(ev) / p.per_rank;
      const uint4* y = at<const uint4>(p.peers[d], sl.y) + static_cast<int64_t>(row) * nvec;
      const uint4* g = reinterpret_cast<const uint4*>(grad_out + static_cast<int64_t>(t) * p.hidden);
      for (int i = lane; i < nvec; i += 32) {
        const uint4 yv = y[i], gv = g[i];
        const __nv_bfloat162* yh = reinterpret_cast<const __nv_bfloat162*>(&yv);
        const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&gv);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float2 yf = __bfloat1622float2(yh[h]), gf = __bfloat1622float2(gh[h]);
          acc = fmaf(yf.x, gf.x, acc);
          acc = fmaf(yf.y, gf.y, acc);
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    }
    if (lane == 0) out[a] = acc;
  }
}

// Tokens per rank (counted once per token) and is_token_in_rank, DeepEP's layout.
__global__ void token_rank_kernel(const int64_t* topk_idx, int num_tokens, int topk,
                                  int num_experts, int per_rank, int world, bool* is_in_rank,
                                  int32_t* tokens_per_rank) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= num_tokens) return;
  unsigned long long mask = 0;
  for (int j = 0; j < topk; ++j) {
    const int64_t e = topk_idx[static_cast<int64_t>(t) * topk + j];
    if (e >= 0 && e < num_experts) mask |= 1ull << (e / per_rank);
  }
  for (int d = 0; d < world; ++d) {
    const bool in = (mask >> d) & 1ull;
    if (is_in_rank != nullptr) is_in_rank[static_cast<int64_t>(t) * world + d] = in;
    if (in && tokens_per_rank != nullptr) atomicAdd(tokens_per_rank + d, 1);
  }
}

__global__ void expert_count_kernel(const int64_t* topk_idx, int64_t assigns, int num_experts,
                                    int32_t* tokens_per_expert) {
  const int64_t a = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (a >= assigns) return;
  const int64_t e = topk_idx[a];
  if (e >= 0 && e < num_experts) atomicAdd(tokens_per_expert + e, 1);
}

// -------------------------------------------------------------------- host --
static uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

static SymLayout plan(int world, int num_experts, int hidden, int max_topk, int64_t cap,
                      int max_tokens) {
  SymLayout L{};
  uint64_t off = 0;
  for (int s = 0; s < 2; ++s) {
    SlotLayout& sl = L.slot[s];
    sl.recv_x = off;
    off = align_up(off + uint64_t(cap) * hidden * 2, 256);
    sl.y = off;
    off = align_up(off + uint64_t(cap) * hidden * 2, 256);
    sl.topk_idx = off;
    off = align_up(off + uint64_t(cap) * max_topk * 8, 256);
    sl.topk_w = off;
    off = align_up(off + uint64_t(cap) * max_topk * 4, 256);
    sl.src = off;
    off = align_up(off + uint64_t(cap) * 8, 256);
    sl.dst = off;
    off = align_up(off + uint64_t(cap) * 4, 256);
    sl.counts = off;
    off = align_up(off + uint64_t(world) * num_experts * 4, 256);
    sl.cb = off;
    off = align_up(off + uint64_t(max_tokens) * max_topk * hidden * 2, 256);
  }
  L.count_flag = off;
  off = align_up(off + 2ull * world * 8, 256);
  L.data_flag = off;
  off = align_up(off + 2ull * world * 8, 256);
  L.ready_flag = off;
  off = align_up(off + 2ull * world * 8, 256);
  L.arrived = off;
  off = align_up(off + 2ull * (num_experts / world) * 4, 256);
  L.bytes = off;
  return L;
}

static Params base_params(const Endpoint* ep, int slot, uint64_t epoch, uint64_t wait_ns,
                          int32_t* status) {
  Params p{};
  p.peers = ep->d_peers;
  p.lay = ep->lay;
  p.rank = ep->rank;
  p.world = ep->world;
  p.num_experts = ep->num_experts;
  p.per_rank = ep->per_rank;
  p.hidden = ep->hidden;
  p.max_topk = ep->max_topk;
  p.cap_rows = ep->cap_rows;
  p.slot = slot;
  p.epoch = epoch;
  p.epoch_ctr = ep->epoch_ctr;
  p.slot_epoch = ep->slot_epoch;
  p.wait_ns = wait_ns;
  p.status = status;
  return p;
}

static int check_launch() { return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA; }

}  // namespace ep
}  // namespace moe

using moe::ep::Endpoint;
using moe::ep::Params;

struct moe_ep_s : Endpoint {};

extern "C" int32_t moe_ep_create(int32_t rank, int32_t world, int32_t num_experts, int32_t hidden,
                                 int32_t max_tokens, int32_t max_topk, int64_t max_recv_rows,
                                 moe_ep_t* out) {
  using namespace moe::ep;
  if (out == nullptr || world < 1 || world > kMaxRanks || rank < 0 || rank >= world ||
      num_experts < world || num_experts > kMaxExperts || num_experts % world != 0 ||
      hidden <= 0 || hidden % 8 != 0 || max_tokens < 0 || max_topk < 1 || max_topk > 8 ||
      max_recv_rows < 0 || max_recv_rows > INT32_MAX ||
      int64_t(max_tokens) * max_topk > INT32_MAX)
    return MOE_ERR_INVALID_ARG;
  *out = nullptr;
  moe_ep_s* ep = new (std::nothrow) moe_ep_s();
  if (ep == nullptr) return MOE_ERR_CAPACITY;
  ep->rank = rank;
  ep->world = world;
  ep->num_experts = num_experts;
  ep->per_rank = num_experts / world;
  ep->hidden = hidden;
  ep->max_tokens = max_tokens;
  ep->max_topk = max_topk;
  ep->cap_rows = max_recv_rows;
  ep->lay = plan(world, num_experts, hidden, max_topk, max_recv_rows, max_tokens);
  if (cudaGetDevice(&ep->device) != cudaSuccess) {
    delete ep;
    return MOE_ERR_CUDA;
  }
  const int64_t assigns = std::max<int64_t>(1, int64_t(max_tokens) * max_topk);
  ep->max_blocks = static_cast<int>((assigns + kAssignPerLayoutBlock - 1) / kAssignPerLayoutBlock);
  uint64_t off = 0;
  const uint64_t o_peers = off;
  off = align_up(off + sizeof(void*) * kMaxRanks, 256);
  const uint64_t o_hist = off;
  off = align_up(off + uint64_t(ep->max_blocks) * num_experts * 4, 256);
  const uint64_t o_rib = off;
  off = align_up(off + uint64_t(assigns) * 4, 256);
  uint64_t o_send[2], o_offs[2], o_cbpos[2];
  for (int s = 0; s < 2; ++s) {
    o_send[s] = off;
    off = align_up(off + uint64_t(assigns) * 4, 256);
    o_cbpos[s] = off;
    off = align_up(off + uint64_t(assigns) * 4, 256);
    o_offs[s] = off;
    off = align_up(off + uint64_t(ep->per_rank + 1) * 4, 256);
  }
  const uint64_t o_cnt = off;
  off = align_up(off + uint64_t(num_experts) * 4, 256);
  const uint64_t o_order = off;
  off = align_up(off + uint64_t(assigns) * 4, 256);
  const uint64_t o_tkey = off;
  off = align_up(off + uint64_t(std::max(1, max_tokens)) * 4, 256);
  const uint64_t o_kcount = off;
  off = align_up(off + uint64_t(num_experts + 1) * 8, 256);  // counts, then cursors
  uint64_t o_expected[2];
  for (int s = 0; s < 2; ++s) {
    o_expected[s] = off;
    off = align_up(off + uint64_t(ep->per_rank) * 4, 256);
  }
  const uint64_t o_done = off;
  off = align_up(off + 256, 256);
  const uint64_t o_maps = off;
  off = align_up(off + 2ull * world * sizeof(CUtensorMap), 256);
  if (cudaMalloc(&ep->sym, ep->lay.bytes) != cudaSuccess) {
    delete ep;
    return MOE_ERR_CUDA;
  }
  if (cudaMalloc(&ep->scratch, off) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void**>(&ep->host_info), 4 * sizeof(int64_t),
                    cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
    cudaFree(ep->sym);
    if (ep->scratch) cudaFree(ep->scratch);
    delete ep;
    return MOE_ERR_CUDA;
  }
  // Flags start at 0 (epochs start at 1); everything else is written before read.
  if (cudaMemset(ep->sym, 0, ep->lay.bytes) != cudaSuccess ||
      cudaMemset(ep->scratch, 0, off) != cudaSuccess) {
    moe_ep_destroy(ep);
    return MOE_ERR_CUDA;
  }
  std::memset(ep->host_info, 0, 4 * sizeof(int64_t));
  ep->d_peers = reinterpret_cast<uint8_t**>(ep->scratch + o_peers);
  ep->block_hist = reinterpret_cast<int32_t*>(ep->scratch + o_hist);
  ep->rank_in_block = reinterpret_cast<int32_t*>(ep->scratch + o_rib);
  ep->d_cb_maps = reinterpret_cast<CUtensorMap*>(ep->scratch + o_maps);
  for (int s = 0; s < 2; ++s) {
    ep->cb_pos[s] = reinterpret_cast<int32_t*>(ep->scratch + o_cbpos[s]);
    ep->send_pos[s] = reinterpret_cast<int32_t*>(ep->scratch + o_send[s]);
    ep->offsets[s] = reinterpret_cast<int32_t*>(ep->scratch + o_offs[s]);
  }
  ep->my_counts = reinterpret_cast<int32_t*>(ep->scratch + o_cnt);
  ep->order = reinterpret_cast<int32_t*>(ep->scratch + o_order);
  ep->token_key = reinterpret_cast<int32_t*>(ep->scratch + o_tkey);
  ep->key_count = reinterpret_cast<int32_t*>(ep->scratch + o_kcount);
  ep->key_cursor = ep->key_count + (num_experts + 1);
  for (int s = 0; s < 2; ++s) ep->expected[s] = reinterpret_cast<int32_t*>(ep->scratch + o_expected[s]);
  ep->done_ctr = reinterpret_cast<unsigned int*>(ep->scratch + o_done);
  ep->epoch_ctr = reinterpret_cast<uint64_t*>(ep->scratch + o_done + 8);
  ep->slot_epoch = reinterpret_cast<uint64_t*>(ep->scratch + o_done + 16);
  *out = ep;
  return MOE_OK;
}

namespace moe {
namespace ep {
__global__ void set_epoch_kernel(uint64_t* ctr, uint64_t epoch) { *ctr = epoch; }
}  // namespace ep
}  // namespace moe

extern "C" int32_t moe_ep_set_device_epoch(moe_ep_t ep, uint64_t epoch, void* stream) {
  if (ep == nullptr) return MOE_ERR_INVALID_ARG;
  moe::ep::set_epoch_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(ep->epoch_ctr, epoch);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int32_t moe_ep_destroy(moe_ep_t ep) {
  if (ep == nullptr) return MOE_OK;
  int rc = MOE_OK;
  if (ep->sym && cudaFree(ep->sym) != cudaSuccess) rc = MOE_ERR_CUDA;
  if (ep->scratch && cudaFree(ep->scratch) != cudaSuccess) rc = MOE_ERR_CUDA;
  if (ep->host_info && cudaFreeHost(ep->host_info) != cudaSuccess) rc = MOE_ERR_CUDA;
  delete ep;
  return rc;
}

extern "C" int32_t moe_ep_buffer(moe_ep_t ep, void** base, uint64_t* bytes) {
  if (ep == nullptr || base == nullptr || bytes == nullptr) return MOE_ERR_INVALID_ARG;
  *base = ep->sym;
  *bytes = ep->lay.bytes;
  return MOE_OK;
}

extern "C" int32_t moe_ep_connect(moe_ep_t ep, void* const* peer_bases) {
  if (ep == nullptr || peer_bases == nullptr) return MOE_ERR_INVALID_ARG;
  for (int d = 0; d < ep->world; ++d) {
    if (peer_bases[d] == nullptr) return MOE_ERR_INVALID_ARG;
    ep->peers[d] = static_cast<uint8_t*>(peer_bases[d]);
  }
  if (ep->peers[ep->rank] != ep->sym) return MOE_ERR_INVALID_ARG;
  if (cudaMemcpy(ep->d_peers, ep->peers, sizeof(void*) * ep->world, cudaMemcpyHostToDevice) !=
      cudaSuccess)
    return MOE_ERR_CUDA;
  // TMA store maps of every rank's combine rows (per slot): 32x32 bf16 boxes with
  // 64-byte swizzle, used by the fused down-projection's epilogue.
  CUtensorMap maps[2 * moe::ep::kMaxRanks];
  std::memset(maps, 0, sizeof(maps));
  const uint64_t cb_rows = uint64_t(ep->max_tokens) * ep->max_topk;
  if (cb_rows > 0) {
    for (int s = 0; s < 2; ++s)
      for (int d = 0; d < ep->world; ++d) {
        const uint64_t dims[2] = {uint64_t(ep->hidden), cb_rows};
        const uint64_t strides[1] = {uint64_t(ep->hidden) * 2};
        const uint32_t box[2] = {32, 32};
        if (int rc = moe::encode_tiled(&maps[s * ep->world + d], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                                       ep->peers[d] + ep->lay.slot[s].cb, dims, strides, box,
                                       CU_TENSOR_MAP_SWIZZLE_64B);
            rc != MOE_OK)
          return rc;
      }
  }
  return cudaMemcpy(ep->d_cb_maps, maps, sizeof(CUtensorMap) * 2 * ep->world,
                    cudaMemcpyHostToDevice) == cudaSuccess
             ? MOE_OK
             : MOE_ERR_CUDA;
}

extern "C" int32_t moe_ep_views(moe_ep_t ep, int32_t slot, moe_ep_views_t* v) {
  if (ep == nullptr || v == nullptr || slot < 0 || slot > 1) return MOE_ERR_INVALID_ARG;
  const auto& sl = ep->lay.slot[slot];
  v->recv_x = ep->sym + sl.recv_x;
  v->expert_out = ep->sym + sl.y;
  v->recv_topk_idx = reinterpret_cast<int64_t*>(ep->sym + sl.topk_idx);
  v->recv_topk_weights = reinterpret_cast<float*>(ep->sym + sl.topk_w);
  v->recv_src = reinterpret_cast<int32_t*>(ep->sym + sl.src);
  v->expert_offsets = ep->offsets[slot];
  v->send_pos = ep->send_pos[slot];
  v->host_info = ep->host_info + 2 * slot;
  v->cap_rows = ep->cap_rows;
  v->max_topk = ep->max_topk;
  v->arrived = reinterpret_cast<uint32_t*>(ep->sym + ep->lay.arrived) + slot * ep->per_rank;
  v->expected = ep->expected[slot];
  return MOE_OK;
}

static int32_t dispatch_begin_impl(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                   const float* topk_weights, int32_t num_tokens, int32_t topk,
                                   int32_t slot, uint64_t epoch, int32_t* status, void* stream_,
                                   bool ordered) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 || num_tokens < 0 ||
      num_tokens > ep->max_tokens || topk < 1 || topk > ep->max_topk ||
      (num_tokens > 0 && (x == nullptr || topk_idx == nullptr || topk_weights == nullptr)) ||
      !moe::aligned16(x))
    return MOE_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  Params p = base_params(ep, slot, epoch, 0, status);
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.topk_idx = topk_idx;
  p.topk_w = topk_weights;
  p.num_tokens = num_tokens;
  p.topk = topk;
  p.block_hist = ep->block_hist;
  p.rank_in_block = ep->rank_in_block;
  p.my_counts = ep->my_counts;
  p.order = ep->order;
  p.token_key = ep->token_key;
  p.key_count = ep->key_count;
  p.key_cursor = ep->key_cursor;
  p.ordered = ordered ? 1 : 0;
  ep->ordered_tokens[slot] = ordered ? num_tokens : -1;
  const int64_t assigns = int64_t(num_tokens) * topk;
  p.num_layout_blocks = static_cast<int>((assigns + kAssignPerLayoutBlock - 1) / kAssignPerLayoutBlock);
  if (p.num_layout_blocks > 0) {
    layout_kernel<<<p.num_layout_blocks, kLayoutThreads, 8 * ep->num_experts * sizeof(int), stream>>>(p);
    if (int rc = check_launch(); rc != MOE_OK) return rc;
  }
  count_kernel<<<1, 256, 0, stream>>>(p);
  if (int rc = check_launch(); rc != MOE_OK || !ordered || assigns == 0) return rc;
  const int tok_blocks = static_cast<int>((int64_t(num_tokens) + 255) / 256);
  if (tok_blocks == 0) return MOE_OK;
  token_key_kernel<<<tok_blocks, 256, 0, stream>>>(p);
  if (int rc = check_launch(); rc != MOE_OK) return rc;
  token_order_kernel<<<tok_blocks, 256, 0, stream>>>(p);
  return check_launch();
}

extern "C" int32_t moe_ep_dispatch_begin(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                         const float* topk_weights, int32_t num_tokens,
                                         int32_t topk, int32_t slot, uint64_t epoch,
                                         int32_t* status, void* stream) {
  return dispatch_begin_impl(ep, x, topk_idx, topk_weights, num_tokens, topk, slot, epoch, status,
                             stream, false);
}

extern "C" int32_t moe_ep_dispatch_ordered_begin(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                                 const float* topk_weights, int32_t num_tokens,
                                                 int32_t topk, int32_t slot, uint64_t epoch,
                                                 int32_t* status, void* stream) {
  return dispatch_begin_impl(ep, x, topk_idx, topk_weights, num_tokens, topk, slot, epoch, status,
                             stream, true);
}

extern "C" int32_t moe_ep_dispatch_ordered_scatter(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                                   const float* topk_weights, int32_t num_tokens,
                                                   int32_t topk, int32_t slot, uint64_t epoch,
                                                   int32_t num_blocks, int32_t pad_rows,
                                                   uint64_t wait_ns, int32_t* status, void* stream_) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 || num_tokens < 0 || num_tokens > ep->max_tokens ||
      topk < 1 || topk > ep->max_topk || num_blocks < 1 ||
      (num_tokens > 0 && (x == nullptr || topk_idx == nullptr || topk_weights == nullptr)) ||
      !moe::aligned16(x))
    return MOE_ERR_INVALID_ARG;
  // The sending order is the one the slot's ordered begin built for these tokens.
  if (ep->ordered_tokens[slot] != num_tokens) return MOE_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  Params p = base_params(ep, slot, epoch, wait_ns, status);
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.topk_idx = topk_idx;
  p.topk_w = topk_weights;
  p.num_tokens = num_tokens;
  p.topk = topk;
  p.block_hist = ep->block_hist;
  p.rank_in_block = ep->rank_in_block;
  p.send_pos = ep->send_pos[slot];
  p.cb_pos = ep->cb_pos[slot];
  p.offsets_out = ep->offsets[slot];
  p.expected_out = ep->expected[slot];
  p.order = ep->order;
  p.done_ctr = ep->done_ctr;
  p.pad_rows = pad_rows ? 1 : 0;
  p.align = 1;
  p.host_info = ep->host_info;
  if (cudaMemsetAsync(ep->done_ctr, 0, sizeof(unsigned int), stream) != cudaSuccess)
    return MOE_ERR_CUDA;
  scatter_ordered_kernel<<<num_blocks, kCommThreads, 0, stream>>>(p);
  return check_launch();
}

// The scatter phase with a bf16 payload (x) or, when x8 is set, an FP8 payload
// (e4m3 rows x8 and their per-128 scales x_scales).
static int32_t dispatch_scatter_impl(moe_ep_t ep, const void* x, bool fp8, const void* x8,
                                     const float* x_scales, const int64_t* topk_idx,
                                     const float* topk_weights, int32_t num_tokens, int32_t topk,
                                     int32_t slot, uint64_t epoch, int32_t num_blocks,
                                     int32_t pad_rows, int32_t expert_alignment,
                                     int32_t scale_rows, uint64_t wait_ns, int32_t* status,
                                     void* stream_) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 || num_tokens < 0 ||
      num_tokens > ep->max_tokens || topk < 1 || topk > ep->max_topk || num_blocks < 1 ||
      expert_alignment < 1 || expert_alignment > 4096)
    return MOE_ERR_INVALID_ARG;
  if (fp8 && (ep->hidden % 128 != 0 || expert_alignment != 1 || scale_rows ||
              (num_tokens > 0 && (x8 == nullptr || x_scales == nullptr)) || !moe::aligned16(x8) ||
              reinterpret_cast<uintptr_t>(x_scales) % 4 != 0))
    return MOE_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  Params p = base_params(ep, slot, epoch, wait_ns, status);
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.x8 = static_cast<const uint8_t*>(x8);
  p.x_scales = x_scales;
  p.fp8 = fp8 ? 1 : 0;
  p.topk_idx = topk_idx;
  p.topk_w = topk_weights;
  p.num_tokens = num_tokens;
  p.topk = topk;
  p.block_hist = ep->block_hist;
  p.rank_in_block = ep->rank_in_block;
  p.send_pos = ep->send_pos[slot];
  p.cb_pos = ep->cb_pos[slot];
  p.offsets_out = ep->offsets[slot];
  p.my_counts = ep->my_counts;
  p.done_ctr = ep->done_ctr;
  p.pad_rows = pad_rows ? 1 : 0;
  p.align = expert_alignment;
  p.scale_rows = scale_rows ? 1 : 0;
  p.host_info = ep->host_info;
  if (cudaMemsetAsync(ep->done_ctr, 0, sizeof(unsigned int), stream) != cudaSuccess)
    return MOE_ERR_CUDA;
  scatter_kernel<<<num_blocks, kCommThreads, 0, stream>>>(p);
  return check_launch();
}

extern "C" int32_t moe_ep_dispatch_scatter(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                           const float* topk_weights, int32_t num_tokens,
                                           int32_t topk, int32_t slot, uint64_t epoch,
                                           int32_t num_blocks, int32_t pad_rows,
                                           int32_t expert_alignment, int32_t scale_rows,
                                           uint64_t wait_ns, int32_t* status, void* stream) {
  return dispatch_scatter_impl(ep, x, false, nullptr, nullptr, topk_idx, topk_weights, num_tokens, topk,
                               slot, epoch, num_blocks, pad_rows, expert_alignment, scale_rows,
                               wait_ns, status, stream);
}

extern "C" int32_t moe_ep_dispatch_end(moe_ep_t ep, int32_t slot, uint64_t epoch, uint64_t wait_ns,
                                       int32_t* status, void* stream_) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1) return MOE_ERR_INVALID_ARG;
  Params p = base_params(ep, slot, epoch, wait_ns, status);
  wait_data_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream_)>>>(p);
  return check_launch();
}

extern "C" int32_t moe_ep_dispatch_cached_begin(moe_ep_t ep, int32_t slot, uint64_t epoch,
                                                void* stream_) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1) return MOE_ERR_INVALID_ARG;
  Params p = base_params(ep, slot, epoch, 0, nullptr);
  cached_begin_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream_)>>>(p);
  return check_launch();
}

extern "C" int32_t moe_ep_dispatch_cached_scatter(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                                  const float* topk_weights, int32_t num_tokens,
                                                  int32_t topk, int32_t src_slot, int32_t slot,
                                                  uint64_t epoch, int32_t num_blocks, int32_t pad_rows,
                                                  int32_t scale_rows, uint64_t wait_ns,
                                                  int32_t* status, void* stream_) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 || src_slot < 0 || src_slot > 1 || src_slot == slot ||
      num_tokens < 0 || num_tokens > ep->max_tokens || topk < 1 || topk > ep->max_topk ||
      num_blocks < 1 ||
      (num_tokens > 0 && (x == nullptr || topk_idx == nullptr || topk_weights == nullptr)) ||
      !moe::aligned16(x))
    return MOE_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  Params p = base_params(ep, slot, epoch, wait_ns, status);
  p.x = static_cast<const __nv_bfloat16*>(x);
  p.topk_idx = topk_idx;
  p.topk_w = topk_weights;
  p.num_tokens = num_tokens;
  p.topk = topk;
  p.send_pos = ep->send_pos[slot];
  p.cb_pos = ep->cb_pos[slot];
  p.offsets_out = ep->offsets[slot];
  p.done_ctr = ep->done_ctr;
  p.pad_rows = pad_rows ? 1 : 0;
  p.scale_rows = scale_rows ? 1 : 0;
  p.host_info = ep->host_info;
  p.src_slot = src_slot;
  p.src_send_pos = ep->send_pos[src_slot];
  p.src_cb_pos = ep->cb_pos[src_slot];
  p.src_offsets = ep->offsets[src_slot];
  if (cudaMemsetAsync(ep->done_ctr, 0, sizeof(unsigned int), stream) != cudaSuccess)
    return MOE_ERR_CUDA;
  cached_scatter_kernel<<<num_blocks, kCommThreads, 0, stream>>>(p);
  return check_launch();
}

extern "C" int32_t moe_ep_dispatch_cached(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                          const float* topk_weights, int32_t num_tokens, int32_t topk,
                                          int32_t src_slot, int32_t slot, uint64_t epoch,
                                          int32_t num_blocks, int32_t pad_rows, int32_t scale_rows,
                                          uint64_t wait_ns, int32_t* status, void* stream) {
  if (ep == nullptr || src_slot < 0 || src_slot > 1 || slot < 0 || slot > 1 || src_slot == slot ||
      num_tokens < 0 || num_tokens > ep->max_tokens || topk < 1 || topk > ep->max_topk ||
      num_blocks < 1 ||
      (num_tokens > 0 && (x == nullptr || topk_idx == nullptr || topk_weights == nullptr)) ||
      !moe::aligned16(x))
    return MOE_ERR_INVALID_ARG;  // checked before the begin phase raises any flag
  int rc = moe_ep_dispatch_cached_begin(ep, slot, epoch, stream);
  if (rc == MOE_OK)
    rc = moe_ep_dispatch_cached_scatter(ep, x, topk_idx, topk_weights, num_tokens, topk, src_slot,
                                        slot, epoch, num_blocks, pad_rows, scale_rows, wait_ns,
                                        status, stream);
  if (rc == MOE_OK) rc = moe_ep_dispatch_end(ep, slot, epoch, wait_ns, status, stream);
  return rc;
}

extern "C" int32_t moe_ep_combine_begin(moe_ep_t ep, int32_t slot, uint64_t epoch, void* stream_) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1) return MOE_ERR_INVALID_ARG;
  Params p = base_params(ep, slot, epoch, 0, nullptr);
  ready_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream_)>>>(p);
  return check_launch();
}

static int32_t combine_reduce(moe_ep_t ep, const int64_t* topk_idx, const float* topk_weights,
                              int32_t num_tokens, int32_t topk, int32_t slot, uint64_t epoch,
                              int32_t weighted, void* out, int32_t num_blocks, uint64_t wait_ns,
                              int32_t* status, void* stream_, int pushed) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 || num_tokens < 0 ||
      num_tokens > ep->max_tokens || topk < 1 || topk > ep->max_topk || num_blocks < 1 ||
      (num_tokens > 0 && (out == nullptr || topk_idx == nullptr)) || !moe::aligned16(out) ||
      (weighted && num_tokens > 0 && topk_weights == nullptr))
    return MOE_ERR_INVALID_ARG;
  Params p = base_params(ep, slot, epoch, wait_ns, status);
  p.topk_idx = topk_idx;
  p.topk_w = topk_weights;
  p.num_tokens = num_tokens;
  p.topk = topk;
  p.send_pos = ep->send_pos[slot];
  p.cb_pos = ep->cb_pos[slot];
  p.out = static_cast<__nv_bfloat16*>(out);
  p.weighted = weighted ? 1 : 0;
  p.pushed = pushed;
  // The pass width bounds the registers a lane needs for all of a token's rows.
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int grid = num_blocks;
  if (topk <= 2)
    pull_kernel<4, 2><<<grid, kPullThreads, 0, stream>>>(p);
  else if (topk <= 4)
    pull_kernel<2, 4><<<grid, kPullThreads, 0, stream>>>(p);
  else
    pull_kernel<1, 8><<<grid, kPullThreads, 0, stream>>>(p);
  return check_launch();
}

extern "C" int32_t moe_ep_combine_end(moe_ep_t ep, const int64_t* topk_idx,
                                      const float* topk_weights, int32_t num_tokens, int32_t topk,
                                      int32_t slot, uint64_t epoch, int32_t weighted, void* out,
                                      int32_t num_blocks, uint64_t wait_ns, int32_t* status,
                                      void* stream) {
  return combine_reduce(ep, topk_idx, topk_weights, num_tokens, topk, slot, epoch, weighted, out,
                        num_blocks, wait_ns, status, stream, 0);
}

extern "C" int32_t moe_ep_combine_pushed(moe_ep_t ep, const int64_t* topk_idx,
                                         const float* topk_weights, int32_t num_tokens,
                                         int32_t topk, int32_t slot, uint64_t epoch,
                                         int32_t weighted, void* out, int32_t num_blocks,
                                         uint64_t wait_ns, int32_t* status, void* stream) {
  return combine_reduce(ep, topk_idx, topk_weights, num_tokens, topk, slot, epoch, weighted, out,
                        num_blocks, wait_ns, status, stream, 1);
}

extern "C" int32_t moe_ep_push_gemm(moe_ep_t ep, const void* a, int64_t lda, const void* b,
                                    int64_t b_stride_e, int64_t b_stride_k, int64_t b_stride_n,
                                    int64_t m_total, int64_t k, int32_t dtype, int32_t num_sms,
                                    int32_t use_atomic_queue, int32_t* work_counter, int32_t slot,
                                    uint64_t epoch, int32_t* status, void* stream_) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 || dtype != MOE_DTYPE_BF16 || m_total < 0 ||
      m_total > ep->cap_rows)
    return MOE_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const SlotLayout& sl = ep->lay.slot[slot];
  moe::gg::PushTarget push;
  push.src = reinterpret_cast<const int2*>(ep->sym + sl.src);
  push.dst = reinterpret_cast<const int32_t*>(ep->sym + sl.dst);
  push.peers = ep->d_peers;
  push.cb = sl.cb;
  push.maps = ep->d_cb_maps + slot * ep->world;
  if (m_total > 0) {
    const int rc = moe::gg::grouped_gemm_launch(
        a, lda, b, b_stride_e, b_stride_k, b_stride_n, nullptr, ep->hidden, ep->offsets[slot], 0,
        m_total, k, ep->hidden, ep->per_rank, dtype, MOE_ACT_NONE, num_sms, use_atomic_queue,
        work_counter, nullptr, nullptr, nullptr, 0, status, stream, &push);
    if (rc != MOE_OK) return rc;
  }
  // Every owner raises its ready flag in every rank once its pushes have landed.
  Params p = base_params(ep, slot, epoch, 0, nullptr);
  ready_kernel<<<1, 64, 0, stream>>>(p);
  return check_launch();
}

extern "C" int32_t moe_ep_dispatch_ordered(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                           const float* topk_weights, int32_t num_tokens,
                                           int32_t topk, int32_t slot, uint64_t epoch,
                                           int32_t num_blocks, int32_t pad_rows, uint64_t wait_ns,
                                           int32_t* status, void* stream) {
  // Checked before the begin phase raises this rank's count flag (see moe_ep_dispatch).
  if (num_blocks < 1) return MOE_ERR_INVALID_ARG;
  int rc = moe_ep_dispatch_ordered_begin(ep, x, topk_idx, topk_weights, num_tokens, topk, slot,
                                         epoch, status, stream);
  if (rc == MOE_OK)
    rc = moe_ep_dispatch_ordered_scatter(ep, x, topk_idx, topk_weights, num_tokens, topk, slot, epoch,
                                         num_blocks, pad_rows, wait_ns, status, stream);
  if (rc == MOE_OK) rc = moe_ep_dispatch_end(ep, slot, epoch, wait_ns, status, stream);
  return rc;
}

extern "C" int32_t moe_ep_expert_gemm(moe_ep_t ep, int32_t slot, const void* b, int64_t b_stride_e,
                                      int64_t b_stride_k, int64_t b_stride_n, void* c, int64_t ldc,
                                      int64_t n, int32_t activation, int32_t num_sms,
                                      int32_t use_atomic_queue, int32_t* work_counter,
                                      uint64_t wait_ns, int32_t* status, void* stream) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 ||
      (activation != MOE_ACT_NONE && activation != MOE_ACT_GELU))
    return MOE_ERR_INVALID_ARG;
  const SymLayout& L = ep->lay;
  moe::gg::ArrivalWait arrival;
  arrival.arrived = reinterpret_cast<const uint32_t*>(ep->sym + L.arrived) + slot * ep->per_rank;
  arrival.expected = ep->expected[slot];
  arrival.wait_ns = wait_ns;
  return moe::gg::grouped_gemm_launch(
      ep->sym + L.slot[slot].recv_x, ep->hidden, b, b_stride_e, b_stride_k, b_stride_n, c, ldc,
      ep->offsets[slot], 0, ep->cap_rows, ep->hidden, n, ep->per_rank, MOE_DTYPE_BF16, activation,
      num_sms, use_atomic_queue, work_counter, nullptr, nullptr, nullptr, 0, status,
      static_cast<cudaStream_t>(stream), nullptr, &arrival);
}

extern "C" int32_t moe_ep_dispatch_layout(const int64_t* topk_idx, int32_t num_tokens,
                                          int32_t topk, int32_t num_experts, int32_t world,
                                          int32_t* tokens_per_rank, int32_t* tokens_per_expert,
                                          bool* is_token_in_rank, void* stream_) {
  using namespace moe::ep;
  if (num_tokens < 0 || topk < 1 || world < 1 || world > 64 || num_experts < world ||
      num_experts % world != 0 || (num_tokens > 0 && topk_idx == nullptr))
    return MOE_ERR_INVALID_ARG;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (tokens_per_rank && cudaMemsetAsync(tokens_per_rank, 0, world * 4, stream) != cudaSuccess)
    return MOE_ERR_CUDA;
  if (tokens_per_expert &&
      cudaMemsetAsync(tokens_per_expert, 0, num_experts * 4, stream) != cudaSuccess)
    return MOE_ERR_CUDA;
  if (num_tokens == 0) return MOE_OK;
  token_rank_kernel<<<(num_tokens + 255) / 256, 256, 0, stream>>>(
      topk_idx, num_tokens, topk, num_experts, num_experts / world, world, is_token_in_rank,
      tokens_per_rank);
  if (int rc = check_launch(); rc != MOE_OK) return rc;
  if (tokens_per_expert) {
    const int64_t assigns = int64_t(num_tokens) * topk;
    expert_count_kernel<<<static_cast<int>((assigns + 255) / 256), 256, 0, stream>>>(
        topk_idx, assigns, num_experts, tokens_per_expert);
    if (int rc = check_launch(); rc != MOE_OK) return rc;
  }
  return MOE_OK;
}

extern "C" int32_t moe_ep_dispatch(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                   const float* topk_weights, int32_t num_tokens, int32_t topk,
                                   int32_t slot, uint64_t epoch, int32_t num_blocks,
                                   int32_t pad_rows, int32_t expert_alignment, int32_t scale_rows,
                                   uint64_t wait_ns, int32_t* status, void* stream) {
  // Every argument the later phases check is checked here first: a phase that
  // fails after the begin phase has raised this rank's count flag would leave the
  // peers waiting for rows that never come.
  if (num_blocks < 1 || expert_alignment < 1 || expert_alignment > 4096)
    return MOE_ERR_INVALID_ARG;
  int rc = moe_ep_dispatch_begin(ep, x, topk_idx, topk_weights, num_tokens, topk, slot, epoch,
                                 status, stream);
  if (rc == MOE_OK)
    rc = moe_ep_dispatch_scatter(ep, x, topk_idx, topk_weights, num_tokens, topk, slot, epoch,
                                 num_blocks, pad_rows, expert_alignment, scale_rows, wait_ns,
                                 status, stream);
  if (rc == MOE_OK) rc = moe_ep_dispatch_end(ep, slot, epoch, wait_ns, status, stream);
  return rc;
}

extern "C" int32_t moe_ep_dispatch_fp8_scatter(moe_ep_t ep, const void* x_fp8, const float* x_scales,
                                               const int64_t* topk_idx, const float* topk_weights,
                                               int32_t num_tokens, int32_t topk, int32_t slot,
                                               uint64_t epoch, int32_t num_blocks, int32_t pad_rows,
                                               uint64_t wait_ns, int32_t* status, void* stream) {
  return dispatch_scatter_impl(ep, nullptr, true, x_fp8, x_scales, topk_idx, topk_weights,
                               num_tokens, topk, slot, epoch, num_blocks, pad_rows, 1, 0, wait_ns,
                               status, stream);
}

extern "C" int32_t moe_ep_dispatch_fp8(moe_ep_t ep, const void* x_fp8, const float* x_scales,
                                       const int64_t* topk_idx, const float* topk_weights,
                                       int32_t num_tokens, int32_t topk, int32_t slot,
                                       uint64_t epoch, int32_t num_blocks, int32_t pad_rows,
                                       uint64_t wait_ns, int32_t* status, void* stream) {
  // Checked before the begin phase raises this rank's count flag (see moe_ep_dispatch).
  if (ep == nullptr || num_blocks < 1 || ep->hidden % 128 != 0 ||
      (num_tokens > 0 && (x_fp8 == nullptr || x_scales == nullptr)) || !moe::aligned16(x_fp8) ||
      reinterpret_cast<uintptr_t>(x_scales) % 4 != 0)
    return MOE_ERR_INVALID_ARG;
  int rc = moe_ep_dispatch_begin(ep, x_fp8, topk_idx, topk_weights, num_tokens, topk, slot, epoch,
                                 status, stream);
  if (rc == MOE_OK)
    rc = moe_ep_dispatch_fp8_scatter(ep, x_fp8, x_scales, topk_idx, topk_weights, num_tokens, topk,
                                     slot, epoch, num_blocks, pad_rows, wait_ns, status, stream);
  if (rc == MOE_OK) rc = moe_ep_dispatch_end(ep, slot, epoch, wait_ns, status, stream);
  return rc;
}

extern "C" int32_t moe_ep_combine(moe_ep_t ep, const int64_t* topk_idx, const float* topk_weights,
                                  int32_t num_tokens, int32_t topk, int32_t slot, uint64_t epoch,
                                  int32_t weighted, void* out, int32_t num_blocks,
                                  uint64_t wait_ns, int32_t* status, void* stream) {
  int rc = moe_ep_combine_begin(ep, slot, epoch, stream);
  if (rc == MOE_OK)
    rc = moe_ep_combine_end(ep, topk_idx, topk_weights, num_tokens, topk, slot, epoch, weighted,
                            out, num_blocks, wait_ns, status, stream);
  return rc;
}

extern "C" int32_t moe_ipc_export(void* dev_ptr, void* handle_out) {
  if (dev_ptr == nullptr || handle_out == nullptr) return MOE_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, dev_ptr) != cudaSuccess) return MOE_ERR_CUDA;
  static_assert(sizeof(h) == MOE_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return MOE_OK;
}

extern "C" int32_t moe_ipc_import(const void* handle, void** dev_ptr_out) {
  if (handle == nullptr || dev_ptr_out == nullptr) return MOE_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess
             ? MOE_OK
             : MOE_ERR_CUDA;
}

extern "C" int32_t moe_ipc_close(void* dev_ptr) {
  if (dev_ptr == nullptr) return MOE_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int32_t moe_ep_topk_weight_grad(moe_ep_t ep, const void* grad_out,
                                           const int64_t* topk_idx, int32_t num_tokens,
                                           int32_t topk, int32_t slot, float* out,
                                           int32_t num_blocks, void* stream) {
  using namespace moe::ep;
  if (ep == nullptr || slot < 0 || slot > 1 || num_tokens < 0 || num_tokens > ep->max_tokens ||
      topk < 1 || topk > ep->max_topk || num_blocks < 1 ||
      (num_tokens > 0 && (grad_out == nullptr || topk_idx == nullptr || out == nullptr)) ||
      !moe::aligned16(grad_out))
    return MOE_ERR_INVALID_ARG;
  if (num_tokens == 0) return MOE_OK;
  Params p = base_params(ep, slot, 1, 0, nullptr);
  p.topk_idx = topk_idx;
  p.num_tokens = num_tokens;
  p.topk = topk;
  p.send_pos = ep->send_pos[slot];
  topk_weight_grad_kernel<<<num_blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      p, static_cast<const __nv_bfloat16*>(grad_out), out);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}
