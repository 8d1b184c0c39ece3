/*
 * moe_overlap.h - C ABI of the B200 (sm_100a) MoE expert hot path.
 *
 * Every entry point takes plain device pointers, element counts/strides and a
 * CUDA stream handle (cudaStream_t passed as void*; NULL = legacy default
 * stream).  Nothing here allocates device memory except where stated; all
 * work is enqueued asynchronously on `stream` and the functions return as soon
 * as it is queued.
 *
 * Return value: MOE_OK (0) or one of the MOE_ERR_* codes below for argument
 * or launch errors found on the host.  Errors found on the device while a
 * kernel runs (bounded wait expired, offsets out of range) are written to the
 * optional `status` word (int32, device memory or mapped pinned host memory,
 * zero-initialised by the caller); a nonzero value there is one of the same
 * codes.
 */
#ifndef MOE_OVERLAP_H_
#define MOE_OVERLAP_H_

#include <stdbool.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MOE_API __attribute__((visibility("default")))
#else
#define MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status -- */
#define MOE_OK 0
#define MOE_ERR_INVALID_ARG 1  /* bad shape / dtype / pointer / alignment   */
#define MOE_ERR_CUDA 2         /* a CUDA runtime/driver call failed         */
#define MOE_ERR_TIMEOUT 3      /* a bounded device-side wait ran out        */
#define MOE_ERR_OFFSETS 4      /* expert_offsets point outside [0, m_total] */
#define MOE_ERR_UNSUPPORTED 5  /* device is not sm_100 / feature missing    */
#define MOE_ERR_CAPACITY 6     /* a fixed-capacity buffer would overflow    */

/* ----------------------------------------------------------------- dtypes -- */
#define MOE_DTYPE_BF16 0
#define MOE_DTYPE_F16 1
#define MOE_DTYPE_F32 2 /* router logits only */

/* ------------------------------------------------------------ activations -- */
#define MOE_ACT_NONE 0
#define MOE_ACT_GELU 1  /* exact GELU, 0.5*x*(1+erf(x/sqrt(2))), on the fp32 accumulator */
#define MOE_ACT_DGELU 2 /* acc * gelu'(aux_in): the GELU backward fused into a dgrad GEMM  */
#define MOE_ACT_GELU_SAVE_GRAD 3 /* GELU(acc); aux_out receives gelu'(acc) instead of acc      */
#define MOE_ACT_MUL_AUX 4        /* acc * aux_in: the backward against a saved gelu'           */

/* Human-readable text for a status code (static storage). */
MOE_API const char* moe_status_string(int32_t code);

/* ABI version of this library, MOE_ABI_VERSION. */
#define MOE_ABI_VERSION 1
MOE_API int32_t moe_abi_version(void);

/*
 * Grouped GEMM over ragged expert segments.
 *
 * Replaces persistent_grouped_gemm (src/triton_grouped_gemm.py:326-443) and
 * the two Triton kernels it launches (_persistent_grouped_gemm_kernel_striped,
 * :101-154, and _persistent_grouped_gemm_kernel_atomic, :157-233), including
 * the work list that _build_work_queue (:240-297) builds on the host side:
 * here the tile list is derived on the device from expert_offsets.
 *
 * For every expert e in [0, num_experts):
 *   C[off[e]:off[e+1], :] = act( A[off[e]:off[e+1], :] @ B[e] )
 * with fp32 accumulation and the result rounded to `dtype`.  Rows outside
 * every expert segment are left untouched, except that when no expert has a
 * row at all, the whole of C is zero-filled (src/triton_grouped_gemm.py:369-371).
 *
 *   a               A, m_total x k, row stride lda elements, unit column stride
 *   b               B, num_experts x k x n; element (e,kk,nn) at
 *                   b + e*b_stride_e + kk*b_stride_k + nn*b_stride_n.
 *                   Either b_stride_n == 1 (N-major, the reference layout) or
 *                   b_stride_k == 1 (K-major, i.e. a transposed weight view).
 *   c               C, m_total x n, row stride ldc elements
 *   expert_offsets  num_experts+1 ints (int32, or int64 if offsets_int64)
 *   dtype           MOE_DTYPE_BF16 or MOE_DTYPE_F16 (A, B and C share it)
 *   activation      MOE_ACT_NONE or MOE_ACT_GELU
 *   num_sms         persistent grid size (clamped to the device's SM count)
 *   use_atomic_queue 0: tiles striped over the grid; 1: dynamic tile queue
 *   work_counter    int32 device scratch word for the dynamic queue; required
 *                   when use_atomic_queue != 0, zeroed on `stream` by this call
 *   status          optional device-visible int32 error word (may be NULL)
 *   stream          cudaStream_t
 *
 * Alignment: a, b, c 16-byte aligned; lda, ldc and the non-unit B strides
 * multiples of 8 elements; k and n multiples of 8.
 */
MOE_API int32_t moe_grouped_gemm(const void* a, int64_t lda, const void* b, int64_t b_stride_e,
                         int64_t b_stride_k, int64_t b_stride_n, void* c, int64_t ldc,
                         const void* expert_offsets, int32_t offsets_int64, int64_t m_total,
                         int64_t k, int64_t n, int32_t num_experts, int32_t dtype,
                         int32_t activation, int32_t num_sms, int32_t use_atomic_queue,
                         int32_t* work_counter, int32_t* status, void* stream);

/*
 * moe_grouped_gemm with optional epilogue operands (any may be NULL / 0):
 *   row_scale  float[m_total]: v = acc * row_scale[row]
 *   aux_out    m_total x n (row stride ld_aux), dtype: receives v before the
 *              activation (the pre-activation a backward pass needs)
 *   aux_in     m_total x n (row stride ld_aux), dtype: with activation
 *              MOE_ACT_DGELU the result is v * gelu'(aux_in), the GELU backward
 *              fused into a dgrad GEMM
 * Two more activations split that work between the passes: MOE_ACT_GELU_SAVE_GRAD
 * writes C = GELU(v) and aux_out = gelu'(v) (required), both from one erf of v, and
 * MOE_ACT_MUL_AUX writes C = v * aux_in (required), so the backward epilogue
 * multiplies instead of evaluating erf and exp again.
 * then C = act(v) as in moe_grouped_gemm.  No counterpart in the reference, which
 * runs inference only (src/train_moe_baseline.py:524-552); these serve the
 * forward-with-saved-activations and backward of the routed experts.
 */
MOE_API int32_t moe_grouped_gemm_ex(const void* a, int64_t lda, const void* b, int64_t b_stride_e,
                                    int64_t b_stride_k, int64_t b_stride_n, void* c, int64_t ldc,
                                    const void* expert_offsets, int32_t offsets_int64,
                                    int64_t m_total, int64_t k, int64_t n, int32_t num_experts,
                                    int32_t dtype, int32_t activation, int32_t num_sms,
                                    int32_t use_atomic_queue, int32_t* work_counter,
                                    const float* row_scale, const void* aux_in, void* aux_out,
                                    int64_t ld_aux, int32_t* status, void* stream);

/*
 * Weight-gradient grouped GEMM: for every expert e with rows r in
 * [off[e], off[e+1]) of A (rows_total x m, row stride lda) and B (rows_total x n,
 * row stride ldb):  C[e] (m x n, row stride ldc, expert stride c_stride_e) =
 * sum_r A[r]^T B[r], fp32 accumulation rounded to dtype.  Every segment must
 * start and end on a multiple of 64 rows (see expert_alignment of the exchange;
 * otherwise MOE_ERR_OFFSETS); an expert without rows gets zeros.  With A = dY and
 * B = H (or A = dA, B = X) of the routed experts this is dW2 (dW1) in nn.Linear
 * layout.  No counterpart in the reference, which has no backward pass.
 */
MOE_API int32_t moe_grouped_gemm_wgrad(const void* a, int64_t lda, const void* b, int64_t ldb,
                                       void* c, int64_t ldc, int64_t c_stride_e,
                                       const void* expert_offsets, int32_t offsets_int64,
                                       int64_t rows_total, int64_t m, int64_t n,
                                       int32_t num_experts, int32_t dtype, int32_t num_sms,
                                       int32_t* status, void* stream);

/*
 * Allocation-free variant of moe_grouped_gemm with the dynamic (atomic) tile
 * queue.  It has no counterpart in the reference; it exists for callers that
 * cannot allocate device memory: code running under a host framework whose
 * memory pool owns the GPU and forbids raw cudaMalloc/cudaFree beside it, and
 * latency-critical loops where an allocation could synchronise the device.
 *
 * Same arguments and result as moe_grouped_gemm with use_atomic_queue = 1,
 * minus work_counter: the queue counter lives in a 256-byte device array inside
 * this library (one per GPU, kept until the process exits).  The caller still
 * passes every input and output.  The call allocates nothing and calls no
 * allocating routine.
 *
 * Limit: the tile count of one call, bounded above by
 * (ceil(m_total/128) + num_experts) * ceil(n/256), must stay below about
 * 2^31 - 4096; larger problems are refused with MOE_ERR_CAPACITY.
 * Set-up: the first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current; make that first call before
 * any stream capture.  A failed lookup returns MOE_ERR_CUDA and is retried by
 * the next call on that device.
 * Sharing: every call on a device uses the same counter, which keeps what the
 * last call left and is re-zeroed on `stream` at the start of each call.  Calls
 * that overlap on the GPU (e.g. on two streams at once) race on it and must be
 * serialised by the caller.
 */
MOE_API int32_t moe_grouped_gemm_noalloc(const void* a, int64_t lda, const void* b,
                                         int64_t b_stride_e, int64_t b_stride_k,
                                         int64_t b_stride_n, void* c, int64_t ldc,
                                         const void* expert_offsets, int32_t offsets_int64,
                                         int64_t m_total, int64_t k, int64_t n,
                                         int32_t num_experts, int32_t dtype, int32_t activation,
                                         int32_t num_sms, int32_t* status, void* stream);

/*
 * Decodes the grouped-GEMM tile list on the device, exactly as the GEMM
 * kernel's scheduler does, for inspection and testing.
 *
 * Replaces _build_work_queue (src/triton_grouped_gemm.py:240-297).  With
 * order == 0 the list is expert-major, then tile_m, then tile_n (the
 * reference's order, :277-286), the order the GEMM kernel walks by default;
 * order == 1 is expert-major, then tile_n, then tile_m (CTAs sharing a weight
 * column block adjacent).  Writes up to max_items entries to out_expert /
 * out_tile_m / out_tile_n (int32 device arrays) and the total count to
 * *out_count (int32 device word).
 */
MOE_API int32_t moe_tile_list(const void* expert_offsets, int32_t offsets_int64, int32_t num_experts,
                      int64_t m_total, int64_t n, int32_t block_m, int32_t block_n, int32_t order,
                      int32_t* out_expert, int32_t* out_tile_m, int32_t* out_tile_n,
                      int32_t max_items, int32_t* out_count, int32_t* status, void* stream);

/*
 * offsets[0] = 0, offsets[i+1] = offsets[i] + counts[i], accumulated in 64-bit
 * and stored as int32 (offsets_int64 == 0, wrapping like a two's-complement
 * cast) or int64.
 *
 * Replaces expert_offsets_from_recv_counts (src/triton_grouped_gemm.py:300-323)
 * for device-resident counts.  counts is int32 (counts_int64 == 0) or int64;
 * an int64 count is narrowed to int32 before it is added, as the reference's
 * .to(torch.int32) does.
 */
MOE_API int32_t moe_expert_offsets(const void* counts, int32_t counts_int64, int32_t num_experts,
                           void* offsets, int32_t offsets_int64, void* stream);

/*
 * Same as moe_expert_offsets for host-resident counts and offsets; runs on the
 * calling thread.  Serves expert_offsets_from_recv_counts
 * (src/triton_grouped_gemm.py:300-323) when the counts are a Python list or a
 * CPU tensor and no device is requested, where the reference returns a CPU tensor.
 */
MOE_API int32_t moe_expert_offsets_host(const void* counts, int32_t counts_int64, int32_t num_experts,
                                void* offsets, int32_t offsets_int64);

/* ================================================ expert-parallel exchange == */
/*
 * Token dispatch/combine between the GPUs of one NVLink/NVSwitch domain.
 * Replaces DeepEPDispatcher (src/deep_ep_comm.py:21-115) and the DeepEP
 * intranode runtime under it (thirdParty/DeepEP/csrc/deep_ep.cpp:131-914,
 * kernels/layout.cu, kernels/intranode.cu, kernels/runtime.cu).
 *
 * Each rank owns an endpoint with one symmetric device buffer (allocated by
 * moe_ep_create).  The host exchanges the buffers between ranks (e.g. CUDA IPC
 * handles gathered over the process group, as deep_ep.cpp:185-199 and
 * buffer.py:96-101 do) and hands every rank's base pointer, as mapped on this
 * GPU, to moe_ep_connect.  Experts are sharded contiguously, num_experts/world
 * per rank (src/train_moe_baseline.py:136-137).
 *
 * Receive layout: one row per (token, selected expert) on the expert's owner,
 * ordered by local expert, then source rank, then (token, slot); the owner gets
 * expert_offsets on the device.  Two slots alternate between consecutive
 * dispatches; at most two dispatches may be outstanding (not yet combined).
 * Every call takes an `epoch` (1, 2, 3, ... in call order, the same on every
 * rank) and a `slot` (the epoch's parity, by convention).  Epoch 0 means "draw
 * it on the device": the dispatch's first kernel takes the endpoint's device
 * counter + 1 and every later kernel of that dispatch and of its combine reads
 * it, so a captured CUDA graph replays with fresh epochs.  Set the counter to the
 * last host epoch with moe_ep_set_device_epoch before the first such call, keep
 * the host's slot alternation, and capture an even number of dispatches so that
 * every replay leaves the slot parity unchanged.
 */
#define MOE_EP_MAX_RANKS 64

typedef struct moe_ep_s* moe_ep_t;

/* Device pointers into this rank's endpoint for one slot. */
typedef struct {
  void* recv_x;               /* [cap_rows][hidden] bf16, expert-ordered rows      */
  void* expert_out;           /* [cap_rows][hidden] bf16, rows read by combine     */
  int64_t* recv_topk_idx;     /* [cap_rows][max_topk]: local expert in the row's slot, else -1 */
  float* recv_topk_weights;   /* [cap_rows][max_topk]: weight in the row's slot, else 0 */
  int32_t* recv_src;          /* [cap_rows][2]: {source rank, source token}        */
  int32_t* expert_offsets;    /* [num_experts/world + 1] int32, on the device      */
  int32_t* send_pos;          /* [max_tokens][topk] row of each sent (token, slot) on its owner, -1 none */
  int64_t* host_info;         /* mapped host [2]: {epoch, rows received} after scatter */
  int64_t cap_rows;
  int32_t max_topk;
  uint32_t* arrived;          /* [num_experts/world] rows of each local expert landed in an
                                 expert-ordered dispatch (peers add to it)            */
  int32_t* expected;          /* [num_experts/world] rows of each local expert expected  */
} moe_ep_views_t;

/* Allocates this rank's endpoint: a symmetric buffer holding two slots of
 * max_recv_rows received rows (plus expert outputs, metadata, counts, flags, and
 * max_tokens * max_topk combine rows for the fused push), and local scratch for
 * max_tokens tokens of up to max_topk experts each.  Limits: world <= 64,
 * num_experts <= 512 and divisible by world, max_topk <= 8, hidden % 8 == 0. */
MOE_API int32_t moe_ep_create(int32_t rank, int32_t world, int32_t num_experts, int32_t hidden,
                              int32_t max_tokens, int32_t max_topk, int64_t max_recv_rows,
                              moe_ep_t* out);
MOE_API int32_t moe_ep_destroy(moe_ep_t ep);
/* Base pointer and size of this rank's symmetric buffer (to export to peers). */
MOE_API int32_t moe_ep_buffer(moe_ep_t ep, void** base, uint64_t* bytes);
/* peer_bases[r] = rank r's symmetric buffer as addressable from this GPU
 * (peer_bases[rank] must be this endpoint's own buffer). */
MOE_API int32_t moe_ep_connect(moe_ep_t ep, void* const* peer_bases);
MOE_API int32_t moe_ep_views(moe_ep_t ep, int32_t slot, moe_ep_views_t* views);

/*
 * Dispatch, in three phases enqueued on `stream` (moe_ep_dispatch runs all three):
 *   begin    per-expert counts of this rank's (token, slot) pairs, pushed into every
 *            rank (no waiting);                         ~ layout.cu + notify_dispatch
 *   scatter  waits (bounded by wait_ns) for every rank's counts, then pushes each
 *            selected token's bf16 row and its metadata into the owner's receive
 *            slot and raises this rank's data flag everywhere; pad_rows != 0 also
 *            sets recv_topk_idx = -1 for this rank's unused receive rows;
 *            expert_alignment (>= 1, DeepEP's argument of that name,
 *            deep_ep/buffer.py:327) rounds every local expert's segment up to a
 *            multiple of that many rows; the padding rows are zeroed with no slot;
 *            scale_rows != 0 pushes each row multiplied by its slot's weight
 *            (rounded to bf16), e.g. the weighted output gradient of a backward;
 *                                                       ~ intranode.cu dispatch
 *   end      waits (bounded) until every rank's rows have landed here.
 * x: [num_tokens][hidden] bf16; topk_idx: [num_tokens][topk] int64 global expert ids
 * (-1 = none); topk_weights: [num_tokens][topk] float.  num_blocks is the grid of
 * the scatter (the SM budget of the exchange).  Device errors go to `status`.
 */
MOE_API int32_t moe_ep_dispatch_begin(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                      const float* topk_weights, int32_t num_tokens,
                                      int32_t topk, int32_t slot, uint64_t epoch,
                                      int32_t* status, void* stream);
MOE_API int32_t moe_ep_dispatch_scatter(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                        const float* topk_weights, int32_t num_tokens,
                                        int32_t topk, int32_t slot, uint64_t epoch,
                                        int32_t num_blocks, int32_t pad_rows,
                                        int32_t expert_alignment, int32_t scale_rows,
                                        uint64_t wait_ns, int32_t* status, void* stream);
MOE_API int32_t moe_ep_dispatch_end(moe_ep_t ep, int32_t slot, uint64_t epoch, uint64_t wait_ns,
                                    int32_t* status, void* stream);
MOE_API int32_t moe_ep_dispatch(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                const float* topk_weights, int32_t num_tokens, int32_t topk,
                                int32_t slot, uint64_t epoch, int32_t num_blocks, int32_t pad_rows,
                                int32_t expert_alignment, int32_t scale_rows, uint64_t wait_ns,
                                int32_t* status, void* stream);

/*
 * Dispatch with an FP8 payload: DeepEP's dispatch of an (x_fp8, x_scales) pair
 * (thirdParty/DeepEP/deep_ep/buffer.py:338-342, per-128 scales copied with each
 * row at csrc/kernels/intranode.cu:397-402).  x_fp8: [num_tokens][hidden] e4m3
 * bytes; x_scales: [num_tokens][hidden/128] float; hidden % 128 == 0.  Same
 * phases, layout, metadata and arguments as moe_ep_dispatch (expert_alignment 1,
 * no scale_rows); both arrays are copied unchanged, so a row crosses NVLink in
 * hidden + hidden/32 bytes instead of 2 * hidden.  In the receive slot the e4m3
 * rows are at views.recv_x as [cap_rows][hidden] bytes and their scales at
 * views.recv_x + cap_rows * hidden as [cap_rows][hidden/128] float.
 */
MOE_API int32_t moe_ep_dispatch_fp8(moe_ep_t ep, const void* x_fp8, const float* x_scales,
                                    const int64_t* topk_idx, const float* topk_weights,
                                    int32_t num_tokens, int32_t topk, int32_t slot, uint64_t epoch,
                                    int32_t num_blocks, int32_t pad_rows, uint64_t wait_ns,
                                    int32_t* status, void* stream);
/* Its scatter phase alone (after moe_ep_dispatch_begin; moe_ep_dispatch_end follows). */
MOE_API int32_t moe_ep_dispatch_fp8_scatter(moe_ep_t ep, const void* x_fp8, const float* x_scales,
                                            const int64_t* topk_idx, const float* topk_weights,
                                            int32_t num_tokens, int32_t topk, int32_t slot,
                                            uint64_t epoch, int32_t num_blocks, int32_t pad_rows,
                                            uint64_t wait_ns, int32_t* status, void* stream);

/*
 * Per-128-column e4m3 quantisation of bf16 rows, as DeepEP's per_token_cast_to_fp8
 * (thirdParty/DeepEP/tests/utils.py:50-58) defines it: for each row and group of
 * 128 columns, amax = max|x| clamped to 1e-4, out = e4m3(x * (1/amax * 448)) with
 * round-to-nearest-even and saturation, scale = amax / 448.  x: [rows][hidden]
 * bf16 (row stride ldx elements); out_fp8: [rows][hidden] bytes (stride ld_out);
 * out_scales: [rows][hidden/128] float (stride ld_scales).  hidden % 128 == 0.
 */
MOE_API int32_t moe_fp8_quantize(const void* x, int64_t ldx, int64_t rows, int32_t hidden,
                                 void* out_fp8, int64_t ld_out, float* out_scales,
                                 int64_t ld_scales, void* stream);

/*
 * The inverse, as DeepEP's per_token_cast_back (tests/utils.py:61-75):
 * out = bf16(float(x_fp8) * scale) for rows [0, rows), where rows = rows_max or,
 * when rows_dev (a device int32) is given, min(rows_max, *rows_dev) read on the
 * device (e.g. the received count, the last of a dispatch's expert_offsets).
 */
MOE_API int32_t moe_fp8_dequantize(const void* x_fp8, int64_t ldx, const float* scales,
                                   int64_t ld_scales, const int32_t* rows_dev, int64_t rows_max,
                                   int32_t hidden, void* out, int64_t ld_out, void* stream);

/*
 * Expert-ordered dispatch, for a GEMM that starts an expert's tiles as soon as
 * that expert's rows have landed instead of after the whole dispatch.  The same
 * receive layout, metadata, offsets and send positions as moe_ep_dispatch
 * (expert_alignment 1, bf16 rows, no scale_rows); the phases differ in:
 *   ordered_begin    also builds the sending order of this rank's tokens: by the
 *                    earliest of each token's experts in the walk (local expert
 *                    index first, then owner), and clears this rank's arrival
 *                    counters of the slot (before its count flag is raised, so no
 *                    peer can add early);
 *   ordered_scatter  every rank pushes its tokens in that order, each token's rows
 *                    to all their owners from one read of the token, and after
 *                    every batch of tokens adds the rows delivered to the owners'
 *                    arrival counters of those experts; it also stores each local
 *                    expert's expected row count.  It takes the tokens of the
 *                    slot's last ordered_begin (MOE_ERR_INVALID_ARG otherwise);
 *   end              moe_ep_dispatch_end (all rows landed), as before.
 * moe_ep_dispatch_ordered runs the three.  No counterpart in DeepEP, whose
 * receiver learns of rows only through its per-channel queues.
 */
MOE_API int32_t moe_ep_dispatch_ordered_begin(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                              const float* topk_weights, int32_t num_tokens,
                                              int32_t topk, int32_t slot, uint64_t epoch,
                                              int32_t* status, void* stream);
MOE_API int32_t moe_ep_dispatch_ordered_scatter(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                                const float* topk_weights, int32_t num_tokens,
                                                int32_t topk, int32_t slot, uint64_t epoch,
                                                int32_t num_blocks, int32_t pad_rows,
                                                uint64_t wait_ns, int32_t* status, void* stream);
MOE_API int32_t moe_ep_dispatch_ordered(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                        const float* topk_weights, int32_t num_tokens, int32_t topk,
                                        int32_t slot, uint64_t epoch, int32_t num_blocks,
                                        int32_t pad_rows, uint64_t wait_ns, int32_t* status,
                                        void* stream);

/*
 * The grouped GEMM over the receive rows of an expert-ordered dispatch into
 * `slot` (A = the slot's bf16 rows, K = hidden, offsets = its expert_offsets),
 * C = act(A @ B[e]) with act none or GELU, as moe_grouped_gemm.  It may be
 * enqueued as soon as this rank's ordered_scatter has been enqueued before it
 * (this rank's expected counts and offsets come from that kernel): the GEMM's
 * producer waits, per expert and bounded by wait_ns, until the expert's arrival
 * counter reaches its expected count, so its tiles start while later experts'
 * rows are still in flight.  An expired wait records MOE_ERR_TIMEOUT in
 * `status` and the kernel returns.  Replaces, for this path, the grouped GEMM
 * after a complete dispatch in src/train_moe_baseline.py:376-399.
 */
MOE_API int32_t moe_ep_expert_gemm(moe_ep_t ep, int32_t slot, const void* b, int64_t b_stride_e,
                                   int64_t b_stride_k, int64_t b_stride_n, void* c, int64_t ldc,
                                   int64_t n, int32_t activation, int32_t num_sms,
                                   int32_t use_atomic_queue, int32_t* work_counter,
                                   uint64_t wait_ns, int32_t* status, void* stream);

/*
 * Cached re-dispatch (DeepEP's dispatch given a handle: deep_ep/buffer.py:383-390,
 * deep_ep.cpp:588-600): new rows x for the tokens and top-k choices of the most
 * recent dispatch, which went into src_slot, pushed into the other slot `slot` at
 * the places that dispatch gave them.  No layout or count phase runs:
 *   begin    raises this rank's count flag for `slot` in every rank ("my side of
 *            the slot is free"); no counts are sent        ~ cached_notify_dispatch
 *   scatter  waits (bounded) for every rank's flag, pushes the rows, copies this
 *            rank's receive metadata and expert offsets from src_slot, zeroes the
 *            alignment padding rows, and raises the data flag everywhere;
 *   end      moe_ep_dispatch_end.
 * topk_idx / topk_weights / num_tokens / topk must be those of the source
 * dispatch (the rows' destinations and, with scale_rows, their weights); every
 * rank runs the cached form for the same dispatch.  The layout, expert_alignment
 * and receive counts are the source dispatch's.
 */
MOE_API int32_t moe_ep_dispatch_cached_begin(moe_ep_t ep, int32_t slot, uint64_t epoch, void* stream);
MOE_API int32_t moe_ep_dispatch_cached_scatter(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                               const float* topk_weights, int32_t num_tokens,
                                               int32_t topk, int32_t src_slot, int32_t slot,
                                               uint64_t epoch, int32_t num_blocks, int32_t pad_rows,
                                               int32_t scale_rows, uint64_t wait_ns,
                                               int32_t* status, void* stream);
MOE_API int32_t moe_ep_dispatch_cached(moe_ep_t ep, const void* x, const int64_t* topk_idx,
                                       const float* topk_weights, int32_t num_tokens, int32_t topk,
                                       int32_t src_slot, int32_t slot, uint64_t epoch,
                                       int32_t num_blocks, int32_t pad_rows, int32_t scale_rows,
                                       uint64_t wait_ns, int32_t* status, void* stream);

/*
 * Fused down-projection + combine push: the grouped GEMM C = A @ B[e] over this
 * rank's received rows (expert_offsets of `slot`, experts = num_experts/world,
 * n = hidden, bf16), whose epilogue writes each result row straight into the
 * combine rows of the token's source rank (peer memory, row src_token * max_topk +
 * slot) instead of a local buffer; then this rank raises its ready flag in every
 * rank.  A = the expert hidden rows [m_total, k] (the receive layout), B as in
 * moe_grouped_gemm.  With moe_ep_combine_pushed this replaces expert_out +
 * moe_ep_combine: the all-to-all back overlaps the GEMM tile by tile, and the
 * combine becomes a local reduce (src/deep_ep_comm.py:107-115 moves the same rows).
 */
MOE_API int32_t moe_ep_push_gemm(moe_ep_t ep, const void* a, int64_t lda, const void* b,
                                 int64_t b_stride_e, int64_t b_stride_k, int64_t b_stride_n,
                                 int64_t m_total, int64_t k, int32_t dtype, int32_t num_sms,
                                 int32_t use_atomic_queue, int32_t* work_counter, int32_t slot,
                                 uint64_t epoch, int32_t* status, void* stream);

/* The combine of rows pushed by moe_ep_push_gemm: waits for every owner's ready
 * flag, then reduces this rank's combine rows as moe_ep_combine_end does (same
 * arguments, same fp32 slot-order sum, bit-identical result). */
MOE_API int32_t moe_ep_combine_pushed(moe_ep_t ep, const int64_t* topk_idx,
                                      const float* topk_weights, int32_t num_tokens,
                                      int32_t topk, int32_t slot, uint64_t epoch,
                                      int32_t weighted, void* out, int32_t num_blocks,
                                      uint64_t wait_ns, int32_t* status, void* stream);

/* Sets the endpoint's device epoch counter (stream-ordered; see epoch 0 above). */
MOE_API int32_t moe_ep_set_device_epoch(moe_ep_t ep, uint64_t epoch, void* stream);

/*
 * Combine, in two phases (moe_ep_combine runs both):
 *   begin  raises "this rank's expert_out rows for `slot` are complete" in every
 *          rank (no waiting);
 *   end    waits (bounded) for every rank's flag, then for each of this rank's
 *          num_tokens tokens writes out[t] = bf16( sum_j s_j * owner_j.expert_out[
 *          send_pos[t][j]] ), summed in fp32 in slot order, with s_j = 1
 *          (weighted == 0: the reference's unweighted combine, intranode.cu:961-1030)
 *          or s_j = topk_weights[t][j] (the fused weighted top-k reduction).
 * topk_idx / topk_weights / num_tokens / topk are those of the matching dispatch.
 */
MOE_API int32_t moe_ep_combine_begin(moe_ep_t ep, int32_t slot, uint64_t epoch, void* stream);
MOE_API int32_t moe_ep_combine_end(moe_ep_t ep, const int64_t* topk_idx, const float* topk_weights,
                                   int32_t num_tokens, int32_t topk, int32_t slot,
                                   uint64_t epoch, int32_t weighted, void* out,
                                   int32_t num_blocks, uint64_t wait_ns, int32_t* status,
                                   void* stream);
MOE_API int32_t moe_ep_combine(moe_ep_t ep, const int64_t* topk_idx, const float* topk_weights,
                               int32_t num_tokens, int32_t topk, int32_t slot, uint64_t epoch,
                               int32_t weighted, void* out, int32_t num_blocks, uint64_t wait_ns,
                               int32_t* status, void* stream);

/*
 * Gradient of the top-k weights for the routed experts' backward:
 * out[t][j] = <grad_out[t], y(t, j)> in fp32, y(t, j) being the expert-output row
 * the owner produced for (token t, slot j) in `slot` (read through the peer
 * pointers, so it works at any world size); 0 where the slot had no expert.
 * grad_out: [num_tokens][hidden] bf16.  No counterpart in the reference.
 */
MOE_API int32_t moe_ep_topk_weight_grad(moe_ep_t ep, const void* grad_out, const int64_t* topk_idx,
                                        int32_t num_tokens, int32_t topk, int32_t slot, float* out,
                                        int32_t num_blocks, void* stream);

/*
 * Router top-k: softmax / top-k / renormalisation after the gate's linear layer
 * (src/train_moe_baseline.py:316-318; the bias and renormalisation are the
 * BASELINE configs' options).  One warp per token, E <= 256, top_k <= 16.
 *   logits          [T, E] bf16 (MOE_DTYPE_BF16) or fp32 (MOE_DTYPE_F32)
 *   bias            [E] fp32 or NULL, added to the logits
 *   probs           [T, E] fp32 out: softmax(logits + bias)
 *   topk_idx        [T, k] int64 out: the k largest probabilities, ties to the
 *                   lower expert id, in descending order
 *   topk_weights    [T, k] fp32 out: those probabilities, divided by their sum
 *                   when renormalize != 0
 */
MOE_API int32_t moe_router_topk(const void* logits, int32_t logits_dtype, const float* bias,
                                int32_t num_tokens, int32_t num_experts, int32_t topk,
                                int32_t renormalize, float* probs, int64_t* topk_idx,
                                float* topk_weights, void* stream);

/*
 * Backward of moe_router_topk's topk_weights with respect to the logits:
 * grad_logits [T, E] fp32 = softmax-backward of the gradient scattered from
 * grad_topk_weights [T, k] (through the renormalisation when renormalize != 0).
 * No counterpart in the reference, which runs inference only.
 */
MOE_API int32_t moe_router_topk_backward(const float* probs, const int64_t* topk_idx,
                                         const float* grad_topk_weights, int32_t num_tokens,
                                         int32_t num_experts, int32_t topk, int32_t renormalize,
                                         float* grad_logits, void* stream);

/*
 * DeepEP's get_dispatch_layout (thirdParty/DeepEP/deep_ep/buffer.py:293-319,
 * kernels/layout.cu:10-121): tokens per rank (each token counted once per rank),
 * tokens per expert and is_token_in_rank [num_tokens][world] (bool, 1 byte).
 * Any output may be NULL.
 */
MOE_API int32_t moe_ep_dispatch_layout(const int64_t* topk_idx, int32_t num_tokens, int32_t topk,
                                       int32_t num_experts, int32_t world,
                                       int32_t* tokens_per_rank, int32_t* tokens_per_expert,
                                       bool* is_token_in_rank, void* stream);

/* CUDA IPC helpers for sharing symmetric buffers between processes. */
#define MOE_IPC_HANDLE_BYTES 64
MOE_API int32_t moe_ipc_export(void* dev_ptr, void* handle_out);
MOE_API int32_t moe_ipc_import(const void* handle, void** dev_ptr_out);
MOE_API int32_t moe_ipc_close(void* dev_ptr);

#ifdef __cplusplus
}
#endif

#endif /* MOE_OVERLAP_H_ */
