// Router top-k on sm_100a: the softmax / top-k / renormalisation that follows the
// gate's linear layer, forward and backward, one warp per token.
//
// Forward (src/train_moe_baseline.py:316-318, with the BASELINE configs' optional
// gate bias and top-k renormalisation):
//   z = float(logits[t]) + bias;  p = softmax(z) (fp32);  idx = top-k of p (ties to
//   the lower expert id);  w = p[idx] (/ sum p[idx] when renormalising).
// Backward of w with respect to the logits, for an upstream gradient dw [T, k]:
//   renormalised:  dp_j = (dw_j - sum_i dw_i w_i) / s,  s = sum_i p[idx_i]
//   otherwise:     dp_j = dw_j
//   dz = p * (dp_scattered - <p, dp_scattered>)     (softmax backward)
// The gate's linear layer (x @ W^T) and its backward stay matrix products
// (cuBLAS through torch); these kernels replace the chain of small elementwise,
// reduction, sort and gather launches between them.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/moe_overlap.h"

namespace moe {
namespace router {

constexpr int kMaxE = 256;   // experts per token handled by one warp (8 per lane)
constexpr int kMaxK = 16;
constexpr int kPerLane = kMaxE / 32;
constexpr int kWarps = 8;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Loads the token's E logits (bf16 or fp32) plus bias into per-lane registers:
// expert e = lane + 32 * i.  Missing experts read -inf.
template <typename T>
__device__ __forceinline__ void load_logits(const T* row, const float* bias, int E, int lane,
                                            float (&z)[kPerLane]) {
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int e = lane + 32 * i;
    float v = -INFINITY;
    if (e < E) {
      if constexpr (sizeof(T) == 2)
        v = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[e]);
      else
        v = static_cast<float>(row[e]);
      if (bias != nullptr) v += bias[e];
    }
    z[i] = v;
  }
}

template <typename T>
__global__ void __launch_bounds__(32 * kWarps) topk_fwd_kernel(const T* logits, const float* bias,
                                                               int num_tokens, int E, int k,
                                                               int renormalize, float* probs,
                                                               int64_t* idx_out, float* w_out) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  float z[kPerLane];
  load_logits(logits + static_cast<int64_t>(t) * E, bias, E, lane, z);
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) m = fmaxf(m, z[i]);
  m = warp_max(m);
  float p[kPerLane], s = 0.0f;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    p[i] = (lane + 32 * i < E) ? expf(z[i] - m) : 0.0f;
    s += p[i];
  }
  s = warp_sum(s);
  const float inv = 1.0f / s;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    p[i] *= inv;
    const int e = lane + 32 * i;
    if (e < E) probs[static_cast<int64_t>(t) * E + e] = p[i];
  }
  // k rounds of a warp arg-max; a taken expert is marked with -1 (probabilities
  // are >= 0, so the mark never ties a candidate).
  float taken_w[kMaxK];
  int taken_e[kMaxK];
  float wsum = 0.0f;
  for (int j = 0; j < k; ++j) {
    float best = -1.0f;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
      const int e = lane + 32 * i;
      if (e < E && p[i] != -1.0f && (p[i] > best || (p[i] == best && e < be))) {
        best = p[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ob > best || (ob == best && oe < be)) {
        best = ob;
        be = oe;
      }
    }
    if (be == 0x7fffffff) {
      // No comparable candidate: a NaN logit makes every probability NaN.  Take
      // the lowest expert id not taken yet, as a stable sort of all-equal values
      // would (the same in every lane, so the branch is warp-uniform).
      int ce = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < kPerLane; ++i) {
        const int e = lane + 32 * i;
        if (e < E && p[i] != -1.0f && e < ce) ce = e;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ce = min(ce, __shfl_xor_sync(0xffffffffu, ce, o));
      be = ce;
      best = __int_as_float(0x7fc00000);  // its probability: NaN
    }
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
      if (lane + 32 * i == be) p[i] = -1.0f;
    taken_w[j] = best;
    taken_e[j] = be;
    wsum += best;
  }
  if (lane < k) {
    float wv = 0.0f;
    int ev = 0;
#pragma unroll
    for (int j = 0; j < kMaxK; ++j)
      if (j == lane) {
        wv = taken_w[j];
        ev = taken_e[j];
      }
    idx_out[static_cast<int64_t>(t) * k + lane] = ev;
    w_out[static_cast<int64_t>(t) * k + lane] = renormalize ? wv / wsum : wv;
  }
}

__global__ void __launch_bounds__(32 * kWarps) topk_bwd_kernel(const float* probs, const int64_t* idx,
                                                               const float* dw, int num_tokens,
                                                               int E, int k, int renormalize,
                                                               float* dlogits) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= num_tokens) return;
  const float* prow = probs + static_cast<int64_t>(t) * E;
  // Gradient with respect to the selected probabilities.
  float dsel = 0.0f;  // lane j < k holds dp for slot j
  int esel = -1;
  if (lane < k) {
    const int64_t ev = idx[static_cast<int64_t>(t) * k + lane];
    if (ev >= 0 && ev < E) {  // an id outside [0, E) selects nothing and reads nothing
      esel = static_cast<int>(ev);
      dsel = dw[static_cast<int64_t>(t) * k + lane];
    }
  }
  if (renormalize) {
    const float ps = (esel >= 0) ? prow[esel] : 0.0f;
    const float s = warp_sum(ps);
    const float wj = ps / s;
    const float dot = warp_sum(esel >= 0 ? dsel * wj : 0.0f);
    dsel = (dsel - dot) / s;
  }
  float dp[kPerLane], pv[kPerLane], inner = 0.0f;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int e = lane + 32 * i;
    pv[i] = (e < E) ? prow[e] : 0.0f;
    dp[i] = 0.0f;
  }
  for (int j = 0; j < k; ++j) {
    const int ej = __shfl_sync(0xffffffffu, esel, j);
    const float dj = __shfl_sync(0xffffffffu, dsel, j);
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
      if (lane + 32 * i == ej) dp[i] += dj;
  }
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) inner += pv[i] * dp[i];
  inner = warp_sum(inner);
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    const int e = lane + 32 * i;
    if (e < E) dlogits[static_cast<int64_t>(t) * E + e] = pv[i] * (dp[i] - inner);
  }
}

}  // namespace router
}  // namespace moe

extern "C" int32_t moe_router_topk(const void* logits, int32_t logits_dtype, const float* bias,
                                   int32_t num_tokens, int32_t num_experts, int32_t topk,
                                   int32_t renormalize, float* probs, int64_t* topk_idx,
                                   float* topk_weights, void* stream) {
  using namespace moe::router;
  if (num_tokens < 0 || num_experts < 1 || num_experts > kMaxE || topk < 1 || topk > kMaxK ||
      topk > num_experts || (logits_dtype != MOE_DTYPE_BF16 && logits_dtype != 2))
    return MOE_ERR_INVALID_ARG;
  if (num_tokens == 0) return MOE_OK;
  if (logits == nullptr || probs == nullptr || topk_idx == nullptr || topk_weights == nullptr)
    return MOE_ERR_INVALID_ARG;
  const int grid = (num_tokens + kWarps - 1) / kWarps;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (logits_dtype == MOE_DTYPE_BF16)
    topk_fwd_kernel<__nv_bfloat16><<<grid, 32 * kWarps, 0, s>>>(
        static_cast<const __nv_bfloat16*>(logits), bias, num_tokens, num_experts, topk, renormalize,
        probs, topk_idx, topk_weights);
  else
    topk_fwd_kernel<float><<<grid, 32 * kWarps, 0, s>>>(static_cast<const float*>(logits), bias,
                                                        num_tokens, num_experts, topk, renormalize,
                                                        probs, topk_idx, topk_weights);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int32_t moe_router_topk_backward(const float* probs, const int64_t* topk_idx,
                                            const float* grad_topk_weights, int32_t num_tokens,
                                            int32_t num_experts, int32_t topk, int32_t renormalize,
                                            float* grad_logits, void* stream) {
  using namespace moe::router;
  if (num_tokens < 0 || num_experts < 1 || num_experts > kMaxE || topk < 1 || topk > kMaxK ||
      topk > num_experts)
    return MOE_ERR_INVALID_ARG;
  if (num_tokens == 0) return MOE_OK;
  if (probs == nullptr || topk_idx == nullptr || grad_topk_weights == nullptr || grad_logits == nullptr)
    return MOE_ERR_INVALID_ARG;
  const int grid = (num_tokens + kWarps - 1) / kWarps;
  topk_bwd_kernel<<<grid, 32 * kWarps, 0, static_cast<cudaStream_t>(stream)>>>(
      probs, topk_idx, grad_topk_weights, num_tokens, num_experts, topk, renormalize, grad_logits);
  return cudaGetLastError() == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}
