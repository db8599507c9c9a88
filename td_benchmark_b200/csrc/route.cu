// On-device routing: softmax -> top-k -> renormalise over router logits.
//
// The reference computes its routing on the host side of the benchmark, outside the timed
// region (moe_bench/data/routing.py:56-64):
//   logits = hidden.float() @ gate.float().T  (+ strength * log(E * p) under imbalanced routing)
//   topk_weights, topk_ids = topk(softmax(logits), k);  topk_weights /= topk_weights.sum(-1)
// b2m_route_topk is every step after the gate GEMM, fused in one pass: one warp per token
// holds the token's E logits in registers (E/32 per lane), adds the optional per-expert
// bias, takes the softmax (max-subtracted exp, warp sum, IEEE division), selects the k
// largest probabilities one warp-argmax at a time (equal probabilities: lower expert index
// first) in descending order, as topk returns them, and divides each by their sum
// (accumulated in that order).  HBM-bound: 4E bytes read and 8k written per token.
#include "b2m_common.cuh"
#include "b2m_host.h"

#include <math.h>

namespace b2m {
namespace {

constexpr int kThreads = 256;

// (value, index) of the larger probability; on equal values the lower expert index wins.
__device__ __forceinline__ void argmax_pair(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

template <int NV>
__global__ void __launch_bounds__(kThreads)
    route_topk_kernel(const float* __restrict__ logits, int64_t tokens, int experts, int top_k,
                      const float* __restrict__ bias, int32_t* __restrict__ ids, float* __restrict__ weights) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  for (int64_t t = warp; t < tokens; t += nwarps) {
    const float* row = logits + t * experts;
    float v[NV];
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int e = i * 32 + lane;
      v[i] = -INFINITY;
      if (e < experts) {
        v[i] = __ldg(row + e);
        if (bias) v[i] += __ldg(bias + e);
      }
      m = fmaxf(m, v[i]);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      v[i] = (i * 32 + lane < experts) ? expf(v[i] - m) : 0.0f;
      s += v[i];
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = (i * 32 + lane < experts) ? v[i] / s : -1.0f;  // probabilities
    float sel_p = 0.0f;  // lane j < top_k: probability of the j-th selection
    int sel_i = 0;
    float sum = 0.0f;
    for (int j = 0; j < top_k; ++j) {
      float bv = -1.0f;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < NV; ++i) argmax_pair(bv, bi, v[i], i * 32 + lane);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        argmax_pair(bv, bi, ov, oi);
      }
      // every lane now holds the winner; its owner removes it from the candidates
#pragma unroll
      for (int i = 0; i < NV; ++i)
        if (i * 32 + lane == bi) v[i] = -1.0f;
      sum += bv;
      if (lane == j) {
        sel_p = bv;
        sel_i = bi;
      }
    }
    if (lane < top_k) {
      ids[t * top_k + lane] = sel_i;
      weights[t * top_k + lane] = sel_p / sum;
    }
  }
}

template <int NV>
int launch_route(const float* logits, int64_t tokens, int experts, int top_k, const float* bias, int32_t* ids,
                 float* weights, int num_sms, cudaStream_t s) {
  int64_t blocks = (tokens * 32 + kThreads - 1) / kThreads;
  if (blocks > int64_t(num_sms) * 8) blocks = int64_t(num_sms) * 8;
  if (blocks < 1) blocks = 1;
  route_topk_kernel<NV><<<static_cast<int>(blocks), kThreads, 0, s>>>(logits, tokens, experts, top_k, bias, ids,
                                                                      weights);
  return check_cuda(cudaGetLastError(), "route_topk launch");
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_route_topk(const float* logits, int64_t tokens, int32_t experts, int32_t top_k, const float* bias,
                              int32_t* topk_ids, float* topk_weights, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (tokens < 0 || experts < 1 || experts > 1024 || top_k < 1 || top_k > 32 || top_k > experts)
    return fail(B2M_ERR_ARG, "route_topk: need 1 <= top_k <= min(32, E), 1 <= E <= 1024 (E=%d, top_k=%d)", experts,
                top_k);
  if (tokens > 0 && (!logits || !topk_ids || !topk_weights)) return fail(B2M_ERR_ARG, "route_topk: null pointer");
  if (tokens == 0) return B2M_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int nv = (experts + 31) / 32;
  if (nv <= 1) return launch_route<1>(logits, tokens, experts, top_k, bias, topk_ids, topk_weights, num_sms, s);
  if (nv <= 2) return launch_route<2>(logits, tokens, experts, top_k, bias, topk_ids, topk_weights, num_sms, s);
  if (nv <= 4) return launch_route<4>(logits, tokens, experts, top_k, bias, topk_ids, topk_weights, num_sms, s);
  if (nv <= 8) return launch_route<8>(logits, tokens, experts, top_k, bias, topk_ids, topk_weights, num_sms, s);
  if (nv <= 16) return launch_route<16>(logits, tokens, experts, top_k, bias, topk_ids, topk_weights, num_sms, s);
  return launch_route<32>(logits, tokens, experts, top_k, bias, topk_ids, topk_weights, num_sms, s);
}
