// Top-k combine (+ shared expert add) and the gate/up weight interleave used at set-up.
#include <atomic>

#include "b2m_common.cuh"
#include "b2m_host.h"

namespace b2m {
namespace {

constexpr int kCombineThreads = 256;

constexpr int64_t kCombineChunk = 1024;  // columns of one work unit (4 warp-wide steps of 8 columns per lane)

// out[t, :] = bf16(sum_j staged[t*k + j, :] + shared[t, :]).  A warp takes one unit -- a
// token's 1024-column chunk -- at a time, so the grid (every resident warp) finishes in
// near-equal shares instead of in waves of whole tokens; the token's expert ids and map
// entries give a warp-uniform pair mask, and the lanes walk the chunk 8 columns at a time.
template <bool kWide>
__global__ void __launch_bounds__(kCombineThreads)
    combine_kernel(const __nv_bfloat16* __restrict__ staged, int64_t tokens, int top_k, int64_t hidden,
                   const int32_t* __restrict__ topk_ids, const int32_t* __restrict__ expert_map,
                   const __nv_bfloat16* __restrict__ shared, __nv_bfloat16* __restrict__ out, int64_t ld_out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kCombineThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kCombineThreads) >> 5;
  const int64_t chunks = (hidden + kCombineChunk - 1) / kCombineChunk;
  for (int64_t u = warp; u < tokens * chunks; u += nwarps) {
    const int64_t t = u / chunks;
    const int64_t c_end = min(hidden, (u - t * chunks + 1) * kCombineChunk);
    const uint32_t mask = local_pair_mask(topk_ids, expert_map, t, top_k, lane);
#pragma unroll 2
    for (int64_t c = (u - t * chunks) * kCombineChunk + lane * 8; c < c_end; c += 256)
      *reinterpret_cast<uint4*>(out + t * ld_out + c) =
          combine_vec<kWide>(staged, t, top_k, hidden, c, mask, topk_ids, expert_map, shared);
  }
}

// w1 [E, 2I, H] (gate rows then up rows) -> [E, 2I, H] with 128-row blocks ordered
// gate0, up0, gate1, up1, ...; scales [E, 2I/128, KB] permuted the same way.
__global__ void interleave_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t experts,
                                       int64_t inter, int64_t hidden) {
  const int64_t vec_per_row = hidden / 16;
  const int64_t rows = experts * 2 * inter;
  const int64_t total = rows * vec_per_row;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t drow = v / vec_per_row;
    const int64_t cv = v - drow * vec_per_row;
    const int64_t e = drow / (2 * inter);
    const int64_t r = drow - e * 2 * inter;  // destination row inside the expert
    const int64_t blk = r / 128, within = r % 128;
    const int64_t g = blk & 1, j = blk >> 1;
    const int64_t srow = e * 2 * inter + g * inter + j * 128 + within;
    reinterpret_cast<uint4*>(dst)[drow * vec_per_row + cv] =
        __ldg(reinterpret_cast<const uint4*>(src) + srow * vec_per_row + cv);
  }
}

__global__ void interleave_scales_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t experts,
                                         int64_t nblk_half, int64_t kb) {
  const int64_t total = experts * 2 * nblk_half * kb;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t k = i % kb;
    const int64_t db = (i / kb) % (2 * nblk_half);
    const int64_t e = i / (kb * 2 * nblk_half);
    const int64_t g = db & 1, j = db >> 1;
    dst[i] = src[(e * 2 * nblk_half + g * nblk_half + j) * kb + k];
  }
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_combine(const void* staged, int64_t tokens, int32_t top_k, int64_t hidden,
                           const int32_t* topk_ids, const int32_t* expert_map, const void* shared, void* out,
                           int64_t ld_out, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (tokens < 0 || top_k <= 0 || hidden <= 0) return fail(B2M_ERR_ARG, "combine: bad shape");
  if (tokens == 0) return B2M_OK;
  if (hidden % 8 || ld_out % 8 || ld_out < hidden)
    return fail(B2M_ERR_ARG, "combine: hidden (%lld) and ld_out (%lld) must be multiples of 8", (long long)hidden,
                (long long)ld_out);
  if (!staged || !out || (expert_map && !topk_ids)) return fail(B2M_ERR_ARG, "combine: null pointer");
  if (!aligned16(staged) || !aligned16(out) || (shared && !aligned16(shared)))
    return fail(B2M_ERR_ARG, "combine: pointers must be 16-byte aligned");
  // every resident warp, or fewer when there are fewer units
  const bool wide = top_k > 32;
  auto kernel = wide ? combine_kernel<true> : combine_kernel<false>;
  static std::atomic<int> resident[2] = {0, 0};  // blocks per SM (the same on every sm_100 device)
  int per_sm = resident[wide].load(std::memory_order_relaxed);
  if (per_sm == 0) {
    B2M_TRY(check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kCombineThreads, 0),
                       "combine: occupancy"));
    per_sm = per_sm > 0 ? per_sm : 1;
    resident[wide].store(per_sm, std::memory_order_relaxed);
  }
  const int64_t units = tokens * ((hidden + kCombineChunk - 1) / kCombineChunk);
  int64_t blocks = (units * 32 + kCombineThreads - 1) / kCombineThreads;
  if (blocks > int64_t(num_sms) * per_sm) blocks = int64_t(num_sms) * per_sm;
  kernel<<<static_cast<unsigned>(blocks), kCombineThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(staged), tokens, top_k, hidden, topk_ids, expert_map,
      static_cast<const __nv_bfloat16*>(shared), static_cast<__nv_bfloat16*>(out), ld_out);
  return check_cuda(cudaGetLastError(), "combine launch");
}

extern "C" int b2m_w1_interleave(const void* w1, const float* w1_scale, int32_t num_experts, int32_t inter,
                                 int64_t hidden, void* w1_out, float* w1_scale_out, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (num_experts <= 0 || inter <= 0 || inter % 128 || hidden <= 0 || hidden % 128)
    return fail(B2M_ERR_ARG, "w1_interleave: inter (%d) and hidden (%lld) must be positive multiples of 128", inter,
                (long long)hidden);
  if (!w1 || !w1_scale || !w1_out || !w1_scale_out) return fail(B2M_ERR_ARG, "w1_interleave: null pointer");
  if (!aligned16(w1) || !aligned16(w1_out)) return fail(B2M_ERR_ARG, "w1_interleave: weights must be 16B aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  interleave_rows_kernel<<<num_sms * 8, 256, 0, s>>>(static_cast<const uint8_t*>(w1), static_cast<uint8_t*>(w1_out),
                                                      num_experts, inter, hidden);
  B2M_TRY(check_cuda(cudaGetLastError(), "interleave rows launch"));
  interleave_scales_kernel<<<num_sms, 256, 0, s>>>(w1_scale, w1_scale_out, num_experts, inter / 128, hidden / 128);
  return check_cuda(cudaGetLastError(), "interleave scales launch");
}
