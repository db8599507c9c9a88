// K1: 1x128 group FP8 (e4m3) quantisation of bf16 activations.
//
// Numerics follow moe_bench/verify.py:108-117 bit for bit:
//   scale = max(amax / 448, 1e-12)   IEEE fp32 division
//   q     = e4m3_rne(clamp(x / scale, -448, 448))   IEEE fp32 division per element
//
// Fast path (cols % 128 == 0, 16-byte aligned rows): a half-warp owns one group;
// each lane loads 8 bf16 with one 128-bit load, the amax is reduced with 4
// xor-shuffles inside the half-warp, and each lane stores 8 bytes.  Every warp
// keeps two groups in flight per iteration to cover HBM latency.
// Generic path (ragged cols or unaligned strides): one warp per group, scalar
// loads, bounds-checked, with missing columns treated as zeros (the reference
// zero-pads before the amax).
#include "b2m_common.cuh"
#include "b2m_host.h"

namespace b2m {
namespace {

constexpr int kQuantThreads = 256;

__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint32_t quant4(const float* f, float scale) {
  uint32_t r = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) r |= static_cast<uint32_t>(f32_to_e4m3(clamp448(f[i] / scale))) << (8 * i);
  return r;
}

// groups = rows * (cols/128); group g covers row g / gpr, columns (g % gpr)*128 ...
__global__ void __launch_bounds__(kQuantThreads) quant_g128_fast(const __nv_bfloat16* __restrict__ x,
                                                                  int64_t ldx, uint8_t* __restrict__ q,
                                                                  int64_t ldq, float* __restrict__ scale,
                                                                  int64_t lds, int64_t groups, int64_t gpr) {
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;
  const int hl = lane & 15;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kQuantThreads) >> 5;
  // Each warp step handles 4 groups: two per half-warp (g0 and g0 + 2).
  for (int64_t base = warp * 4; base < groups; base += nwarps * 4) {
    int64_t g[2] = {base + half, base + 2 + half};
    uint4 raw[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (g[u] < groups) {
        const int64_t row = g[u] / gpr;
        const int64_t col = (g[u] - row * gpr) * 128 + hl * 8;
        raw[u] = __ldg(reinterpret_cast<const uint4*>(x + row * ldx + col));
      } else {
        raw[u] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float f[8];
      bf16x8_to_f32(raw[u], f);
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(f[i]));
#pragma unroll
      for (int off = 8; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float s = fmaxf(amax / 448.0f, 1e-12f);
      if (g[u] < groups) {
        const int64_t row = g[u] / gpr;
        const int64_t gi = g[u] - row * gpr;
        uint2 out;
        out.x = quant4(f, s);
        out.y = quant4(f + 4, s);
        *reinterpret_cast<uint2*>(q + row * ldq + gi * 128 + hl * 8) = out;
        if (hl == 0) scale[row * lds + gi] = s;
      }
    }
  }
}

__global__ void __launch_bounds__(kQuantThreads) quant_g128_generic(const __nv_bfloat16* __restrict__ x,
                                                                     int64_t ldx, uint8_t* __restrict__ q,
                                                                     int64_t ldq, float* __restrict__ scale,
                                                                     int64_t lds, int64_t rows, int64_t cols,
                                                                     int64_t gpr) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kQuantThreads) >> 5;
  for (int64_t g = warp; g < rows * gpr; g += nwarps) {
    const int64_t row = g / gpr;
    const int64_t c0 = (g - row * gpr) * 128;
    float f[4];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t c = c0 + lane * 4 + i;
      f[i] = c < cols ? __bfloat162float(x[row * ldx + c]) : 0.0f;
      amax = fmaxf(amax, fabsf(f[i]));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float s = fmaxf(amax / 448.0f, 1e-12f);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t c = c0 + lane * 4 + i;
      if (c < cols) q[row * ldq + c] = f32_to_e4m3(clamp448(f[i] / s));
    }
    if (lane == 0) scale[row * lds + (g - row * gpr)] = s;
  }
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_quant_g128(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq,
                              float* scale, int64_t ld_scale, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (rows < 0 || cols < 0) return fail(B2M_ERR_ARG, "quant_g128: negative shape (%lld, %lld)", (long long)rows,
                                        (long long)cols);
  if (rows == 0 || cols == 0) return B2M_OK;
  const int64_t gpr = (cols + 127) / 128;
  if (!x || !q || !scale) return fail(B2M_ERR_ARG, "quant_g128: null pointer");
  if (ldx < cols || ldq < cols || ld_scale < gpr)
    return fail(B2M_ERR_ARG, "quant_g128: strides (ldx=%lld, ldq=%lld, ld_scale=%lld) smaller than the row",
                (long long)ldx, (long long)ldq, (long long)ld_scale);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool fast = (cols % 128 == 0) && (ldx % 8 == 0) && (ldq % 8 == 0) && aligned16(x) &&
                    (reinterpret_cast<uintptr_t>(q) & 7u) == 0;
  const int64_t groups = rows * gpr;
  if (fast) {
    const int64_t warps = (groups + 3) / 4;
    int64_t blocks = (warps * 32 + kQuantThreads - 1) / kQuantThreads;
    blocks = blocks < static_cast<int64_t>(num_sms) * 16 ? blocks : static_cast<int64_t>(num_sms) * 16;
    quant_g128_fast<<<static_cast<unsigned>(blocks), kQuantThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<uint8_t*>(q), ldq, scale, ld_scale, groups, gpr);
  } else {
    int64_t blocks = (groups * 32 + kQuantThreads - 1) / kQuantThreads;
    blocks = blocks < static_cast<int64_t>(num_sms) * 16 ? blocks : static_cast<int64_t>(num_sms) * 16;
    quant_g128_generic<<<static_cast<unsigned>(blocks), kQuantThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<uint8_t*>(q), ldq, scale, ld_scale, rows, cols,
        gpr);
  }
  return check_cuda(cudaGetLastError(), "quant_g128 launch");
}
