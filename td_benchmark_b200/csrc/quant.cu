// K1: 1x128 group FP8 (e4m3) quantisation of bf16 activations, and the row dispatch
// into the sorted (expert-contiguous) operand layout of the gate/up GEMM.
//
// Numerics follow moe_bench/verify.py:108-117 bit for bit:
//   scale = max(amax / 448, 1e-12)   IEEE fp32 division
//   q     = e4m3_rne(clamp(x / scale, -448, 448))   IEEE fp32 division per element
//
// Fast path (cols % 128 == 0, 16-byte aligned rows): a half-warp owns one group;
// each lane loads 8 bf16 with one 128-bit load, the amax is reduced with 4
// xor-shuffles inside the half-warp, and each lane stores 8 bytes.  Every warp
// keeps two groups in flight per iteration to cover HBM latency.  The same pass can
// scatter each token's codes and scale to the sorted rows of its top-k pairs
// (pair_pos from the alignment), so the gate/up GEMM reads A with plain tiled TMA.
// Generic path (ragged cols or unaligned strides): one warp per group, scalar
// loads, bounds-checked, with missing columns treated as zeros (the reference
// zero-pads before the amax).
#include "b2m_common.cuh"
#include "b2m_host.h"

namespace b2m {
namespace {

constexpr int kQuantThreads = 256;

struct Dispatch {
  const int32_t* pair_pos;  // [tokens * top_k], sorted row of each pair or -1; nullptr = no dispatch
  int32_t top_k;
  uint8_t* a_sorted;        // [rows_cap, cols]
  float* as_t;              // [cols/128, rows_cap]
  int64_t rows_cap;
};

// groups = rows * (cols/128); group g covers row g / gpr, columns (g % gpr)*128 ...
// q / scale (token order) may be null when only the dispatched copy is wanted.
__global__ void __launch_bounds__(kQuantThreads)
    quant_g128_fast(const __nv_bfloat16* __restrict__ x, int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                    float* __restrict__ scale, int64_t s_row, int64_t s_col, int64_t groups, int64_t gpr,
                    Dispatch d) {
  const int lane = threadIdx.x & 31;
  const int half = lane >> 4;
  const int hl = lane & 15;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kQuantThreads) >> 5;
  const int64_t cols = gpr * 128;
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
      const float s = fmaxf(halfwarp_amax(f) / 448.0f, 1e-12f);
      if (g[u] < groups) {
        const int64_t row = g[u] / gpr;
        const int64_t gi = g[u] - row * gpr;
        const uint2 out = quant8(f, s);
        if (q) *reinterpret_cast<uint2*>(q + row * ldq + gi * 128 + hl * 8) = out;
        if (scale && hl == 0) scale[row * s_row + gi * s_col] = s;
        if (d.pair_pos) {
          for (int j = 0; j < d.top_k; ++j) {
            const int32_t pos = __ldg(d.pair_pos + row * d.top_k + j);
            if (pos < 0) continue;
            *reinterpret_cast<uint2*>(d.a_sorted + pos * cols + gi * 128 + hl * 8) = out;
            if (hl == 0) d.as_t[gi * d.rows_cap + pos] = s;
          }
        }
      }
    }
  }
}

__global__ void __launch_bounds__(kQuantThreads)
    quant_g128_generic(const __nv_bfloat16* __restrict__ x, int64_t ldx, uint8_t* __restrict__ q, int64_t ldq,
                       float* __restrict__ scale, int64_t s_row, int64_t s_col, int64_t rows, int64_t cols,
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
    if (lane == 0) scale[row * s_row + (g - row * gpr) * s_col] = s;
  }
}

// Copy already-quantised token rows (and their group scales) to the sorted rows of
// their top-k pairs: a_sorted[pos] = xq[t], as_t[g, pos] = xs[t, g].
__global__ void __launch_bounds__(kQuantThreads)
    dispatch_rows_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs, int64_t tokens,
                         int64_t cols, Dispatch d) {
  const int64_t vec = cols / 16;
  const int64_t kb = cols / 128;
  const int64_t total = tokens * vec;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kQuantThreads;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x; v < total; v += stride) {
    const int64_t t = v / vec;
    const int64_t c = v - t * vec;
    bool any = false;  // expert parallel: rows of tokens with no local pair are not read
    for (int j = 0; j < d.top_k && !any; ++j) any = __ldg(d.pair_pos + t * d.top_k + j) >= 0;
    if (!any) continue;
    const uint4 val = __ldg(reinterpret_cast<const uint4*>(xq + t * cols) + c);
    for (int j = 0; j < d.top_k; ++j) {
      const int32_t pos = __ldg(d.pair_pos + t * d.top_k + j);
      if (pos >= 0) reinterpret_cast<uint4*>(d.a_sorted + pos * cols)[c] = val;
    }
  }
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * kQuantThreads + threadIdx.x; v < tokens * kb; v += stride) {
    const int64_t t = v / kb;
    const int64_t g = v - t * kb;
    const float s = __ldg(xs + t * kb + g);
    for (int j = 0; j < d.top_k; ++j) {
      const int32_t pos = __ldg(d.pair_pos + t * d.top_k + j);
      if (pos >= 0) d.as_t[g * d.rows_cap + pos] = s;
    }
  }
}

int launch_quant(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq, float* scale,
                 int64_t s_row, int64_t s_col, const Dispatch& d, void* stream) {
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (rows < 0 || cols < 0)
    return fail(B2M_ERR_ARG, "quant_g128: negative shape (%lld, %lld)", (long long)rows, (long long)cols);
  if (rows == 0 || cols == 0) return B2M_OK;
  const int64_t gpr = (cols + 127) / 128;
  if (!x || ((!q || !scale) && !d.pair_pos)) return fail(B2M_ERR_ARG, "quant_g128: null pointer");
  if (ldx < cols || (q && ldq < cols))
    return fail(B2M_ERR_ARG, "quant_g128: row strides (ldx=%lld, ldq=%lld) smaller than the row", (long long)ldx,
                (long long)ldq);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool fast = (cols % 128 == 0) && (ldx % 8 == 0) && aligned16(x) &&
                    (!q || ((ldq % 8 == 0) && (reinterpret_cast<uintptr_t>(q) & 7u) == 0));
  const int64_t groups = rows * gpr;
  if (fast) {
    const int64_t warps = (groups + 3) / 4;
    int64_t blocks = (warps * 32 + kQuantThreads - 1) / kQuantThreads;
    blocks = blocks < static_cast<int64_t>(num_sms) * 16 ? blocks : static_cast<int64_t>(num_sms) * 16;
    quant_g128_fast<<<static_cast<unsigned>(blocks), kQuantThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<uint8_t*>(q), ldq, scale, s_row, s_col, groups, gpr,
        d);
  } else {
    if (d.pair_pos) return fail(B2M_ERR_ARG, "quant_dispatch: needs cols %% 128 == 0 and 16-byte aligned rows");
    int64_t blocks = (groups * 32 + kQuantThreads - 1) / kQuantThreads;
    blocks = blocks < static_cast<int64_t>(num_sms) * 16 ? blocks : static_cast<int64_t>(num_sms) * 16;
    quant_g128_generic<<<static_cast<unsigned>(blocks), kQuantThreads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<uint8_t*>(q), ldq, scale, s_row, s_col, rows, cols,
        gpr);
  }
  return check_cuda(cudaGetLastError(), "quant_g128 launch");
}

int check_dispatch(const Dispatch& d, int64_t cols) {
  if (!d.pair_pos || !d.a_sorted || !d.as_t || d.top_k <= 0 || d.rows_cap <= 0)
    return fail(B2M_ERR_ARG, "dispatch: null pointer or empty shape");
  if (cols % 128 || !aligned16(d.a_sorted)) return fail(B2M_ERR_ARG, "dispatch: cols %% 128 and 16B alignment");
  return B2M_OK;
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_quant_g128(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq,
                              float* scale, int64_t ld_scale, void* stream) {
  using namespace b2m;
  const int64_t gpr = (cols + 127) / 128;
  if (ld_scale < gpr) return fail(B2M_ERR_ARG, "quant_g128: ld_scale=%lld < %lld groups", (long long)ld_scale,
                                  (long long)gpr);
  if (rows > 0 && cols > 0 && (!q || !scale)) return fail(B2M_ERR_ARG, "quant_g128: null pointer");
  return launch_quant(x, rows, cols, ldx, q, ldq, scale, ld_scale, 1, Dispatch{}, stream);
}

extern "C" int b2m_quant_g128_t(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq,
                                float* scale_t, int64_t ld_scale_t, void* stream) {
  using namespace b2m;
  if (ld_scale_t < rows) return fail(B2M_ERR_ARG, "quant_g128_t: ld_scale_t=%lld < rows", (long long)ld_scale_t);
  if (rows > 0 && cols > 0 && (!q || !scale_t)) return fail(B2M_ERR_ARG, "quant_g128_t: null pointer");
  return launch_quant(x, rows, cols, ldx, q, ldq, scale_t, 1, ld_scale_t, Dispatch{}, stream);
}

extern "C" int b2m_quant_dispatch(const void* x, int64_t tokens, int64_t hidden, int64_t ldx, const int32_t* pair_pos,
                                  int32_t top_k, void* a_sorted, float* a_scale_t, int64_t rows_cap, void* q_tok,
                                  float* scale_tok_t, int64_t ld_scale_tok_t, void* stream) {
  using namespace b2m;
  const Dispatch d{pair_pos, top_k, static_cast<uint8_t*>(a_sorted), a_scale_t, rows_cap};
  if (tokens == 0) return B2M_OK;
  B2M_TRY(check_dispatch(d, hidden));
  if ((q_tok == nullptr) != (scale_tok_t == nullptr))
    return fail(B2M_ERR_ARG, "quant_dispatch: q_tok and scale_tok_t go together");
  if (scale_tok_t && ld_scale_tok_t < tokens) return fail(B2M_ERR_ARG, "quant_dispatch: ld_scale_tok_t < tokens");
  return launch_quant(x, tokens, hidden, ldx, q_tok, hidden, scale_tok_t, 1, ld_scale_tok_t, d, stream);
}

extern "C" int b2m_dispatch_rows(const void* xq, const float* xs, int64_t tokens, int64_t hidden,
                                 const int32_t* pair_pos, int32_t top_k, void* a_sorted, float* a_scale_t,
                                 int64_t rows_cap, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (tokens == 0) return B2M_OK;
  const Dispatch d{pair_pos, top_k, static_cast<uint8_t*>(a_sorted), a_scale_t, rows_cap};
  B2M_TRY(check_dispatch(d, hidden));
  if (!xq || !xs || !aligned16(xq)) return fail(B2M_ERR_ARG, "dispatch_rows: bad source pointers");
  const int64_t total = tokens * (hidden / 16);
  int64_t blocks = (total + kQuantThreads - 1) / kQuantThreads;
  if (blocks > int64_t(num_sms) * 8) blocks = int64_t(num_sms) * 8;
  dispatch_rows_kernel<<<static_cast<unsigned>(blocks), kQuantThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(xq), xs, tokens, hidden, d);
  return check_cuda(cudaGetLastError(), "dispatch_rows launch");
}
