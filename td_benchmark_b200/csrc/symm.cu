// Peer-memory exchange: the fused all-gather and reduce-scatter of the MoE layer.
//
// The reference moves activations with NCCL all_gather_into_tensor (FP8 bytes +
// fp32 scales, moe_bench/overlap/overlap_forward.py:494-505) and partial outputs
// with reduce_scatter_tensor (:603-608).  Over NVSwitch every peer is one hop away,
// so here each rank writes straight into its peers' memory:
//
//  all-gather   b2m_quant_push quantises the rank's tokens and stores the codes and
//               scales into the same rows of every rank's gather buffer (512-byte warp
//               writes); the last CTA to finish publishes ag_flag[src] = epoch on every
//               rank (system-scope release).  b2m_dispatch_rows_wait then moves rows
//               into expert order, reading a source rank's rows only after its flag
//               (own rows first, bounded acquire spin per source).
//               Tensor parallel alternative: b2m_quant_dispatch_push stores the rows
//               straight into the ranks' expert-sorted operand (the sorted positions
//               agree on every rank), destination by destination with a flag each.
//  reduce-scatter  b2m_combine_push sums each token's top-k rows (+ shared expert) over a
//               column window and stores the bf16 partial into the owning rank's slot
//               for this source; the last CTA publishes rs_flag[src] = epoch on every
//               owner.  b2m_rs_reduce waits for all sources and sums the slots in rank
//               order (deterministic, fp32, one rounding).  b2m_rs_combine is the owner
//               side when the down GEMM stored the pair rows itself (b2m_gemm2_scatter).
//
// Epochs only grow, so flags are never reset.  Buffers need no extra barrier between
// calls: a rank starts call i+1 only after its reduce of call i saw every peer's
// combine of call i, and a peer runs that combine only after it finished reading the
// gather buffer of call i (stream order); symmetrically for the slots.
//
// Symmetric buffers are plain cudaMalloc blocks shared through CUDA IPC handles.
// b2m_copy_async / b2m_copy2d_async / b2m_signal let the host drive the same exchange
// with the copy engines instead (one cudaMemcpyAsync per peer block, then the epoch
// flag as a stream memory operation), which occupies no SM.
#include <cudaTypedefs.h>

#include "b2m_common.cuh"
#include "b2m_host.h"

#include <string.h>

#include <mutex>

namespace b2m {
namespace {

constexpr int kMaxWorld = 8;
constexpr int kThreads = 256;

struct PeerPtrs {
  void* p[kMaxWorld];
};
struct FlagPtrs {
  uint32_t* p[kMaxWorld];
};

// Every thread fences its own peer stores, the CTA syncs, and the last CTA of the
// grid publishes `epoch` to every flag (then re-arms the counter for the next launch).
__device__ __forceinline__ void publish_when_grid_done(int32_t* counter, const FlagPtrs& flags, int world,
                                                       uint32_t epoch) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(counter, 1);
    if (prev == static_cast<int>(gridDim.x) - 1) {
      fence_sys();
      for (int r = 0; r < world; ++r) st_release_sys(flags.p[r], epoch);
      atomicExch(counter, 0);
    }
  }
}

// The rank holding global expert `id` (owner table int32 [experts]); 32 (no rank) for an id
// outside [0, experts).
__device__ __forceinline__ uint32_t expert_rank(const int32_t* __restrict__ owner, int experts, int32_t id) {
  return (id >= 0 && id < experts) ? static_cast<uint32_t>(__ldg(owner + id)) : 32u;
}

// Bit r set when token t routes to at least one expert held by rank r.  Expert parallel
// only: every rank holds the routing of all tokens and the same owner table, so source and
// destination agree on this mask without exchanging any index.
__device__ __forceinline__ uint32_t token_rank_mask(const int32_t* __restrict__ ids, int64_t t, int top_k,
                                                   const int32_t* __restrict__ owner, int experts) {
  uint32_t m = 0;
  for (int j = 0; j < top_k; ++j) {
    const uint32_t r = expert_rank(owner, experts, __ldg(ids + t * top_k + j));
    m |= r < 32u ? 1u << r : 0u;
  }
  return m;
}

// ---------------------------------------------------------------- all-gather push
// Eight lanes share one 128-group (16 consecutive values each), so a warp covers four
// consecutive groups of a row and every store to a destination is one coalesced
// 512-byte warp write (16 B per lane) -- NVLink carries full lines, not 8-byte pieces.
// The group scale and codes are computed exactly as by b2m_quant_g128 (amax / 448,
// IEEE division, clamp, RNE).  Destinations are visited starting after the source's
// own rank so that the ranks do not all hit the same peer first.
__global__ void __launch_bounds__(kThreads)
    quant_push_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t rows, int64_t gpr, int world,
                      const __grid_constant__ PeerPtrs qdst, const __grid_constant__ PeerPtrs sdst, int64_t row0,
                      const __grid_constant__ FlagPtrs flags, uint32_t epoch, int32_t* counter,
                      const int32_t* __restrict__ sparse_ids, int top_k, const int32_t* __restrict__ owner,
                      int experts) {
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;  // group of the warp's four
  const int gl = lane & 7;    // 16-value slice of that group
  const int64_t cols = gpr * 128;
  const int64_t groups = rows * gpr;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  const int src = static_cast<int>(row0 / rows);
  const int first = (src + 1) % world;
  for (int64_t base = warp * 4; base < groups; base += nwarps * 4) {
    const int64_t g = base + sub;
    uint4 raw0 = make_uint4(0, 0, 0, 0), raw1 = raw0;
    int64_t row = 0, gi = 0;
    if (g < groups) {
      row = g / gpr;
      gi = g - row * gpr;
      const uint4* src = reinterpret_cast<const uint4*>(x + row * ldx + gi * 128 + gl * 16);
      raw0 = __ldg(src);
      raw1 = __ldg(src + 1);
    }
    float f0[8], f1[8];
    bf16x8_to_f32(raw0, f0);
    bf16x8_to_f32(raw1, f1);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fmaxf(fabsf(f0[i]), fabsf(f1[i])));
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float s = fmaxf(amax / 448.0f, 1e-12f);
    if (g < groups) {
      const uint2 q0 = quant8(f0, s);
      const uint2 q1 = quant8(f1, s);
      const uint4 q = make_uint4(q0.x, q0.y, q1.x, q1.y);
      const int64_t dst_row = row0 + row;
      // sparse (expert parallel): only the ranks that hold one of the token's experts, and
      // this rank (its own rows also feed its shared expert)
      const uint32_t need =
          sparse_ids ? (token_rank_mask(sparse_ids, dst_row, top_k, owner, experts) | (1u << src)) : ~0u;
      for (int i = 0; i < world; ++i) {
        const int r = first + i < world ? first + i : first + i - world;
        if (!((need >> r) & 1u)) continue;
        *reinterpret_cast<uint4*>(static_cast<uint8_t*>(qdst.p[r]) + dst_row * cols + gi * 128 + gl * 16) = q;
        if (gl == 0) static_cast<float*>(sdst.p[r])[dst_row * gpr + gi] = s;
      }
    }
  }
  publish_when_grid_done(counter, flags, world, epoch);
}

// ---------------------------------------------------------------- all-gather into the peers' sorted operand
// Tensor parallel only: every rank aligns the same topk_ids, so pair_pos (sorted position of
// each (token, j) pair) is the same on every rank and a source can store its quantised rows
// straight into each destination's expert-sorted A operand (top_k copies per token) and the
// K-block-major A scales -- no gather buffer, no dispatch kernel.  Destination-major: the
// grid serves the own rank first, then rank-1, rank-2, ...; a CTA that finished its share of
// a destination counts itself on that destination's counter and moves on, and the last CTA
// publishes the flag.  Destination d thus receives source d+1 first, then d+2, ..., the order
// in which its gate/up GEMM visits the blocks (b2m_block_order).  Quantisation is that of
// b2m_quant_g128 (recomputed per destination from x, which stays in L2).
__global__ void __launch_bounds__(kThreads)
    quant_dispatch_push_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, int64_t rows, int64_t gpr,
                               const int32_t* __restrict__ pair_pos, int top_k, int64_t token0, int world, int rank,
                               const __grid_constant__ PeerPtrs adst, const __grid_constant__ PeerPtrs sdst,
                               int64_t rows_cap, const __grid_constant__ FlagPtrs flags, uint32_t epoch,
                               int32_t* counters) {
  const int lane = threadIdx.x & 31;
  const int sub = lane >> 3;
  const int gl = lane & 7;
  const int64_t cols = gpr * 128;
  const int64_t groups = rows * gpr;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  for (int i = 0; i < world; ++i) {
    const int d = (rank - i + world) % world;
    uint8_t* a = static_cast<uint8_t*>(adst.p[d]);
    float* sc = static_cast<float*>(sdst.p[d]);
    for (int64_t base = warp * 4; base < groups; base += nwarps * 4) {
      const int64_t g = base + sub;
      uint4 raw0 = make_uint4(0, 0, 0, 0), raw1 = raw0;
      int64_t row = 0, gi = 0;
      if (g < groups) {
        row = g / gpr;
        gi = g - row * gpr;
        const uint4* src = reinterpret_cast<const uint4*>(x + row * ldx + gi * 128 + gl * 16);
        raw0 = __ldg(src);
        raw1 = __ldg(src + 1);
      }
      float f0[8], f1[8];
      bf16x8_to_f32(raw0, f0);
      bf16x8_to_f32(raw1, f1);
      float amax = 0.0f;
#pragma unroll
      for (int u = 0; u < 8; ++u) amax = fmaxf(amax, fmaxf(fabsf(f0[u]), fabsf(f1[u])));
#pragma unroll
      for (int off = 4; off >= 1; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float s = fmaxf(amax / 448.0f, 1e-12f);
      if (g < groups) {
        const uint2 q0 = quant8(f0, s);
        const uint2 q1 = quant8(f1, s);
        const uint4 q = make_uint4(q0.x, q0.y, q1.x, q1.y);
        const int32_t* pp = pair_pos + (token0 + row) * top_k;
        for (int j = 0; j < top_k; ++j) {
          const int64_t pos = __ldg(pp + j);
          if (pos < 0) continue;
          *reinterpret_cast<uint4*>(a + pos * cols + gi * 128 + gl * 16) = q;
          if (gl == 0) sc[gi * rows_cap + pos] = s;
        }
      }
    }
    __threadfence_system();  // this thread's stores to destination d are visible system-wide
    __syncthreads();
    if (threadIdx.x == 0) {
      const int prev = atomicAdd(counters + d, 1);
      if (prev == static_cast<int>(gridDim.x) - 1) {  // the grid is done with destination d
        fence_sys();
        st_release_sys(flags.p[d], epoch);
        atomicExch(counters + d, 0);
      }
    }
  }
}

// ---------------------------------------------------------------- dispatch with arrival waits
// One warp per token row.  Tokens are visited starting at this rank's own rows.
__global__ void __launch_bounds__(kThreads)
    dispatch_wait_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ xs, int64_t tokens, int64_t cols,
                         const int32_t* __restrict__ pair_pos, int top_k, uint8_t* __restrict__ a_sorted,
                         float* __restrict__ as_t, int64_t rows_cap, const uint32_t* flags, int world, int rank,
                         uint32_t epoch, int32_t* status, uint64_t timeout_ns) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  const int64_t per_rank = tokens / world;
  const int64_t vec = cols / 16;
  const int64_t kb = cols / 128;
  uint32_t ready = 0;  // bit r: rank r's rows have arrived (for this warp)
  bool ok = true;
  for (int64_t i = warp; i < tokens && ok; i += nwarps) {
    const int64_t t = (i + static_cast<int64_t>(rank) * per_rank) % tokens;
    const int src = static_cast<int>(t / per_rank);
    if (!(ready & (1u << src))) {
      int good = 1;
      if (lane == 0) good = wait_flag_geq(flags + src, epoch, timeout_ns, status, B2M_STATUS_TIMEOUT_PEER);
      good = __shfl_sync(0xffffffffu, good, 0);
      __syncwarp();  // lane 0's acquire orders the other lanes' reads of this source's rows
      if (!good) {
        ok = false;
        break;
      }
      ready |= 1u << src;
    }
    int32_t pos[8];
    bool any = false;
    for (int j = 0; j < top_k && j < 8; ++j) {
      pos[j] = __ldg(pair_pos + t * top_k + j);
      any = any || pos[j] >= 0;
    }
    if (!any) continue;  // no pair of this token is local (expert parallel): its row is not read
    for (int64_t c = lane; c < vec; c += 32) {
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(xq + t * cols + c * 16));
      for (int j = 0; j < top_k && j < 8; ++j)
        if (pos[j] >= 0) reinterpret_cast<uint4*>(a_sorted + pos[j] * cols)[c] = v;
    }
    for (int64_t g = lane; g < kb; g += 32) {
      const float sv = __ldcg(xs + t * kb + g);
      for (int j = 0; j < top_k && j < 8; ++j)
        if (pos[j] >= 0) as_t[g * rows_cap + pos[j]] = sv;
    }
  }
}

// ---------------------------------------------------------------- reduce-scatter push
// One warp per token (pair mask read once), lanes over the column window 8 at a time;
// the combined row goes to the owner's slot for this source.
template <bool kWide>
__global__ void __launch_bounds__(kThreads)
    combine_push_kernel(const __nv_bfloat16* __restrict__ staged, int64_t tokens, int top_k, int64_t hidden,
                        int64_t col0, int64_t col1, const int32_t* __restrict__ topk_ids,
                        const int32_t* __restrict__ expert_map, const __nv_bfloat16* __restrict__ shared, int world,
                        int rank, const __grid_constant__ PeerPtrs slots, const __grid_constant__ FlagPtrs flags,
                        uint32_t epoch, int32_t* counter, int sparse) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  const int64_t per_rank = tokens / world;
  for (int64_t t = warp; t < tokens; t += nwarps) {
    const uint32_t mask = local_pair_mask(topk_ids, expert_map, t, top_k, lane);
    if (sparse && mask == 0) continue;  // no local pair: the owner does not read this slot
    const int owner = static_cast<int>(t / per_rank);
    const int64_t slot_row = static_cast<int64_t>(rank) * per_rank + (t - owner * per_rank);
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(slots.p[owner]) + slot_row * hidden;
#pragma unroll 2
    for (int64_t c = col0 + lane * 8; c < col1; c += 256)
      *reinterpret_cast<uint4*>(dst + c) =
          combine_vec<kWide>(staged, t, top_k, hidden, c, mask, topk_ids, expert_map, shared);
  }
  if (counter) publish_when_grid_done(counter, flags, world, epoch);
}

__global__ void __launch_bounds__(kThreads)
    rs_reduce_kernel(const __nv_bfloat16* __restrict__ slots, int64_t rows, int64_t hidden, int world, int nflags,
                     const uint32_t* flags, uint32_t epoch, const __nv_bfloat16* __restrict__ add,
                     __nv_bfloat16* __restrict__ out, int32_t* status, uint64_t timeout_ns) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < nflags && !wait_flag_geq(flags + threadIdx.x, epoch, timeout_ns, status, B2M_STATUS_TIMEOUT_PEER))
    s_ok = 0;
  __syncthreads();
  if (!s_ok) return;  // status already records the timeout
  const int64_t vec = hidden / 8;
  const int64_t total = rows * vec;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t t = v / vec;
    const int64_t c = (v - t * vec) * 8;
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < world; ++r)
      acc_bf16x8(__ldcg(reinterpret_cast<const uint4*>(slots + (static_cast<int64_t>(r) * rows + t) * hidden + c)), a);
    if (add) acc_bf16x8(*reinterpret_cast<const uint4*>(add + t * hidden + c), a);
    *reinterpret_cast<uint4*>(out + t * hidden + c) = pack_bf16x8(a);
  }
}

// Owner side of the scattered reduce-scatter (b2m_gemm2_scatter wrote every pair row of this
// owner's tokens into recv): out[t] = bf16(sum over sources s, then pairs j, of
// recv[(s * rows + t) * top_k + j] + add[t]) in fp32 with one rounding, after every flag
// reached epoch.  One warp per token; all loads of a group of eight rows are issued first.
__global__ void __launch_bounds__(kThreads)
    rs_combine_kernel(const __nv_bfloat16* __restrict__ recv, int64_t rows, int top_k, int64_t hidden, int nsrc,
                      const uint32_t* flags, int nflags, uint32_t epoch, const __nv_bfloat16* __restrict__ add,
                      __nv_bfloat16* __restrict__ out, int32_t* status, uint64_t timeout_ns) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < nflags && !wait_flag_geq(flags + threadIdx.x, epoch, timeout_ns, status, B2M_STATUS_TIMEOUT_PEER))
    s_ok = 0;
  __syncthreads();
  if (!s_ok) return;  // status already records the timeout
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  const int nrow = nsrc * top_k;
  for (int64_t t = warp; t < rows; t += nwarps) {
    for (int64_t c = lane * 8; c < hidden; c += 256) {
      float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int i0 = 0; i0 < nrow; i0 += 8) {
        uint4 u[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (i0 + i < nrow) {
            const int src = (i0 + i) / top_k, j = (i0 + i) - src * top_k;
            u[i] = __ldcg(reinterpret_cast<const uint4*>(recv + ((src * rows + t) * top_k + j) * hidden + c));
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (i0 + i < nrow) acc_bf16x8(u[i], a);
      }
      if (add) acc_bf16x8(*reinterpret_cast<const uint4*>(add + t * hidden + c), a);
      *reinterpret_cast<uint4*>(out + t * hidden + c) = pack_bf16x8(a);
    }
  }
}

// ---------------------------------------------------------------- reduce-scatter push, FP8 payload
// The b3 variant of the reduce-scatter (moe_bench/overlap/overlap_forward.py:900-946): each
// token's combined partial row -- its local top-k rows (+ shared expert) summed in fp32 and
// rounded to bf16, which is what the reference quantises -- is quantised per 128 columns by the
// activation rule (amax / 448 floored at 1e-12, IEEE division, clamp, RNE e4m3), and the codes
// (hidden bytes) and fp32 scales (hidden / 128) go to the owner's FP8 slot for this source:
// H + H/32 bytes per row instead of 2H.  One warp per token; in each 256-column step lanes
// 0-15 hold one 128-group (8 values each) and lanes 16-31 the next.
template <bool kWide>
__global__ void __launch_bounds__(kThreads)
    combine_push_fp8_kernel(const __nv_bfloat16* __restrict__ staged, int64_t tokens, int top_k, int64_t hidden,
                            const int32_t* __restrict__ topk_ids, const int32_t* __restrict__ expert_map,
                            const __nv_bfloat16* __restrict__ shared, int world, int rank,
                            const __grid_constant__ PeerPtrs codes, const __grid_constant__ PeerPtrs scales,
                            const __grid_constant__ FlagPtrs flags, uint32_t epoch, int32_t* counter, int sparse) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  const int64_t per_rank = tokens / world;
  const int64_t gpr = hidden / 128;
  for (int64_t t = warp; t < tokens; t += nwarps) {
    const uint32_t mask = local_pair_mask(topk_ids, expert_map, t, top_k, lane);
    if (sparse && mask == 0) continue;  // no local pair: the owner does not read this slot
    const int owner = static_cast<int>(t / per_rank);
    const int64_t slot_row = static_cast<int64_t>(rank) * per_rank + (t - owner * per_rank);
    uint8_t* qrow = static_cast<uint8_t*>(codes.p[owner]) + slot_row * hidden;
    float* srow = static_cast<float*>(scales.p[owner]) + slot_row * gpr;
    for (int64_t c0 = 0; c0 < hidden; c0 += 256) {
      const int64_t c = c0 + lane * 8;
      const bool in = c < hidden;  // hidden % 128 == 0: a half-warp is all in or all out
      uint4 v = make_uint4(0, 0, 0, 0);
      if (in) v = combine_vec<kWide>(staged, t, top_k, hidden, c, mask, topk_ids, expert_map, shared);
      float f[8];
      bf16x8_to_f32(v, f);
      const float scale = fmaxf(halfwarp_amax(f) / 448.0f, 1e-12f);
      if (in) {
        *reinterpret_cast<uint2*>(qrow + c) = quant8(f, scale);
        if ((lane & 15) == 0) srow[c / 128] = scale;
      }
    }
  }
  if (counter) publish_when_grid_done(counter, flags, world, epoch);
}

// Owner side of the FP8 reduce-scatter: out[t] = bf16(sum over sources r in rank order of
// e4m3(codes[r][t]) * scale[r][t][group], + add[t]) in fp32 with one rounding, after every
// source's flag reached epoch (flags == nullptr: the slots were filled by a collective that
// has already completed on this stream).
__global__ void __launch_bounds__(kThreads)
    rs_reduce_fp8_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales, int64_t rows,
                         int64_t hidden, int world, const uint32_t* flags, uint32_t epoch,
                         const __nv_bfloat16* __restrict__ add, __nv_bfloat16* __restrict__ out, int32_t* status,
                         uint64_t timeout_ns) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (flags && threadIdx.x < world && !wait_flag_geq(flags + threadIdx.x, epoch, timeout_ns, status,
                                                     B2M_STATUS_TIMEOUT_PEER))
    s_ok = 0;
  __syncthreads();
  if (!s_ok) return;  // status already records the timeout
  const int64_t vec = hidden / 8;
  const int64_t gpr = hidden / 128;
  const int64_t total = rows * vec;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; v < total;
       v += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t t = v / vec;
    const int64_t c = (v - t * vec) * 8;
    float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < world; ++r) {
      const int64_t row = static_cast<int64_t>(r) * rows + t;
      const uint2 q = __ldcg(reinterpret_cast<const uint2*>(codes + row * hidden + c));
      const float sc = __ldcg(scales + row * gpr + c / 128);
      const uint32_t w[2] = {q.x, q.y};
#pragma unroll
      for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(
              static_cast<__nv_fp8x2_storage_t>((w[i] >> (16 * j)) & 0xFFFFu), __NV_E4M3);
          const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&h));
          // dequantise, then add: two roundings, as the reference's (codes * scales).sum(0)
          // (no fused multiply-add)
          a[4 * i + 2 * j] = __fadd_rn(a[4 * i + 2 * j], __fmul_rn(d.x, sc));
          a[4 * i + 2 * j + 1] = __fadd_rn(a[4 * i + 2 * j + 1], __fmul_rn(d.y, sc));
        }
      }
    }
    if (add) acc_bf16x8(*reinterpret_cast<const uint4*>(add + t * hidden + c), a);
    *reinterpret_cast<uint4*>(out + t * hidden + c) = pack_bf16x8(a);
  }
}

// Owner side of the sparse expert-parallel reduce-scatter, either payload: one warp per
// owned token; the sources summed are exactly the ranks holding one of the token's experts
// (the same mask the sources used to decide whether to push), in rank order, fp32, plus
// `add`, one rounding -- so the result equals the dense reduce, in which the other sources'
// slots hold zero partials.  ids = the routing rows of this owner's tokens.
template <bool kFp8>
__global__ void __launch_bounds__(kThreads)
    rs_reduce_sparse_kernel(const void* __restrict__ slots, const float* __restrict__ scales, int64_t rows,
                            int64_t hidden, int world, const int32_t* __restrict__ ids, int top_k,
                            const int32_t* __restrict__ owner, int experts,
                            const uint32_t* flags, uint32_t epoch, const __nv_bfloat16* __restrict__ add,
                            __nv_bfloat16* __restrict__ out, int32_t* status, uint64_t timeout_ns) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (flags && threadIdx.x < world && !wait_flag_geq(flags + threadIdx.x, epoch, timeout_ns, status,
                                                     B2M_STATUS_TIMEOUT_PEER))
    s_ok = 0;
  __syncthreads();
  if (!s_ok) return;  // status already records the timeout
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * kThreads) >> 5;
  const int64_t gpr = hidden / 128;
  for (int64_t t = warp; t < rows; t += nwarps) {
    const uint32_t rk = lane < top_k ? expert_rank(owner, experts, __ldg(ids + t * top_k + lane)) : 32u;
    const uint32_t mine = rk < 32u ? 1u << rk : 0u;
    const uint32_t srcs = __reduce_or_sync(0xffffffffu, mine);
    for (int64_t c = lane * 8; c < hidden; c += 256) {
      float a[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int r = 0; r < world; ++r) {
        if (!((srcs >> r) & 1u)) continue;
        const int64_t row = static_cast<int64_t>(r) * rows + t;
        if (kFp8) {
          const uint2 q = __ldcg(reinterpret_cast<const uint2*>(static_cast<const uint8_t*>(slots) + row * hidden + c));
          const float sc = __ldcg(scales + row * gpr + c / 128);
          const uint32_t w[2] = {q.x, q.y};
#pragma unroll
          for (int i = 0; i < 2; ++i) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(
                  static_cast<__nv_fp8x2_storage_t>((w[i] >> (16 * j)) & 0xFFFFu), __NV_E4M3);
              const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&h));
              a[4 * i + 2 * j] = __fadd_rn(a[4 * i + 2 * j], __fmul_rn(d.x, sc));
              a[4 * i + 2 * j + 1] = __fadd_rn(a[4 * i + 2 * j + 1], __fmul_rn(d.y, sc));
            }
          }
        } else {
          acc_bf16x8(__ldcg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(slots) + row * hidden + c)),
                     a);
        }
      }
      if (add) acc_bf16x8(*reinterpret_cast<const uint4*>(add + t * hidden + c), a);
      *reinterpret_cast<uint4*>(out + t * hidden + c) = pack_bf16x8(a);
    }
  }
}

int grid_for(int64_t work, int num_sms, int per_sm) {
  int64_t b = (work + kThreads - 1) / kThreads;
  if (b > int64_t(num_sms) * per_sm) b = int64_t(num_sms) * per_sm;
  return static_cast<int>(b < 1 ? 1 : b);
}

}  // namespace
}  // namespace b2m

// ---------------------------------------------------------------- allocation-free all-gather push
// Callers that cannot allocate device memory (a runtime that owns every byte through
// its own arena, or code that must not call cudaMalloc at all) cannot hand
// b2m_quant_push its completion counter.  b2m_quant_push_noalloc keeps that counter
// in this library's own static device memory instead: 64 int32 (256 bytes) per GPU
// that loads the library, held until the process exits; one call uses one counter
// (independent of rows and hidden) and world is limited to 8 as for b2m_quant_push.
// Every call shares that counter: calls that overlap on the GPU (other streams,
// other threads) race on it, so a caller must serialise them.
namespace b2m {
namespace {
constexpr int kPushScratchInts = 64;
constexpr int kPushScratchNeeded = 1;  // one grid-completion counter per call
static __device__ __align__(256) int32_t g_push_scratch[kPushScratchInts];

// cuStreamWriteValue32 from the driver (the runtime is linked statically and has no
// equivalent): a stream memory operation that writes a 32-bit value after all earlier
// work on the stream, preceded by a fence with the effect of __threadfence_system, and
// executed by the GPU front end rather than by an SM.
int stream_write_fn(PFN_cuStreamWriteValue32_v11070* out) {
  void* p = nullptr;
  B2M_TRY(driver_entry("cuStreamWriteValue32", &p));
  *out = reinterpret_cast<PFN_cuStreamWriteValue32_v11070>(p);
  return B2M_OK;
}

// Device address of g_push_scratch on the current device, looked up once per device
// (the host-side name is only a stand-in and must never be handed to a kernel).
int push_scratch_ptr(int32_t** out) {
  static std::mutex mu;
  static int32_t* addr[64] = {nullptr};
  int dev = 0;
  B2M_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  if (dev < 0 || dev >= 64) return fail(B2M_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    B2M_TRY(check_cuda(cudaGetSymbolAddress(&p, g_push_scratch), "cudaGetSymbolAddress(g_push_scratch)"));
    addr[dev] = static_cast<int32_t*>(p);
  }
  *out = addr[dev];
  return B2M_OK;
}
}  // namespace
}  // namespace b2m

extern "C" {

int b2m_symm_alloc(int64_t bytes, void** dev_ptr) {
  using namespace b2m;
  if (bytes <= 0 || !dev_ptr) return fail(B2M_ERR_ARG, "symm_alloc: bad arguments");
  B2M_TRY(check_cuda(cudaMalloc(dev_ptr, static_cast<size_t>(bytes)), "symm_alloc: cudaMalloc"));
  return check_cuda(cudaMemset(*dev_ptr, 0, static_cast<size_t>(bytes)), "symm_alloc: cudaMemset");
}

int b2m_symm_free(void* dev_ptr) {
  using namespace b2m;
  if (!dev_ptr) return B2M_OK;
  return check_cuda(cudaFree(dev_ptr), "symm_free: cudaFree");
}

int b2m_ipc_handle(void* dev_ptr, void* handle_out) {
  using namespace b2m;
  if (!dev_ptr || !handle_out) return fail(B2M_ERR_ARG, "ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  B2M_TRY(check_cuda(cudaIpcGetMemHandle(&h, dev_ptr), "cudaIpcGetMemHandle"));
  memcpy(handle_out, &h, sizeof(h));
  return B2M_OK;
}

int b2m_ipc_open(const void* handle, void** peer_ptr) {
  using namespace b2m;
  if (!handle || !peer_ptr) return fail(B2M_ERR_ARG, "ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

int b2m_ipc_close(void* peer_ptr) {
  using namespace b2m;
  if (!peer_ptr) return B2M_OK;
  return check_cuda(cudaIpcCloseMemHandle(peer_ptr), "cudaIpcCloseMemHandle");
}

int b2m_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  using namespace b2m;
  if (bytes < 0 || (bytes > 0 && (!dst || !src))) return fail(B2M_ERR_ARG, "copy_async: bad arguments");
  if (bytes == 0) return B2M_OK;
  return check_cuda(cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault,
                                    static_cast<cudaStream_t>(stream)),
                    "copy_async: cudaMemcpyAsync");
}

int b2m_copy2d_async(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                     void* stream) {
  using namespace b2m;
  if (width < 0 || height < 0 || dpitch < width || spitch < width || ((width && height) && (!dst || !src)))
    return fail(B2M_ERR_ARG, "copy2d_async: bad arguments");
  if (width == 0 || height == 0) return B2M_OK;
  return check_cuda(cudaMemcpy2DAsync(dst, static_cast<size_t>(dpitch), src, static_cast<size_t>(spitch),
                                      static_cast<size_t>(width), static_cast<size_t>(height), cudaMemcpyDefault,
                                      static_cast<cudaStream_t>(stream)),
                    "copy2d_async: cudaMemcpy2DAsync");
}

}  // extern "C"

namespace b2m {
namespace {
// Argument checks of b2m_quant_push other than the counter (shared with the no-alloc variant).
int check_quant_push(const void* x, int64_t rows, int64_t hidden, int64_t ldx, int32_t world, void* const* q_dst,
                     void* const* s_dst, uint32_t* const* flag_dst, const char* who) {
  if (world < 1 || world > kMaxWorld) return fail(B2M_ERR_ARG, "%s: world=%d outside [1, 8]", who, world);
  if (rows <= 0 || hidden <= 0 || hidden % 128 || ldx < hidden || ldx % 8 || !x || !aligned16(x) || !q_dst ||
      !s_dst || !flag_dst)
    return fail(B2M_ERR_ARG, "%s: bad shape/pointers (hidden %% 128 == 0, 16-byte rows)", who);
  for (int r = 0; r < world; ++r)
    if (!q_dst[r] || !s_dst[r] || !flag_dst[r]) return fail(B2M_ERR_ARG, "%s: null peer pointer %d", who, r);
  return B2M_OK;
}
}  // namespace
}  // namespace b2m

extern "C" {

int b2m_quant_push(const void* x, int64_t rows, int64_t hidden, int64_t ldx, int32_t world, void* const* q_dst,
                   void* const* s_dst, int64_t row0, uint32_t* const* flag_dst, uint32_t epoch, int32_t* counter,
                   void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  B2M_TRY(check_quant_push(x, rows, hidden, ldx, world, q_dst, s_dst, flag_dst, "quant_push"));
  if (!counter) return fail(B2M_ERR_ARG, "quant_push: null counter");
  PeerPtrs q{}, s{};
  FlagPtrs f{};
  for (int r = 0; r < world; ++r) {
    q.p[r] = q_dst[r];
    s.p[r] = s_dst[r];
    f.p[r] = flag_dst[r];
  }
  const int64_t groups = rows * (hidden / 128);
  quant_push_kernel<<<grid_for(groups * 8, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, rows, hidden / 128, world, q, s, row0, f, epoch, counter, nullptr, 0,
      nullptr, 0);
  return check_cuda(cudaGetLastError(), "quant_push launch");
}

int b2m_quant_push_sparse(const void* x, int64_t rows, int64_t hidden, int64_t ldx, int32_t world, void* const* q_dst,
                          void* const* s_dst, int64_t row0, uint32_t* const* flag_dst, uint32_t epoch, int32_t* counter,
                          const int32_t* topk_ids, int32_t top_k, const int32_t* expert_owner, int32_t num_experts,
                          void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  B2M_TRY(check_quant_push(x, rows, hidden, ldx, world, q_dst, s_dst, flag_dst, "quant_push_sparse"));
  if (!counter || !topk_ids || !expert_owner || top_k < 1 || top_k > 32 || num_experts < 1 || row0 % rows)
    return fail(B2M_ERR_ARG, "quant_push_sparse: need counter, topk_ids, expert_owner, 1 <= top_k <= 32, "
                             "num_experts >= 1 and row0 a multiple of rows");
  PeerPtrs q{}, s{};
  FlagPtrs f{};
  for (int r = 0; r < world; ++r) {
    q.p[r] = q_dst[r];
    s.p[r] = s_dst[r];
    f.p[r] = flag_dst[r];
  }
  const int64_t groups = rows * (hidden / 128);
  quant_push_kernel<<<grid_for(groups * 8, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, rows, hidden / 128, world, q, s, row0, f, epoch, counter, topk_ids,
      top_k, expert_owner, num_experts);
  return check_cuda(cudaGetLastError(), "quant_push_sparse launch");
}

int b2m_quant_push_noalloc(const void* x, int64_t rows, int64_t hidden, int64_t ldx, int32_t world,
                           void* const* q_dst, void* const* s_dst, int64_t row0, uint32_t* const* flag_dst,
                           uint32_t epoch, void* stream) {
  using namespace b2m;
  static_assert(kPushScratchNeeded <= kPushScratchInts, "scratch capacity");
  if (world < 1 || world > kMaxWorld)
    return fail(B2M_ERR_ARG, "quant_push_noalloc: world=%d outside [1, %d]", world, kMaxWorld);
  // The scratch need is one counter whatever rows/hidden are, so no problem size can
  // outgrow the static array; the peer table bounds world (checked above).  Every other
  // argument is checked before anything is enqueued, so a rejected call leaves the
  // caller's stream untouched.
  B2M_TRY(check_quant_push(x, rows, hidden, ldx, world, q_dst, s_dst, flag_dst, "quant_push_noalloc"));
  int32_t* counter = nullptr;
  B2M_TRY(require_sm100(nullptr));
  B2M_TRY(push_scratch_ptr(&counter));
  // The counter must start at zero; a previous call normally leaves it zero, but one
  // that was aborted might not, so clear it on the stream (no allocation involved).
  B2M_TRY(check_cuda(cudaMemsetAsync(counter, 0, sizeof(int32_t) * kPushScratchNeeded,
                                     static_cast<cudaStream_t>(stream)),
                     "quant_push_noalloc: clear scratch"));
  return b2m_quant_push(x, rows, hidden, ldx, world, q_dst, s_dst, row0, flag_dst, epoch, counter, stream);
}

int b2m_quant_dispatch_push(const void* x, int64_t rows, int64_t hidden, int64_t ldx, const int32_t* pair_pos,
                            int32_t top_k, int64_t token0, int32_t world, int32_t rank, void* const* a_dst,
                            void* const* s_dst, int64_t rows_cap, uint32_t* const* flag_dst, uint32_t epoch,
                            int32_t* counters, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return fail(B2M_ERR_ARG, "quant_dispatch_push: world=%d / rank=%d outside [1, 8]", world, rank);
  if (rows <= 0 || hidden <= 0 || hidden % 128 || ldx < hidden || ldx % 8 || top_k < 1 || token0 < 0 ||
      rows_cap <= 0 || !x || !aligned16(x) || !pair_pos || !a_dst || !s_dst || !flag_dst || !counters)
    return fail(B2M_ERR_ARG, "quant_dispatch_push: bad shape/pointers (hidden %% 128 == 0, 16-byte rows)");
  PeerPtrs a{}, sc{};
  FlagPtrs f{};
  for (int r = 0; r < world; ++r) {
    if (!a_dst[r] || !s_dst[r] || !flag_dst[r] || !aligned16(a_dst[r]))
      return fail(B2M_ERR_ARG, "quant_dispatch_push: bad peer pointer %d", r);
    a.p[r] = a_dst[r];
    sc.p[r] = s_dst[r];
    f.p[r] = flag_dst[r];
  }
  const int64_t groups = rows * (hidden / 128);
  quant_dispatch_push_kernel<<<grid_for(groups * 8, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(x), ldx, rows, hidden / 128, pair_pos, top_k, token0, world, rank, a, sc,
      rows_cap, f, epoch, counters);
  return check_cuda(cudaGetLastError(), "quant_dispatch_push launch");
}

int b2m_dispatch_rows_wait(const void* xq, const float* xs, int64_t tokens, int64_t hidden, const int32_t* pair_pos,
                           int32_t top_k, void* a_sorted, float* a_scale_t, int64_t rows_cap, const uint32_t* flags,
                           int32_t world, int32_t rank, uint32_t epoch, int32_t* dev_status, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || tokens % world || top_k < 1 || top_k > 8)
    return fail(B2M_ERR_ARG, "dispatch_rows_wait: bad world/rank/top_k (top_k <= 8, tokens %% world == 0)");
  if (!xq || !xs || !pair_pos || !a_sorted || !a_scale_t || !flags || hidden % 128 || !aligned16(xq) ||
      !aligned16(a_sorted))
    return fail(B2M_ERR_ARG, "dispatch_rows_wait: bad pointers/shape");
  if (tokens == 0) return B2M_OK;
  dispatch_wait_kernel<<<grid_for(tokens * 32, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(xq), xs, tokens, hidden, pair_pos, top_k, static_cast<uint8_t*>(a_sorted),
      a_scale_t, rows_cap, flags, world, rank, epoch, dev_status, timeout_ns());
  return check_cuda(cudaGetLastError(), "dispatch_rows_wait launch");
}

int b2m_combine_push(const void* staged, int64_t tokens, int32_t top_k, int64_t hidden, int64_t col_begin,
                     int64_t col_end, const int32_t* topk_ids, const int32_t* expert_map, const void* shared,
                     int32_t world, int32_t rank, void* const* slot_dst, uint32_t* const* flag_dst, uint32_t epoch,
                     int32_t* counter, int32_t max_ctas, int32_t sparse, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || tokens <= 0 || tokens % world ||
      hidden % 8 || top_k <= 0)
    return fail(B2M_ERR_ARG, "combine_push: bad shape (tokens %% world == 0, hidden %% 8 == 0)");
  if (!staged || !slot_dst || (counter && !flag_dst) || (expert_map && !topk_ids) || !aligned16(staged) ||
      (sparse && !expert_map))
    return fail(B2M_ERR_ARG, "combine_push: bad pointers (sparse needs the expert map)");
  if (col_end <= 0) col_end = hidden;
  if (col_begin < 0 || col_begin % 8 || col_end % 8 || col_end > hidden || col_begin >= col_end)
    return fail(B2M_ERR_ARG, "combine_push: column window [%lld, %lld) outside [0, %lld) or not 8-aligned",
                (long long)col_begin, (long long)col_end, (long long)hidden);
  PeerPtrs sl{};
  FlagPtrs f{};
  for (int r = 0; r < world; ++r) {
    if (!slot_dst[r] || (counter && !flag_dst[r]) || !aligned16(slot_dst[r]))
      return fail(B2M_ERR_ARG, "combine_push: bad peer pointer %d", r);
    sl.p[r] = slot_dst[r];
    f.p[r] = counter ? flag_dst[r] : nullptr;
  }
  int grid = grid_for(tokens * 32, num_sms, 8);  // a warp per token
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  (top_k > 32 ? combine_push_kernel<true> : combine_push_kernel<false>)<<<grid, kThreads, 0,
                                                                          static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(staged), tokens, top_k, hidden, col_begin, col_end, topk_ids, expert_map,
      static_cast<const __nv_bfloat16*>(shared), world, rank, sl, f, epoch, counter, sparse);
  return check_cuda(cudaGetLastError(), "combine_push launch");
}

int b2m_signal(uint32_t* const* flag_dst, int32_t world, uint32_t epoch, void* stream) {
  using namespace b2m;
  if (world < 1 || world > kMaxWorld || !flag_dst) return fail(B2M_ERR_ARG, "signal: bad arguments");
  PFN_cuStreamWriteValue32_v11070 write = nullptr;
  B2M_TRY(stream_write_fn(&write));
  for (int r = 0; r < world; ++r) {
    if (!flag_dst[r]) return fail(B2M_ERR_ARG, "signal: null flag %d", r);
    const CUresult rc = write(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag_dst[r]), epoch,
                              CU_STREAM_WRITE_VALUE_DEFAULT);
    if (rc != CUDA_SUCCESS) return fail(B2M_ERR_CUDA, "signal: cuStreamWriteValue32 failed (%d) on flag %d", (int)rc, r);
  }
  return B2M_OK;
}

int b2m_rs_combine(const void* recv, int64_t rows, int32_t top_k, int64_t hidden, int32_t nsrc,
                   const uint32_t* flags, int32_t nflags, uint32_t epoch, const void* add, void* out,
                   int32_t* dev_status, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (rows <= 0 || hidden <= 0 || hidden % 8 || top_k < 1 || nsrc < 1 || nsrc > kMaxWorld || nflags < 1 ||
      nflags > kThreads || !recv || !flags || !out || !aligned16(recv) || !aligned16(out) || (add && !aligned16(add)))
    return fail(B2M_ERR_ARG, "rs_combine: bad shape/pointers (hidden %% 8 == 0, 1 <= nsrc <= 8, 16-byte rows)");
  rs_combine_kernel<<<grid_for(rows * 32, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(recv), rows, top_k, hidden, nsrc, flags, nflags, epoch,
      static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out), dev_status, timeout_ns());
  return check_cuda(cudaGetLastError(), "rs_combine launch");
}

int b2m_rs_reduce(const void* slots, int64_t rows, int64_t hidden, int32_t world, int32_t nchunks,
                  const uint32_t* flags, uint32_t epoch, const void* add, void* out, const int32_t* topk_ids,
                  int32_t top_k, const int32_t* expert_owner, int32_t num_experts, int32_t* dev_status, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (world < 1 || world > kMaxWorld || rows <= 0 || hidden % 8 || !slots || !flags || !out ||
      !aligned16(slots) || !aligned16(out) || (add && !aligned16(add)) || nchunks < 1 || nchunks * world > kThreads)
    return fail(B2M_ERR_ARG, "rs_reduce: bad shape/pointers/chunks");
  if (topk_ids) {  // sparse expert-parallel reduce: only the sources holding one of the token's experts
    if (nchunks != 1 || top_k < 1 || top_k > 32 || !expert_owner || num_experts < 1)
      return fail(B2M_ERR_ARG, "rs_reduce: sparse reduce needs nchunks == 1, 1 <= top_k <= 32 and the owner table");
    rs_reduce_sparse_kernel<false><<<grid_for(rows * 32, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        slots, nullptr, rows, hidden, world, topk_ids, top_k, expert_owner, num_experts, flags, epoch,
        static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out), dev_status, timeout_ns());
    return check_cuda(cudaGetLastError(), "rs_reduce (sparse) launch");
  }
  rs_reduce_kernel<<<grid_for(rows * (hidden / 8), num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(slots), rows, hidden, world, nchunks * world, flags, epoch,
      static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out), dev_status, timeout_ns());
  return check_cuda(cudaGetLastError(), "rs_reduce launch");
}

int b2m_combine_push_fp8(const void* staged, int64_t tokens, int32_t top_k, int64_t hidden, const int32_t* topk_ids,
                         const int32_t* expert_map, const void* shared, int32_t world, int32_t rank,
                         void* const* code_dst, void* const* scale_dst, uint32_t* const* flag_dst, uint32_t epoch,
                         int32_t* counter, int32_t sparse, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || tokens <= 0 || tokens % world ||
      hidden <= 0 || hidden % 128 || top_k <= 0)
    return fail(B2M_ERR_ARG, "combine_push_fp8: bad shape (tokens %% world == 0, hidden %% 128 == 0)");
  if (!staged || !code_dst || !scale_dst || (counter && !flag_dst) || (expert_map && !topk_ids) ||
      !aligned16(staged) || (shared && !aligned16(shared)) || (sparse && !expert_map))
    return fail(B2M_ERR_ARG, "combine_push_fp8: bad pointers (sparse needs the expert map)");
  PeerPtrs q{}, sc{};
  FlagPtrs f{};
  for (int r = 0; r < world; ++r) {
    if (!code_dst[r] || !scale_dst[r] || (counter && !flag_dst[r]) ||
        (reinterpret_cast<uintptr_t>(code_dst[r]) & 7u) || (reinterpret_cast<uintptr_t>(scale_dst[r]) & 3u))
      return fail(B2M_ERR_ARG, "combine_push_fp8: bad peer pointer %d (codes 8-byte, scales 4-byte aligned)", r);
    q.p[r] = code_dst[r];
    sc.p[r] = scale_dst[r];
    f.p[r] = counter ? flag_dst[r] : nullptr;
  }
  (top_k > 32 ? combine_push_fp8_kernel<true> : combine_push_fp8_kernel<false>)<<<
      grid_for(tokens * 32, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(staged), tokens, top_k, hidden, topk_ids, expert_map,
      static_cast<const __nv_bfloat16*>(shared), world, rank, q, sc, f, epoch, counter, sparse);
  return check_cuda(cudaGetLastError(), "combine_push_fp8 launch");
}

int b2m_rs_reduce_fp8(const void* codes, const float* scales, int64_t rows, int64_t hidden, int32_t world,
                      const uint32_t* flags, uint32_t epoch, const void* add, void* out, const int32_t* topk_ids,
                      int32_t top_k, const int32_t* expert_owner, int32_t num_experts, int32_t* dev_status,
                      void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (world < 1 || world > kMaxWorld || rows <= 0 || hidden <= 0 || hidden % 128 || !codes || !scales || !out ||
      (reinterpret_cast<uintptr_t>(codes) & 7u) || !aligned16(out) || (add && !aligned16(add)))
    return fail(B2M_ERR_ARG, "rs_reduce_fp8: bad shape/pointers (hidden %% 128 == 0, 16-byte rows)");
  if (topk_ids) {
    if (top_k < 1 || top_k > 32 || !expert_owner || num_experts < 1)
      return fail(B2M_ERR_ARG, "rs_reduce_fp8: sparse reduce needs 1 <= top_k <= 32 and the owner table");
    rs_reduce_sparse_kernel<true><<<grid_for(rows * 32, num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        codes, scales, rows, hidden, world, topk_ids, top_k, expert_owner, num_experts, flags, epoch,
        static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out), dev_status, timeout_ns());
    return check_cuda(cudaGetLastError(), "rs_reduce_fp8 (sparse) launch");
  }
  rs_reduce_fp8_kernel<<<grid_for(rows * (hidden / 8), num_sms, 8), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(codes), scales, rows, hidden, world, flags, epoch,
      static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(out), dev_status, timeout_ns());
  return check_cuda(cudaGetLastError(), "rs_reduce_fp8 launch");
}

}  // extern "C"
