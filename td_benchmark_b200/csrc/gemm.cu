// K3 / K4: FP8 grouped GEMMs over ragged expert segments on tcgen05 + TMEM + TMA.
//
// Both GEMMs share one persistent, warp-specialised kernel (one CTA per SM):
//   warp 0      TMA producer.  B (weights) by 2D tiled TMA; A by TMA gather4 of the
//               routed token rows (gate/up GEMM) or by 2D tiled TMA of the sorted
//               intermediate (down GEMM).  4-stage smem ring, 48 KB per stage.
//   warp 1      TMEM allocator and single-thread MMA issuer: per 128-wide K block,
//               4 x tcgen05.mma kind::f8f6f4 (M=128, N=256, K=32) into one of two
//               TMEM accumulators (2 x 256 fp32 columns).
//   warps 4-11  promotion + epilogue.  The reference applies block scales per 128-K
//               step (moe_bench/overlap/kernels.py:179: acc += dot(a, b) * a_s * b_s);
//               so does this kernel: each K block's partial product is read from TMEM
//               (tcgen05.ld), multiplied by a_scale[row, kb] * b_scale[nblk, kb] and
//               added to fp32 registers.  The double-buffered TMEM lets the tensor
//               pipe run one K block ahead of the promotion.
// Tiles are (128 sorted rows) x (256 output columns).  The tile space is walked
// with a static stride of gridDim.x; blocks whose expert id is -1 are skipped.
//
// Gate/up epilogue (replaces silu_and_mul + the second quant, overlap_forward.py:554-561):
// the weight rows are interleaved at set-up so one tile holds gate columns
// [128j, 128j+128) and the matching up columns; warp half h owns gate/up columns
// [64h, 64h+64) of its row, computes h = silu(g) * u in fp32, exchanges the partial
// amax with the other half through shared memory and writes the 1x128 e4m3 codes
// and the scale (K-block-major scale layout for the down GEMM).
// Down epilogue (replaces MUL_ROUTED_WEIGHT + bf16 store, kernels.py:221-310): the
// row's routed weight times the accumulator, rounded to bf16, stored at the pair's
// row of the top-k staging buffer.
//
// All waits are bounded (b2m_set_timeout_ns); on a timeout the kernel records the
// site in dev_status, drains its own TMA copies and frees TMEM before returning.
#include <cudaTypedefs.h>

#include "b2m_common.cuh"
#include "b2m_host.h"

namespace b2m {
namespace {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;  // 16 KB
constexpr int B_BYTES = BN * BK;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 384;
constexpr int NUM_EPI_THREADS = 256;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_e4m3_f32(BM, BN);

struct Control {
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t amax_bar[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  float amax[2][2][BM];  // [tile parity][column half][row]
};

constexpr size_t SMEM_BYTES = size_t(STAGES) * STAGE_BYTES + sizeof(Control) + 1024;
static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");

struct GemmParams {
  const int32_t* sorted_ids;
  const int32_t* expert_ids;
  const int32_t* ntpp;
  int32_t max_blocks;  // rows_cap / BM
  int32_t numel;       // pad id
  int32_t top_k;
  int32_t num_kb;      // K / 128
  int32_t num_nt;      // output tiles along N
  int32_t n_blocks;    // 128-row scale blocks per expert of B
  int32_t n_rows;      // rows of B per expert
  int32_t a_rows;      // gate/up: token rows of A (row id a_rows reads zeros)
  const float* a_scale;
  int64_t a_scale_ld;  // gate/up: row stride of [a_rows, KB]; down: column count rows_cap of [KB, rows_cap]
  const float* b_scale;
  int64_t rows_cap;
  uint8_t* out_q;
  float* out_scale_t;
  int32_t inter;
  __nv_bfloat16* out_bf16;
  const float* topk_weights;
  int64_t hidden;
  int32_t* status;
  uint64_t timeout_ns;
};

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

template <bool kGateUp>
__device__ __forceinline__ void producer_warp(const CUtensorMap* map_a, const CUtensorMap* map_b,
                                              const GemmParams& p, uint8_t* smem, Control* C, int64_t num_tiles,
                                              int num_mb, int lane) {
  volatile int* abort = &C->abort;
  uint32_t kbg = 0;
  bool alive = true;
  for (int64_t tile = blockIdx.x; tile < num_tiles && alive; tile += gridDim.x) {
    const int mb = static_cast<int>(tile % num_mb);
    const int nt = static_cast<int>(tile / num_mb);
    const int e = __ldg(p.expert_ids + mb);
    if (e < 0) continue;
    int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
    if (kGateUp) {
      const int4 ids = __ldg(reinterpret_cast<const int4*>(p.sorted_ids + mb * BM) + lane);
      r0 = ids.x < p.numel ? ids.x / p.top_k : p.a_rows;
      r1 = ids.y < p.numel ? ids.y / p.top_k : p.a_rows;
      r2 = ids.z < p.numel ? ids.z / p.top_k : p.a_rows;
      r3 = ids.w < p.numel ? ids.w / p.top_k : p.a_rows;
    }
    const int b_row = e * p.n_rows + nt * BN;
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      const int s = kbg % STAGES;
      const uint32_t ph = (kbg / STAGES) & 1;
      int ok = 1;
      if (lane == 0) ok = mbar_wait(&C->empty[s], ph ^ 1, p.timeout_ns, p.status, B2M_STATUS_TIMEOUT_PRODUCER, abort);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        alive = false;
        break;
      }
      uint8_t* sa = smem + s * STAGE_BYTES;
      uint8_t* sb = sa + A_BYTES;
      if (lane == 0) mbar_arrive_expect_tx(&C->full[s], STAGE_BYTES);
      __syncwarp();
      if (kGateUp) {
        tma_gather4(sa + lane * 4 * BK, map_a, &C->full[s], kb * BK, r0, r1, r2, r3);
      } else if (lane == 0) {
        tma_load_2d(sa, map_a, &C->full[s], kb * BK, mb * BM);
      }
      if (lane == 0) tma_load_2d(sb, map_b, &C->full[s], kb * BK, b_row);
      __syncwarp();
    }
  }
  // Drain: every stage issued in the last STAGES iterations must have landed
  // before the CTA may exit (the normal path has consumed them all already).
  if (lane == 0) {
    const uint32_t first = kbg > STAGES ? kbg - STAGES : 0;
    for (uint32_t i = first; i < kbg; ++i)
      mbar_wait(&C->full[i % STAGES], (i / STAGES) & 1, p.timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN, nullptr);
  }
  __syncwarp();
}

__device__ __forceinline__ void mma_thread(const GemmParams& p, uint8_t* smem, Control* C, int64_t num_tiles,
                                           int num_mb, uint32_t tmem_base) {
  volatile int* abort = &C->abort;
  uint32_t kbg = 0;
  bool alive = true;
  for (int64_t tile = blockIdx.x; tile < num_tiles && alive; tile += gridDim.x) {
    const int mb = static_cast<int>(tile % num_mb);
    if (__ldg(p.expert_ids + mb) < 0) continue;
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      const int s = kbg % STAGES;
      const uint32_t ph = (kbg / STAGES) & 1;
      const int b = kbg & 1;
      const uint32_t tph = (kbg >> 1) & 1;
      if (!mbar_wait(&C->tempty[b], tph ^ 1, p.timeout_ns, p.status, B2M_STATUS_TIMEOUT_MMA, abort) ||
          !mbar_wait(&C->full[s], ph, p.timeout_ns, p.status, B2M_STATUS_TIMEOUT_MMA, abort)) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint64_t adesc = smem_desc_sw128(smem_u32(smem + s * STAGE_BYTES));
      const uint64_t bdesc = smem_desc_sw128(smem_u32(smem + s * STAGE_BYTES + A_BYTES));
      const uint32_t d = tmem_base + static_cast<uint32_t>(b * BN);
#pragma unroll
      for (int k = 0; k < BK / 32; ++k) mma_e4m3(d, adesc + 2 * k, bdesc + 2 * k, IDESC, k > 0 ? 1u : 0u);
      mma_commit(&C->empty[s]);
      mma_commit(&C->tfull[b]);
    }
  }
  // TMEM is freed after this CTA exits its roles: wait until every MMA issued here
  // has completed (on the normal path they all have; after an abort some may not).
  if (kbg > 0) {
    mma_commit(&C->mma_done);
    mbar_wait(&C->mma_done, 0, p.timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN, nullptr);
  }
}

template <bool kGateUp>
__device__ __forceinline__ void epilogue_warps(const GemmParams& p, Control* C, int64_t num_tiles, int num_mb,
                                               uint32_t tmem_base, int warp, int lane) {
  volatile int* abort = &C->abort;
  const int q = warp & 3;          // TMEM lane quarter this warp may access
  const int h = (warp - 4) >> 2;   // column half
  const int r = q * 32 + lane;     // tile row
  const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
  uint32_t kbg = 0;
  uint32_t tiles_done = 0;
  bool alive = true;
  for (int64_t tile = blockIdx.x; tile < num_tiles && alive; tile += gridDim.x) {
    const int mb = static_cast<int>(tile % num_mb);
    const int nt = static_cast<int>(tile / num_mb);
    const int e = __ldg(p.expert_ids + mb);
    if (e < 0) continue;
    const int64_t prow = static_cast<int64_t>(mb) * BM + r;
    const int pair = __ldg(p.sorted_ids + prow);
    const bool valid = pair < p.numel;

    // Per-K-block scale pointers.
    const float* as_ptr;
    int64_t as_step;
    const float* bs0;
    const float* bs1;
    bool bvalid = true;
    if (kGateUp) {
      as_ptr = valid ? p.a_scale + static_cast<int64_t>(pair / p.top_k) * p.a_scale_ld : nullptr;
      as_step = 1;
      bs0 = p.b_scale + (static_cast<int64_t>(e) * p.n_blocks + 2 * nt) * p.num_kb;  // gate block
      bs1 = bs0 + p.num_kb;                                                         // up block
    } else {
      as_ptr = p.a_scale + prow;
      as_step = p.a_scale_ld;
      const int blk = 2 * nt + h;
      bvalid = blk < p.n_blocks;
      bs0 = p.b_scale + (static_cast<int64_t>(e) * p.n_blocks + (bvalid ? blk : 0)) * p.num_kb;
      bs1 = bs0;
    }

    float acc[128];
#pragma unroll
    for (int i = 0; i < 128; ++i) acc[i] = 0.0f;

    float na = as_ptr ? __ldg(as_ptr) : 0.0f;
    float nb0 = __ldg(bs0), nb1 = __ldg(bs1);
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      const float sa = na, sb0 = nb0, sb1 = nb1;
      if (kb + 1 < p.num_kb) {  // prefetch next K block's scales
        na = as_ptr ? __ldg(as_ptr + (kb + 1) * as_step) : 0.0f;
        nb0 = __ldg(bs0 + kb + 1);
        nb1 = __ldg(bs1 + kb + 1);
      }
      const int b = kbg & 1;
      const uint32_t tph = (kbg >> 1) & 1;
      int ok = mbar_wait(&C->tfull[b], tph, p.timeout_ns, p.status, B2M_STATUS_TIMEOUT_EPILOGUE, abort);
      if (!__all_sync(0xffffffffu, ok)) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint32_t base = tmem_base + lane_off + static_cast<uint32_t>(b * BN);
      // Column chunks owned by this thread (32 fp32 columns each).
      uint32_t c0, c1, c2, c3;
      if (kGateUp) {
        c0 = 64 * h;
        c1 = 64 * h + 32;
        c2 = 128 + 64 * h;
        c3 = 128 + 64 * h + 32;
      } else {
        c0 = 128 * h;
        c1 = c0 + 32;
        c2 = c0 + 64;
        c3 = c0 + 96;
      }
      const float s_lo = sa * sb0;
      const float s_hi = sa * sb1;
      {
        float v0[32], v1[32];
        tmem_ld32(base + c0, v0);
        tmem_ld32(base + c1, v1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = fmaf(v0[i], s_lo, acc[i]);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[32 + i] = fmaf(v1[i], s_lo, acc[32 + i]);
      }
      {
        float v2[32], v3[32];
        tmem_ld32(base + c2, v2);
        tmem_ld32(base + c3, v3);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&C->tempty[b]);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[64 + i] = fmaf(v2[i], s_hi, acc[64 + i]);
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[96 + i] = fmaf(v3[i], s_hi, acc[96 + i]);
      }
    }
    if (!alive) break;

    if (kGateUp) {
      // h = silu(gate) * up, then 1x128 quant across both column halves of the row.
      float amax = 0.0f;
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float v = silu(acc[i]) * acc[64 + i];
        acc[i] = v;
        amax = fmaxf(amax, fabsf(v));
      }
      const int par = tiles_done & 1;
      C->amax[par][h][r] = amax;
      mbar_arrive(&C->amax_bar[par]);
      int ok = mbar_wait(&C->amax_bar[par], (tiles_done >> 1) & 1, p.timeout_ns, p.status,
                         B2M_STATUS_TIMEOUT_EPILOGUE, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      amax = fmaxf(C->amax[par][0][r], C->amax[par][1][r]);
      const float scale = fmaxf(amax / 448.0f, 1e-12f);
      uint8_t* dst = p.out_q + prow * p.inter + nt * 128 + 64 * h;
#pragma unroll
      for (int i = 0; i < 64; i += 16) {
        uint4 w;
        w.x = pack4_e4m3(clamp448(acc[i + 0] / scale), clamp448(acc[i + 1] / scale), clamp448(acc[i + 2] / scale),
                         clamp448(acc[i + 3] / scale));
        w.y = pack4_e4m3(clamp448(acc[i + 4] / scale), clamp448(acc[i + 5] / scale), clamp448(acc[i + 6] / scale),
                         clamp448(acc[i + 7] / scale));
        w.z = pack4_e4m3(clamp448(acc[i + 8] / scale), clamp448(acc[i + 9] / scale),
                         clamp448(acc[i + 10] / scale), clamp448(acc[i + 11] / scale));
        w.w = pack4_e4m3(clamp448(acc[i + 12] / scale), clamp448(acc[i + 13] / scale),
                         clamp448(acc[i + 14] / scale), clamp448(acc[i + 15] / scale));
        *reinterpret_cast<uint4*>(dst + i) = w;
      }
      if (h == 0) p.out_scale_t[static_cast<int64_t>(nt) * p.rows_cap + prow] = scale;
    } else {
      if (valid && bvalid) {
        const float w = p.topk_weights ? __ldg(p.topk_weights + pair) : 1.0f;
        __nv_bfloat16* dst = p.out_bf16 + static_cast<int64_t>(pair) * p.hidden + nt * BN + 128 * h;
#pragma unroll
        for (int i = 0; i < 128; i += 8) {
          uint32_t u[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162 v = __floats2bfloat162_rn(acc[i + 2 * j] * w, acc[i + 2 * j + 1] * w);
            u[j] = *reinterpret_cast<const uint32_t*>(&v);
          }
          *reinterpret_cast<uint4*>(dst + i) = make_uint4(u[0], u[1], u[2], u[3]);
        }
      }
    }
    ++tiles_done;
  }
}

template <bool kGateUp>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Control* C = reinterpret_cast<Control*>(smem + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int32_t ntpp = __ldg(p.ntpp);
  int num_mb = ntpp / BM;
  if (ntpp < 0 || ntpp % BM != 0 || num_mb > p.max_blocks) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_status(p.status, B2M_STATUS_BAD_ROUTING);
    num_mb = 0;
  }
  const int64_t num_tiles = static_cast<int64_t>(num_mb) * p.num_nt;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&C->full[s], 1);
      mbar_init(&C->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&C->tfull[b], 1);
      mbar_init(&C->tempty[b], NUM_EPI_THREADS / 32);
      mbar_init(&C->amax_bar[b], NUM_EPI_THREADS);
    }
    mbar_init(&C->mma_done, 1);
    C->abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) tmem_alloc(&C->tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = C->tmem_base;

  if (warp < 4) {
    reg_dealloc<56>();
    if (warp == 0) {
      producer_warp<kGateUp>(&map_a, &map_b, p, smem, C, num_tiles, num_mb, lane);
    } else if (warp == 1) {
      if (lane == 0) mma_thread(p, smem, C, num_tiles, num_mb, tmem_base);
      __syncwarp();
    }
  } else {
    reg_alloc<224>();
    epilogue_warps<kGateUp>(p, C, num_tiles, num_mb, tmem_base, warp, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
int encode_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                  uint32_t box_inner, uint32_t box_outer) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    B2M_TRY(check_cuda(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
                       "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)"));
    if (q != cudaDriverEntryPointSuccess || !fn)
      return fail(B2M_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled not available from the driver");
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t elem_strides[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(B2M_ERR_ARG, "cuTensorMapEncodeTiled failed (%d) for a [%llu x %llu] operand, box %u x %u", (int)r,
                (unsigned long long)outer, (unsigned long long)inner, box_outer, box_inner);
  return B2M_OK;
}

template <bool kGateUp>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p, int num_sms, cudaStream_t s) {
  static int attr_done[64] = {0};
  int dev = 0;
  B2M_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    B2M_TRY(check_cuda(cudaFuncSetAttribute(moe_gemm_kernel<kGateUp>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(SMEM_BYTES)),
                       "gemm: cudaFuncSetAttribute"));
    attr_done[dev] = 1;
  }
  int64_t upper = static_cast<int64_t>(p.max_blocks) * p.num_nt;
  int grid = static_cast<int>(upper < num_sms ? upper : num_sms);
  if (grid < 1) grid = 1;
  moe_gemm_kernel<kGateUp><<<grid, NUM_THREADS, SMEM_BYTES, s>>>(ma, mb, p);
  return check_cuda(cudaGetLastError(), kGateUp ? "gemm1 launch" : "gemm2 launch");
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_gemm1(const void* a_fp8, const float* a_scale, int64_t a_rows, int64_t hidden, const void* w1,
                         const float* w1_scale, int32_t num_experts, int32_t inter, const int32_t* sorted_token_ids,
                         const int32_t* expert_ids, const int32_t* num_tokens_post_padded, int64_t rows_cap,
                         int64_t numel, int32_t top_k, void* out_q, float* out_scale_t, int32_t* dev_status,
                         void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128 || num_experts <= 0 || top_k <= 0 || a_rows < 0 ||
      rows_cap <= 0 || rows_cap % BM || numel < 0)
    return fail(B2M_ERR_ARG,
                "gemm1: need hidden%%128==0 (%lld), inter%%128==0 (%d), rows_cap%%128==0 (%lld), E>0, top_k>0",
                (long long)hidden, inter, (long long)rows_cap);
  if (!a_fp8 || !a_scale || !w1 || !w1_scale || !sorted_token_ids || !expert_ids || !num_tokens_post_padded ||
      !out_q || !out_scale_t)
    return fail(B2M_ERR_ARG, "gemm1: null pointer");
  if (!aligned16(a_fp8) || !aligned16(w1) || !aligned16(out_q) || !aligned16(sorted_token_ids))
    return fail(B2M_ERR_ARG, "gemm1: A, W1, out_q and sorted_token_ids must be 16-byte aligned");
  if (rows_cap / BM > INT32_MAX || a_rows >= INT32_MAX || numel >= INT32_MAX)
    return fail(B2M_ERR_ARG, "gemm1: sizes overflow int32 indices");
  CUtensorMap ma, mb;
  // A rows are gathered 4 at a time; the map spans a_rows rows (at least one so it is valid).
  B2M_TRY(encode_map_2d(&ma, a_fp8, hidden, a_rows > 0 ? a_rows : 1, hidden, BK, 1));
  B2M_TRY(encode_map_2d(&mb, w1, hidden, static_cast<uint64_t>(num_experts) * 2 * inter, hidden, BK, BN));
  GemmParams p{};
  p.sorted_ids = sorted_token_ids;
  p.expert_ids = expert_ids;
  p.ntpp = num_tokens_post_padded;
  p.max_blocks = static_cast<int32_t>(rows_cap / BM);
  p.numel = static_cast<int32_t>(numel);
  p.top_k = top_k;
  p.num_kb = static_cast<int32_t>(hidden / BK);
  p.num_nt = inter / 128;
  p.n_blocks = 2 * inter / 128;
  p.n_rows = 2 * inter;
  p.a_rows = static_cast<int32_t>(a_rows);
  p.a_scale = a_scale;
  p.a_scale_ld = hidden / 128;
  p.b_scale = w1_scale;
  p.rows_cap = rows_cap;
  p.out_q = static_cast<uint8_t*>(out_q);
  p.out_scale_t = out_scale_t;
  p.inter = inter;
  p.status = dev_status;
  p.timeout_ns = timeout_ns();
  return launch_gemm<true>(ma, mb, p, num_sms, static_cast<cudaStream_t>(stream));
}

extern "C" int b2m_gemm2(const void* a_fp8, const float* a_scale_t, int64_t rows_cap, int32_t inter, const void* w2,
                         const float* w2_scale, int32_t num_experts, int64_t hidden, const int32_t* sorted_token_ids,
                         const int32_t* expert_ids, const int32_t* num_tokens_post_padded, int64_t numel,
                         const float* topk_weights, void* out_bf16, int32_t* dev_status, void* stream) {
  using namespace b2m;
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128 || num_experts <= 0 || rows_cap <= 0 ||
      rows_cap % BM || numel < 0)
    return fail(B2M_ERR_ARG, "gemm2: need hidden%%128==0 (%lld), inter%%128==0 (%d), rows_cap%%128==0 (%lld)",
                (long long)hidden, inter, (long long)rows_cap);
  if (!a_fp8 || !a_scale_t || !w2 || !w2_scale || !sorted_token_ids || !expert_ids || !num_tokens_post_padded ||
      !out_bf16)
    return fail(B2M_ERR_ARG, "gemm2: null pointer");
  if (!aligned16(a_fp8) || !aligned16(w2) || !aligned16(out_bf16))
    return fail(B2M_ERR_ARG, "gemm2: A, W2 and out must be 16-byte aligned");
  if (rows_cap / BM > INT32_MAX || numel >= INT32_MAX) return fail(B2M_ERR_ARG, "gemm2: sizes overflow int32");
  CUtensorMap ma, mb;
  B2M_TRY(encode_map_2d(&ma, a_fp8, inter, rows_cap, inter, BK, BM));
  B2M_TRY(encode_map_2d(&mb, w2, inter, static_cast<uint64_t>(num_experts) * hidden, inter, BK, BN));
  GemmParams p{};
  p.sorted_ids = sorted_token_ids;
  p.expert_ids = expert_ids;
  p.ntpp = num_tokens_post_padded;
  p.max_blocks = static_cast<int32_t>(rows_cap / BM);
  p.numel = static_cast<int32_t>(numel);
  p.top_k = 1;
  p.num_kb = inter / BK;
  p.num_nt = static_cast<int32_t>((hidden + BN - 1) / BN);
  p.n_blocks = static_cast<int32_t>(hidden / 128);
  p.n_rows = static_cast<int32_t>(hidden);
  p.a_rows = 0;
  p.a_scale = a_scale_t;
  p.a_scale_ld = rows_cap;
  p.b_scale = w2_scale;
  p.rows_cap = rows_cap;
  p.out_bf16 = static_cast<__nv_bfloat16*>(out_bf16);
  p.topk_weights = topk_weights;
  p.hidden = hidden;
  p.status = dev_status;
  p.timeout_ns = timeout_ns();
  return launch_gemm<false>(ma, mb, p, num_sms, static_cast<cudaStream_t>(stream));
}
