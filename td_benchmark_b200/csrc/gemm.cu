// K3 / K4: FP8 grouped GEMMs over ragged expert segments on tcgen05 + TMEM + TMA.
//
// Both GEMMs share one persistent, warp-specialised kernel (one CTA per SM,
// 384 threads, 4-stage shared-memory ring of 48 KB operand stages):
//   warp 0      stage producer: A (2D tiled TMA of the expert-sorted rows: the token
//               rows dispatched by b2m_quant_dispatch / b2m_dispatch_rows for the gate/up
//               GEMM, the gate/up output for the down GEMM), its 128 row scales (one
//               512-byte bulk copy of the K-block-major scale array), B (weights) by 2D
//               tiled TMA, and the B block scales of the stage (prefetched 32 K blocks at
//               a time across the warp's lanes).  The scales go to an 8-deep ring with
//               its own barriers, so an operand stage is recycled as soon as the MMA that
//               read it completes.
//   warp 1      TMEM allocator and single-thread MMA issuer: per 128-wide K block,
//               4 x tcgen05.mma kind::f8f6f4 (M=128, N=256, K=32) into one of two
//               TMEM accumulators (2 x 256 fp32 columns).
//   warps 4-11  promotion + epilogue.  The reference applies block scales per 128-K
//               step (moe_bench/overlap/kernels.py:179: acc += dot(a, b) * a_s * b_s);
//               so does this kernel: each K block's partial product is read from TMEM
//               (tcgen05.ld), multiplied by a_scale[row, kb] * b_scale[nblk, kb] (read
//               from the stage in shared memory) and added to fp32 registers with packed
//               f32x2 FMAs.  The double-buffered TMEM lets the tensor pipe run one K
//               block ahead.
// Tiles are (128 sorted rows) x (256 output columns), visited in bands of 16 M blocks
// (N tile by N tile inside a band) so CTAs running together share weight tiles and
// A rows in L2.  The tile space is walked with
// a static stride of gridDim.x; blocks whose expert id is -1 are skipped.
//
// Gate/up epilogue (replaces silu_and_mul + the second quant, overlap_forward.py:554-561):
// the weight rows are interleaved at set-up so one tile holds gate columns
// [128j, 128j+128) and the matching up columns; warp half h owns gate/up columns
// [64h, 64h+64) of its row, computes h = silu(g) * u in fp32, exchanges the partial
// amax with the other half through shared memory and writes the 1x128 e4m3 codes
// and the scale (K-block-major scale layout for the down GEMM).
// Down epilogue (replaces MUL_ROUTED_WEIGHT + bf16 store, kernels.py:221-310): the
// row's routed weight times the accumulator, rounded to bf16, stored at the pair's
// row of the top-k staging buffer, or (b2m_gemm2_scatter) straight into the row's
// owner rank's receive buffer.
//
// Gate/up GEMM fed by peers (b2m_gemm1_wait, tensor parallel): the M blocks are visited
// in a given order (own rows first), the producer waits per block for the flags of the
// source ranks the block holds, and warps 2-3 -- otherwise idle -- can push this rank's
// rows to the same rows of every peer while the MMA pipeline runs.
//
// All waits are bounded (b2m_set_timeout_ns); on a timeout the kernel records the
// site in dev_status, drains its own copies and MMAs and frees TMEM before returning.
// Waits on another rank's flag use the set bound, waits on the CTA's own pipeline twice
// that, so a pipeline stalled behind a missing peer records TIMEOUT_PEER (the cause).
#include <cudaTypedefs.h>

#include <atomic>

#include "b2m_common.cuh"
#include "b2m_host.h"

namespace b2m {
namespace {

constexpr int BM = 128, BN = 256, BK = 128;
constexpr int STAGES = 4;          // operand stages of the grouped GEMMs
constexpr int SCATTER_STAGES = 3;  // the down GEMM storing into owners: 3 stages + the row staging tile
constexpr int SRING = 8;     // scale ring depth (decoupled from the operand stages)
constexpr int GROUP_M = 16;  // tile raster: bands of GROUP_M M-blocks x all N tiles
constexpr int A_BYTES = BM * BK;  // 16 KB
constexpr int B_BYTES = BN * BK;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 384;
constexpr int NUM_EPI_WARPS = 8;
constexpr int NUM_EPI_THREADS = NUM_EPI_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t IDESC = idesc_e4m3_f32(BM, BN);

template <int S>
struct ControlT {
  uint64_t full[S];
  uint64_t empty[S];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t amax_bar[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;
  uint64_t sfull[SRING];
  uint64_t sempty[SRING];
  alignas(16) float as[SRING][BM];  // A row scales of K block kbg (slot kbg % SRING)
  alignas(16) float bs[SRING][4];   // B block scales of that K block: tile rows [0,128) and [128,256)
  float amax[2][2][BM];              // [tile parity][column half][row]
  uint64_t stg_free[2];              // row staging: every epilogue thread may overwrite it ([tile parity])
  uint64_t stg_full[2];              // row staging: every epilogue thread has written its row piece
};

// Row staging of the scattering down GEMM: the tile's 128 bf16 output rows (256 columns)
// with 16 bytes of padding per row so that the epilogue's 16-byte stores (32 lanes on 32
// consecutive rows) spread over all banks.
constexpr int STG_ROW_BYTES = BN * 2 + 16;
constexpr int STG_BYTES = BM * STG_ROW_BYTES;

template <int S>
constexpr size_t smem_bytes() {
  return size_t(S) * STAGE_BYTES + sizeof(ControlT<S>) + (S == SCATTER_STAGES ? STG_BYTES + 128 : 0) + 1024;
}
static_assert(smem_bytes<STAGES>() <= 227 * 1024, "shared memory budget");
static_assert(smem_bytes<SCATTER_STAGES>() <= 227 * 1024, "shared memory budget (scattering down GEMM)");

struct GemmParams {
  const int32_t* sorted_ids;
  const int32_t* expert_ids;
  const int32_t* ntpp;
  int32_t max_blocks;  // rows_cap / BM
  int32_t numel;       // pad id
  int32_t top_k;
  int32_t num_kb;      // K / 128
  int32_t num_nt;      // output tiles along N in this launch (window [nt_begin, nt_begin + num_nt))
  int32_t nt_begin;    // first N tile of the window
  int32_t n_blocks;    // 128-row scale blocks per expert of B
  int32_t n_rows;      // rows of B per expert
  const float* a_scale;  // [KB, rows_cap]: scale of sorted row p, K block kb at kb * rows_cap + p
  int64_t a_scale_ld;    // rows_cap
  const float* b_scale;
  int64_t rows_cap;
  uint8_t* out_q;
  float* out_scale_t;
  int32_t inter;
  __nv_bfloat16* out_bf16;
  const float* topk_weights;
  int64_t hidden;
  int32_t* status;
  uint64_t timeout_ns;       // bound of a wait on another rank's flag
  uint64_t pipe_timeout_ns;  // bound of a wait on this CTA's own pipeline (2 x timeout_ns): a
                             // stalled pipeline behind a missing peer reports the peer, not itself
  // Down GEMM scatter (rs_world > 0): the row of pair p goes to owner q = p / rs_pairs_per_owner,
  // row rs_row0 + p - q * rs_pairs_per_owner of rs_dst[q] (another rank's receive buffer),
  // instead of row p of out_bf16.
  __nv_bfloat16* rs_dst[8];
  int64_t rs_pairs_per_owner;
  int64_t rs_row0;
  int32_t rs_world;
  // Gate/up GEMM whose A rows are stored by the source ranks (b2m_quant_dispatch_push):
  // before loading a block, the producer waits until src_flags[s] >= src_epoch for every
  // source s among the block's rows (token of pair p = p / top_k, source = token /
  // tokens_per_src).  src_flags == nullptr: no waits.  block_order: M-block visiting order.
  const uint32_t* src_flags;
  uint32_t src_epoch;
  int64_t tokens_per_src;
  const int32_t* block_order;
  // All-gather pushed from inside the gate/up GEMM (push_world > 1): warps 2-3 of every CTA
  // copy this rank's pair rows -- already quantised into the own sorted operand (A) and its
  // K-block-major scales -- to the same rows of every peer, destination by destination
  // (rank-1, rank-2, ...), and publish push_flag[d] = src_epoch when the grid is done with d.
  const int32_t* push_pos;  // sorted position of each of this rank's pairs, -1: none
  int64_t push_pairs;
  const uint8_t* push_src_a;
  const float* push_src_s;
  uint8_t* push_a[8];
  float* push_s[8];
  uint32_t* push_flag[8];
  int32_t* push_counters;   // [push_world], zero between calls
  int32_t push_world;
  int32_t push_rank;
};

// silu(x) = x * sigmoid(x).  The gate/up intermediate is requantised to e4m3 right
// after, so the fast exponential and reciprocal are far inside its tolerance.
__device__ __forceinline__ float silu(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// Shared tile walk of every role: returns false when the tile is skipped (expert -1).
struct TileWalk {
  int64_t num_tiles;
  int num_mb;
  int num_nt;
  int nt_begin;
  const int32_t* order;  // M-block visiting order (nullptr: 0, 1, 2, ...)
};

// Tile t -> (M block, N tile): bands of GROUP_M consecutive M blocks (experts are
// contiguous in M) walked N-tile by N-tile, so the CTAs running together share a few
// weight tiles and a band of A rows, both L2-resident.
__device__ __forceinline__ void tile_coords(int64_t t, const TileWalk& tw, int& mb, int& nt) {
  const int64_t per_band = static_cast<int64_t>(GROUP_M) * tw.num_nt;
  const int64_t band = t / per_band;
  const int first = static_cast<int>(band * GROUP_M);
  const int rows = tw.num_mb - first < GROUP_M ? tw.num_mb - first : GROUP_M;
  const int64_t in_band = t - band * per_band;
  mb = first + static_cast<int>(in_band % rows);
  nt = tw.nt_begin + static_cast<int>(in_band / rows);
  if (tw.order) mb = __ldg(tw.order + mb);
}

// Producer warp, before the loads of block mb: the lowest and highest source rank among the
// block's rows (pairs ascend inside an expert segment, so the rows of one source are
// contiguous), then lane 0 waits (bounded) for each of those sources' flags not seen yet and
// orders the copies that follow after the peers' stores (acquire, then a proxy fence: the
// operand and scale copies are async-proxy reads of memory the peers wrote with ordinary
// stores).  Returns false after a timeout (status recorded, the CTA aborts).
__device__ __forceinline__ bool wait_block_sources(const GemmParams& p, int mb, uint32_t& ready, int lane,
                                                   volatile int* abort) {
  int lo = 1 << 30, hi = -1;
#pragma unroll
  for (int i = 0; i < BM / 32; ++i) {
    const int32_t id = __ldg(p.sorted_ids + static_cast<int64_t>(mb) * BM + i * 32 + lane);
    if (id >= 0 && id < p.numel) {
      const int src = static_cast<int>((id / p.top_k) / p.tokens_per_src);
      lo = min(lo, src);
      hi = max(hi, src);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, off));
    hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
  }
  int ok = 1;
  if (lane == 0) {
    for (int src = lo; src <= hi && ok; ++src) {
      if (src < 0 || src >= 32 || (ready >> src) & 1u) continue;  // the host bounds sources to 8
      if (!wait_flag_geq(p.src_flags + src, p.src_epoch, p.timeout_ns, p.status, B2M_STATUS_TIMEOUT_PEER)) {
        ok = 0;
        *abort = 1;
      } else {
        ready |= 1u << src;
      }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
  }
  ready = __shfl_sync(0xffffffffu, ready, 0);
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// ---------------------------------------------------------------- warps 2-3: all-gather pusher
// Pusher warp g of G = 2 * gridDim.x copies pair rows g, g + G, ...: the row (hidden e4m3
// codes, 16 bytes per lane per step, 4 steps in flight) and its hidden/128 scales, from the
// own sorted operand to the same row of each peer.  The warp counts itself on the peer's
// counter after its last row for that peer; the last warp publishes the peer's flag.
__device__ __forceinline__ void push_rows(const GemmParams& p, int lane) {
  const int64_t g = static_cast<int64_t>(blockIdx.x) * 2 + ((threadIdx.x >> 5) - 2);
  const int64_t G = static_cast<int64_t>(gridDim.x) * 2;
  const int64_t cols = p.hidden;
  const int kbn = static_cast<int>(cols / 128);
  for (int i = 1; i < p.push_world; ++i) {
    const int d = (p.push_rank - i + p.push_world) % p.push_world;
    uint8_t* dst_a = p.push_a[d];
    float* dst_s = p.push_s[d];
    for (int64_t pr = g; pr < p.push_pairs; pr += G) {
      const int64_t pos = __ldg(p.push_pos + pr);
      if (pos < 0) continue;
      const uint8_t* src = p.push_src_a + pos * cols;
      uint8_t* dst = dst_a + pos * cols;
      // 4 x 16 bytes in flight per lane: this role runs after setmaxnreg.dec to 72 registers
      for (int64_t c0 = static_cast<int64_t>(lane) * 16; c0 < cols; c0 += 32 * 16 * 4) {
        uint4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t c = c0 + u * 512;
          if (c < cols) v[u] = __ldg(reinterpret_cast<const uint4*>(src + c));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int64_t c = c0 + u * 512;
          if (c < cols) *reinterpret_cast<uint4*>(dst + c) = v[u];
        }
      }
      for (int kb = lane; kb < kbn; kb += 32) dst_s[kb * p.rows_cap + pos] = __ldg(p.push_src_s + kb * p.rows_cap + pos);
    }
    __threadfence_system();
    __syncwarp();
    if (lane == 0) {
      const int prev = atomicAdd(p.push_counters + d, 1);
      if (prev == static_cast<int>(G) - 1) {
        fence_sys();
        st_release_sys(p.push_flag[d], p.src_epoch);
        atomicExch(p.push_counters + d, 0);
      }
    }
  }
}

// ---------------------------------------------------------------- warp 0: B (+A for the down GEMM)
template <bool kGateUp, int S>
__device__ __forceinline__ void stage_producer(const CUtensorMap* map_a, const CUtensorMap* map_b,
                                               const GemmParams& p, uint8_t* smem, ControlT<S>* C, TileWalk tw,
                                               int lane) {
  volatile int* abort = &C->abort;
  uint32_t kbg = 0;
  bool alive = true;
  uint32_t ready = 0;  // sources whose rows have arrived (gate/up GEMM fed by peers)
  const uint32_t tx = A_BYTES + B_BYTES;
  for (int64_t tile = blockIdx.x; tile < tw.num_tiles && alive; tile += gridDim.x) {
    int mb, nt;
    tile_coords(tile, tw, mb, nt);
    const int e = __ldg(p.expert_ids + mb);
    if (e < 0) continue;
    const int blk0 = 2 * nt;
    const int blk1 = 2 * nt + 1 < p.n_blocks ? 2 * nt + 1 : 2 * nt;  // the down GEMM's last tile may be half wide
    const float* bs0 = p.b_scale + (static_cast<int64_t>(e) * p.n_blocks + blk0) * p.num_kb;
    const float* bs1 = p.b_scale + (static_cast<int64_t>(e) * p.n_blocks + blk1) * p.num_kb;
    const int b_row = e * p.n_rows + nt * BN;
    if (p.src_flags && !wait_block_sources(p, mb, ready, lane, abort)) {
      alive = false;
      break;
    }
    float pre0 = 0.0f, pre1 = 0.0f;
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      if ((kb & 31) == 0) {  // lane j holds the scales of K block kb + j
        const int k = kb + lane;
        pre0 = k < p.num_kb ? __ldg(bs0 + k) : 0.0f;
        pre1 = k < p.num_kb ? __ldg(bs1 + k) : 0.0f;
      }
      const float s0 = __shfl_sync(0xffffffffu, pre0, kb & 31);
      const float s1 = __shfl_sync(0xffffffffu, pre1, kb & 31);
      const int s = kbg % S;
      const uint32_t ph = (kbg / S) & 1;
      const int r = kbg % SRING;
      const uint32_t rph = (kbg / SRING) & 1;
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait(&C->sempty[r], rph ^ 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_PRODUCER, abort) &&
             mbar_wait(&C->empty[s], ph ^ 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_PRODUCER, abort);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        alive = false;
        break;
      }
      if (lane == 0) {
        uint8_t* sa = smem + s * STAGE_BYTES;
        C->bs[r][0] = s0;
        C->bs[r][1] = s1;
        mbar_arrive_expect_tx(&C->sfull[r], BM * 4);  // releases the bs stores, counts the bulk copy
        bulk_load(C->as[r], p.a_scale + static_cast<int64_t>(kb) * p.a_scale_ld + static_cast<int64_t>(mb) * BM,
                  BM * 4, &C->sfull[r]);
        mbar_arrive_expect_tx(&C->full[s], tx);
        tma_load_2d(sa, map_a, &C->full[s], kb * BK, mb * BM);
        tma_load_2d(sa + A_BYTES, map_b, &C->full[s], kb * BK, b_row);
      }
      __syncwarp();
    }
  }
  // Drain: the copies of the last S stages (and SRING scale slots) must have
  // landed before the CTA exits.
  if (lane == 0) {
    const uint32_t first = kbg > S ? kbg - S : 0;
    for (uint32_t i = first; i < kbg; ++i)
      mbar_wait(&C->full[i % S], (i / S) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN, nullptr);
    const uint32_t rfirst = kbg > SRING ? kbg - SRING : 0;
    for (uint32_t i = rfirst; i < kbg; ++i)
      mbar_wait(&C->sfull[i % SRING], (i / SRING) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN, nullptr);
  }
  __syncwarp();
}

// ---------------------------------------------------------------- warp 1 lane 0: MMA issue
template <int S>
__device__ __forceinline__ void mma_thread(const GemmParams& p, uint8_t* smem, ControlT<S>* C, TileWalk tw,
                                           uint32_t tmem_base) {
  volatile int* abort = &C->abort;
  uint32_t kbg = 0;
  bool alive = true;
  for (int64_t tile = blockIdx.x; tile < tw.num_tiles && alive; tile += gridDim.x) {
    int mb, nt;
    tile_coords(tile, tw, mb, nt);
    if (__ldg(p.expert_ids + mb) < 0) continue;
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      const int s = kbg % S;
      const uint32_t ph = (kbg / S) & 1;
      const int b = kbg & 1;
      const uint32_t tph = (kbg >> 1) & 1;
      if (!mbar_wait(&C->tempty[b], tph ^ 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_MMA, abort) ||
          !mbar_wait(&C->full[s], ph, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_MMA, abort)) {
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
  // TMEM is freed after the roles finish: wait until every MMA issued here has
  // completed (on the normal path they all have; after an abort some may not).
  if (kbg > 0) {
    mma_commit(&C->mma_done);
    mbar_wait(&C->mma_done, 0, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN, nullptr);
  }
}

// End of a tile for one epilogue thread (row r of the tile, column half h), acc holding
// its 128 promoted fp32 columns.  Gate/up: h = silu(gate) * up, 1x128 requant across the
// row's two column halves (partial amax exchanged through shared memory), codes + scale
// stored at sorted row prow.  Down: routed weight, bf16, stored at the pair's row.
// Returns false when the amax exchange timed out.
template <bool kGateUp>
__device__ __forceinline__ bool finish_tile(const GemmParams& p, float (*amax_x)[2][BM], uint64_t* amax_bar,
                                           float (&acc)[128], int64_t prow, int nt, int h, int r, int pair,
                                           float wrow, bool valid, uint32_t tiles_done, int lane,
                                           volatile int* abort, uint8_t* staging = nullptr,
                                           uint64_t* stg_free = nullptr, uint64_t* stg_full = nullptr) {
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
    amax_x[par][h][r] = amax;
    mbar_arrive(&amax_bar[par]);
    int ok = mbar_wait(&amax_bar[par], (tiles_done >> 1) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_EPILOGUE,
                       abort);
    if (!__all_sync(0xffffffffu, ok)) return false;
    amax = fmaxf(amax_x[par][0][r], amax_x[par][1][r]);
    const float scale = fmaxf(amax / 448.0f, 1e-12f);
    const float inv = 1.0f / scale;  // one IEEE division per row; codes use x * (1/scale)
    uint8_t* dst = p.out_q + prow * p.inter + nt * 128 + 64 * h;
#pragma unroll
    for (int i = 0; i < 64; i += 16) {
      uint4 w;
      w.x = pack4_e4m3(clamp448(acc[i + 0] * inv), clamp448(acc[i + 1] * inv), clamp448(acc[i + 2] * inv),
                       clamp448(acc[i + 3] * inv));
      w.y = pack4_e4m3(clamp448(acc[i + 4] * inv), clamp448(acc[i + 5] * inv), clamp448(acc[i + 6] * inv),
                       clamp448(acc[i + 7] * inv));
      w.z = pack4_e4m3(clamp448(acc[i + 8] * inv), clamp448(acc[i + 9] * inv), clamp448(acc[i + 10] * inv),
                       clamp448(acc[i + 11] * inv));
      w.w = pack4_e4m3(clamp448(acc[i + 12] * inv), clamp448(acc[i + 13] * inv), clamp448(acc[i + 14] * inv),
                       clamp448(acc[i + 15] * inv));
      *reinterpret_cast<uint4*>(dst + i) = w;
    }
    if (h == 0) p.out_scale_t[static_cast<int64_t>(nt) * p.rows_cap + prow] = scale;
  } else if (staging) {
    // Scattering down GEMM: whole rows leave through shared memory.  Each thread writes its
    // 128 columns of row r into the staging tile; then lanes 0-15 of every epilogue warp
    // each send one of the tile's rows (512 bytes: both column halves) to its owner with a
    // bulk store -- NVLink carries whole row pieces, and the stores drain while the next
    // tile's MMAs run.  The staging tile is reused only after this thread's previous bulk
    // stores have read it and every thread has passed that point (bounded mbarrier waits,
    // so a warp that aborted cannot leave the others waiting).
    const int par = tiles_done & 1;
    const bool issuer = lane < 16;
    if (issuer) bulk_wait_read_all();
    mbar_arrive(&stg_free[par]);
    int ok = mbar_wait(&stg_free[par], (tiles_done >> 1) & 1, p.pipe_timeout_ns, p.status,
                       B2M_STATUS_TIMEOUT_EPILOGUE, abort);
    if (!__all_sync(0xffffffffu, ok)) return false;
    if (2 * nt + h < p.n_blocks) {
      uint8_t* srow = staging + r * STG_ROW_BYTES + h * 256;
#pragma unroll
      for (int i = 0; i < 128; i += 8) {
        uint32_t u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __nv_bfloat162 v = __floats2bfloat162_rn(acc[i + 2 * j] * wrow, acc[i + 2 * j + 1] * wrow);
          u[j] = *reinterpret_cast<const uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(srow + i * 2) = make_uint4(u[0], u[1], u[2], u[3]);
      }
    }
    fence_proxy_async_smem();  // the bulk stores read these rows through the async proxy
    mbar_arrive(&stg_full[par]);
    ok = mbar_wait(&stg_full[par], (tiles_done >> 1) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_EPILOGUE,
                   abort);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const int src_lane = h * 16 + (lane & 15);  // the lane of this warp that holds the row this lane sends
    const int rpair = __shfl_sync(0xffffffffu, pair, src_lane);
    if (issuer && rpair < p.numel) {
      const int rr = (r - lane) + src_lane;
      const int qo = static_cast<int>(rpair / p.rs_pairs_per_owner);
      __nv_bfloat16* dst =
          p.rs_dst[qo] + (p.rs_row0 + rpair - qo * p.rs_pairs_per_owner) * p.hidden + static_cast<int64_t>(nt) * BN;
      bulk_store(dst, staging + rr * STG_ROW_BYTES, 2 * nt + 1 < p.n_blocks ? 512u : 256u);
      bulk_commit();
    }
  } else {
    const bool cols_valid = 2 * nt + h < p.n_blocks;
    if (valid && cols_valid) {
      __nv_bfloat16* row = p.out_bf16 + static_cast<int64_t>(pair) * p.hidden;
      if (p.rs_world > 0) {
        const int q = static_cast<int>(pair / p.rs_pairs_per_owner);
        row = p.rs_dst[q] + (p.rs_row0 + pair - q * p.rs_pairs_per_owner) * p.hidden;
      }
      __nv_bfloat16* dst = row + nt * BN + 128 * h;
#pragma unroll
      for (int i = 0; i < 128; i += 8) {
        uint32_t u[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const __nv_bfloat162 v = __floats2bfloat162_rn(acc[i + 2 * j] * wrow, acc[i + 2 * j + 1] * wrow);
          u[j] = *reinterpret_cast<const uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(dst + i) = make_uint4(u[0], u[1], u[2], u[3]);
      }
    }
  }
  return true;
}

// ---------------------------------------------------------------- warps 4-11: promotion + epilogue
template <bool kGateUp, int S>
__device__ __forceinline__ void epilogue_warps(const GemmParams& p, ControlT<S>* C, TileWalk tw, uint32_t tmem_base,
                                               int warp, int lane, uint8_t* staging) {
  volatile int* abort = &C->abort;
  const int q = warp & 3;         // TMEM lane quarter this warp may access
  const int h = (warp - 4) >> 2;  // column half
  const int r = q * 32 + lane;    // tile row
  const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
  uint32_t kbg = 0;
  uint32_t tiles_done = 0;
  bool alive = true;
  // Column chunks owned by this thread (32 fp32 columns each) and which stage scale they use.
  const uint32_t c0 = kGateUp ? 64 * h : 128 * h;
  const uint32_t c1 = c0 + 32;
  const uint32_t c2 = kGateUp ? 128 + 64 * h : c0 + 64;
  const uint32_t c3 = c2 + 32;
  const int sidx_lo = kGateUp ? 0 : h;
  const int sidx_hi = kGateUp ? 1 : h;

  // Row info of the next tile is loaded one tile ahead.
  int64_t tile = blockIdx.x;
  auto mb_of = [&](int64_t t) {
    int m, n;
    tile_coords(t, tw, m, n);
    return m;
  };
  auto next_valid = [&](int64_t t) {
    while (t < tw.num_tiles && __ldg(p.expert_ids + mb_of(t)) < 0) t += gridDim.x;
    return t;
  };
  tile = next_valid(tile);
  int pair_next = (!kGateUp && tile < tw.num_tiles) ? __ldg(p.sorted_ids + mb_of(tile) * BM + r) : 0;
  for (; tile < tw.num_tiles && alive;) {
    int mb, nt;
    tile_coords(tile, tw, mb, nt);
    const int64_t prow = static_cast<int64_t>(mb) * BM + r;
    const int pair = pair_next;
    const bool valid = pair < p.numel;
    float wrow = 1.0f;
    if (!kGateUp && valid && p.topk_weights) wrow = __ldg(p.topk_weights + pair);
    const int64_t tile_after = next_valid(tile + gridDim.x);
    if (!kGateUp && tile_after < tw.num_tiles) pair_next = __ldg(p.sorted_ids + mb_of(tile_after) * BM + r);

    float acc[128];
#pragma unroll
    for (int i = 0; i < 128; ++i) acc[i] = 0.0f;

    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      const int rs = kbg % SRING;
      const int b = kbg & 1;
      int ok = mbar_wait(&C->tfull[b], (kbg >> 1) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_EPILOGUE, abort);
      ok = ok && mbar_wait(&C->sfull[rs], (kbg / SRING) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_EPILOGUE,
                           abort);
      if (!__all_sync(0xffffffffu, ok)) {
        alive = false;
        break;
      }
      tc_fence_after();
      const float sa = C->as[rs][r];
      const float s_lo = sa * C->bs[rs][sidx_lo];
      const float s_hi = sa * C->bs[rs][sidx_hi];
      __syncwarp();
      if (lane == 0) mbar_arrive(&C->sempty[rs]);
      const uint32_t base = tmem_base + lane_off + static_cast<uint32_t>(b * BN);
      {
        float v0[32], v1[32];
        tmem_ld32(base + c0, v0);
        tmem_ld32(base + c1, v1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) fma2(acc[i], acc[i + 1], v0[i], v0[i + 1], s_lo);
#pragma unroll
        for (int i = 0; i < 32; i += 2) fma2(acc[32 + i], acc[33 + i], v1[i], v1[i + 1], s_lo);
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
        for (int i = 0; i < 32; i += 2) fma2(acc[64 + i], acc[65 + i], v2[i], v2[i + 1], s_hi);
#pragma unroll
        for (int i = 0; i < 32; i += 2) fma2(acc[96 + i], acc[97 + i], v3[i], v3[i + 1], s_hi);
      }
    }
    if (!alive) break;

    if (!finish_tile<kGateUp>(p, C->amax, C->amax_bar, acc, prow, nt, h, r, pair, wrow, valid, tiles_done, lane,
                              abort, staging, C->stg_free, C->stg_full))
      break;
    ++tiles_done;
    tile = tile_after;
  }
  if (staging && lane < 16) bulk_wait_all();  // the rows this thread sent have landed before the CTA exits
}

template <bool kGateUp, int S>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    moe_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  ControlT<S>* C = reinterpret_cast<ControlT<S>*>(smem + S * STAGE_BYTES);
  uint8_t* staging = nullptr;
  if (S == SCATTER_STAGES)
    staging = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem + S * STAGE_BYTES + sizeof(ControlT<S>)) + 127) & ~uintptr_t(127));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int32_t ntpp = __ldg(p.ntpp);
  int num_mb = ntpp / BM;
  if (ntpp < 0 || ntpp % BM != 0 || num_mb > p.max_blocks) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_status(p.status, B2M_STATUS_BAD_ROUTING);
    num_mb = 0;
  }
  const TileWalk tw{static_cast<int64_t>(num_mb) * p.num_nt, num_mb > 0 ? num_mb : 1, p.num_nt, p.nt_begin,
                    p.block_order};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&C->full[s], 1);
      mbar_init(&C->empty[s], 1);
    }
    for (int r = 0; r < SRING; ++r) {
      mbar_init(&C->sfull[r], 1);
      mbar_init(&C->sempty[r], NUM_EPI_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&C->tfull[b], 1);
      mbar_init(&C->tempty[b], NUM_EPI_WARPS);
      mbar_init(&C->amax_bar[b], NUM_EPI_THREADS);
      mbar_init(&C->stg_free[b], NUM_EPI_THREADS);
      mbar_init(&C->stg_full[b], NUM_EPI_THREADS);
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
    reg_dealloc<72>();
    if (warp == 0) {
      stage_producer<kGateUp, S>(&map_a, &map_b, p, smem, C, tw, lane);
    } else if (warp == 1) {
      if (lane == 0) mma_thread<S>(p, smem, C, tw, tmem_base);
      __syncwarp();
    } else if (kGateUp && p.push_world > 1) {
      push_rows(p, lane);
    }
  } else {
    reg_alloc<216>();
    epilogue_warps<kGateUp, S>(p, C, tw, tmem_base, warp, lane, staging);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ================================================================ paired-CTA variant
// Cluster of two CTAs on one work item = a pair of consecutive 128-row blocks of the same
// expert (from the alignment's block-pair list) x one 256-column N tile.  The leader
// issues tcgen05.mma.cta_group::2 (M=256, N=256, K=32): A rows [0,128) come from the
// leader's shared memory and [128,256) from the peer's; the 256 B rows are split the
// same way, so each CTA stages 32 KB per K block (6 stages instead of 4 x 48 KB) and the
// accumulator rows of each CTA land in its own TMEM.  Each CTA promotes and stores its
// own 128 rows exactly as the single-CTA kernel does.  A trailing odd block runs with a
// partner that repeats its rows and skips its stores.  All TMA loads are plain (no
// multicast); the only cluster-wide operations are the MMA commits and barrier arrives.
constexpr int PSTAGES = 6;
constexpr int BH = BN / 2;  // B rows staged per CTA
constexpr int PA_BYTES = BM * BK;
constexpr int PB_BYTES = BH * BK;
constexpr int PSTAGE_BYTES = PA_BYTES + PB_BYTES;
constexpr int GROUP_P = 8;  // raster band: GROUP_P pairs x all N tiles
constexpr uint32_t IDESC_PAIR = idesc_e4m3_f32(2 * BM, BN);

struct PairControl {
  uint64_t full[PSTAGES];   // leader: both CTAs' operand bytes of a stage
  uint64_t empty[PSTAGES];  // each CTA: its stage was consumed by the pair MMA
  uint64_t tfull[2];        // each CTA: accumulator buffer ready
  uint64_t tempty[2];       // leader: both CTAs' epilogues released the buffer (16 warp arrivals)
  uint64_t amax_bar[2];
  uint64_t mma_done;
  uint64_t sfull[SRING];
  uint64_t sempty[SRING];
  uint32_t tmem_base;
  int abort;
  alignas(16) float as[SRING][BM];
  alignas(16) float bs[SRING][4];
  float amax[2][2][BM];
};
constexpr size_t PSMEM_BYTES = size_t(PSTAGES) * PSTAGE_BYTES + sizeof(PairControl) + 1024;
static_assert(PSMEM_BYTES <= 227 * 1024, "shared memory budget (pair)");

struct PairWalk {
  const int32_t* pairs;  // [0] = count, then (first, second or -1)
  int num_pairs;
  int num_nt;
  int64_t num_items;
  int nt_begin;
};

struct PairItem {
  int b0, b1, nt;
};

__device__ __forceinline__ PairItem pair_item(int64_t w, const PairWalk& pw) {
  const int64_t per_band = static_cast<int64_t>(GROUP_P) * pw.num_nt;
  const int64_t band = w / per_band;
  const int first = static_cast<int>(band * GROUP_P);
  const int rows = pw.num_pairs - first < GROUP_P ? pw.num_pairs - first : GROUP_P;
  const int64_t in_band = w - band * per_band;
  const int pi = first + static_cast<int>(in_band % rows);
  PairItem it;
  it.nt = pw.nt_begin + static_cast<int>(in_band / rows);
  it.b0 = __ldg(pw.pairs + 1 + 2 * pi);
  it.b1 = __ldg(pw.pairs + 2 + 2 * pi);
  return it;
}

template <bool kGateUp>
__device__ __forceinline__ void pair_producer(const CUtensorMap* map_a, const CUtensorMap* map_b, const GemmParams& p,
                                              uint8_t* smem, PairControl* C, const PairWalk& pw, uint32_t cr,
                                              int lane) {
  volatile int* abort = &C->abort;
  uint32_t kbg = 0;
  bool alive = true;
  const int64_t cluster = blockIdx.x >> 1;
  const int64_t nclusters = gridDim.x >> 1;
  for (int64_t w = cluster; w < pw.num_items && alive; w += nclusters) {
    const PairItem it = pair_item(w, pw);
    const int mb = (cr == 0 || it.b1 < 0) ? it.b0 : it.b1;
    const int e = __ldg(p.expert_ids + it.b0);
    const int blk1 = 2 * it.nt + 1 < p.n_blocks ? 2 * it.nt + 1 : 2 * it.nt;
    const float* bs0 = p.b_scale + (static_cast<int64_t>(e) * p.n_blocks + 2 * it.nt) * p.num_kb;
    const float* bs1 = p.b_scale + (static_cast<int64_t>(e) * p.n_blocks + blk1) * p.num_kb;
    const int b_row = e * p.n_rows + it.nt * BN + static_cast<int>(cr) * BH;
    float pre0 = 0.0f, pre1 = 0.0f;
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      if ((kb & 31) == 0) {
        const int k = kb + lane;
        pre0 = k < p.num_kb ? __ldg(bs0 + k) : 0.0f;
        pre1 = k < p.num_kb ? __ldg(bs1 + k) : 0.0f;
      }
      const float s0 = __shfl_sync(0xffffffffu, pre0, kb & 31);
      const float s1 = __shfl_sync(0xffffffffu, pre1, kb & 31);
      const int s = kbg % PSTAGES;
      const uint32_t ph = (kbg / PSTAGES) & 1;
      const int r = kbg % SRING;
      const uint32_t rph = (kbg / SRING) & 1;
      int ok = 1;
      if (lane == 0)
        ok = mbar_wait(&C->sempty[r], rph ^ 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_PRODUCER, abort) &&
             mbar_wait(&C->empty[s], ph ^ 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_PRODUCER, abort);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) {
        alive = false;
        break;
      }
      if (lane == 0) {
        uint8_t* sa = smem + s * PSTAGE_BYTES;
        C->bs[r][0] = s0;
        C->bs[r][1] = s1;
        mbar_arrive_expect_tx(&C->sfull[r], BM * 4);
        bulk_load(C->as[r], p.a_scale + static_cast<int64_t>(kb) * p.a_scale_ld + static_cast<int64_t>(mb) * BM,
                  BM * 4, &C->sfull[r]);
        const uint32_t full_leader = mapa_shared(smem_u32(&C->full[s]), 0);
        if (cr == 0) mbar_arrive_expect_tx(&C->full[s], 2 * PSTAGE_BYTES);  // both CTAs' operand bytes
        tma_load_2d_pair(sa, map_a, full_leader, kb * BK, mb * BM);
        tma_load_2d_pair(sa + PA_BYTES, map_b, full_leader, kb * BK, b_row);
      }
      __syncwarp();
    }
  }
  // Drain: the leader's full barriers count both CTAs' bytes; the scale ring is local.
  if (lane == 0) {
    if (cr == 0) {
      const uint32_t first = kbg > PSTAGES ? kbg - PSTAGES : 0;
      for (uint32_t i = first; i < kbg; ++i)
        mbar_wait(&C->full[i % PSTAGES], (i / PSTAGES) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN,
                  nullptr);
    }
    const uint32_t rfirst = kbg > SRING ? kbg - SRING : 0;
    for (uint32_t i = rfirst; i < kbg; ++i)
      mbar_wait(&C->sfull[i % SRING], (i / SRING) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN, nullptr);
  }
  __syncwarp();
}

__device__ __forceinline__ void pair_mma_thread(const GemmParams& p, uint8_t* smem, PairControl* C,
                                                const PairWalk& pw, uint32_t tmem_base) {
  volatile int* abort = &C->abort;
  uint32_t kbg = 0;
  bool alive = true;
  const int64_t cluster = blockIdx.x >> 1;
  const int64_t nclusters = gridDim.x >> 1;
  for (int64_t w = cluster; w < pw.num_items && alive; w += nclusters) {
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      const int s = kbg % PSTAGES;
      const uint32_t ph = (kbg / PSTAGES) & 1;
      const int b = kbg & 1;
      const uint32_t tph = (kbg >> 1) & 1;
      if (!mbar_wait(&C->tempty[b], tph ^ 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_MMA, abort) ||
          !mbar_wait(&C->full[s], ph, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_MMA, abort)) {
        alive = false;
        break;
      }
      tc_fence_after();
      const uint64_t adesc = smem_desc_sw128(smem_u32(smem + s * PSTAGE_BYTES));
      const uint64_t bdesc = smem_desc_sw128(smem_u32(smem + s * PSTAGE_BYTES + PA_BYTES));
      const uint32_t d = tmem_base + static_cast<uint32_t>(b * BN);
#pragma unroll
      for (int k = 0; k < BK / 32; ++k) mma_e4m3_pair(d, adesc + 2 * k, bdesc + 2 * k, IDESC_PAIR, k > 0 ? 1u : 0u);
      mma_commit_pair(&C->empty[s], 0x3);
      mma_commit_pair(&C->tfull[b], 0x3);
    }
  }
  if (kbg > 0) {
    mma_commit_pair(&C->mma_done, 0x1);
    mbar_wait(&C->mma_done, 0, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_DRAIN, nullptr);
  }
}

template <bool kGateUp>
__device__ __forceinline__ void pair_epilogue(const GemmParams& p, PairControl* C, const PairWalk& pw,
                                              uint32_t tmem_base, uint32_t cr, int warp, int lane) {
  volatile int* abort = &C->abort;
  const int q = warp & 3;
  const int h = (warp - 4) >> 2;
  const int r = q * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
  const uint32_t tempty_leader0 = mapa_shared(smem_u32(&C->tempty[0]), 0);
  const uint32_t tempty_leader1 = mapa_shared(smem_u32(&C->tempty[1]), 0);
  uint32_t kbg = 0, tiles_done = 0;
  bool alive = true;
  const uint32_t c0 = kGateUp ? 64 * h : 128 * h;
  const uint32_t c1 = c0 + 32;
  const uint32_t c2 = kGateUp ? 128 + 64 * h : c0 + 64;
  const uint32_t c3 = c2 + 32;
  const int sidx_lo = kGateUp ? 0 : h;
  const int sidx_hi = kGateUp ? 1 : h;
  const int64_t cluster = blockIdx.x >> 1;
  const int64_t nclusters = gridDim.x >> 1;
  for (int64_t w = cluster; w < pw.num_items && alive; w += nclusters) {
    const PairItem it = pair_item(w, pw);
    const bool mine = cr == 0 || it.b1 >= 0;  // a repeated partner block stores nothing
    const int mb = (cr == 0 || it.b1 < 0) ? it.b0 : it.b1;
    const int64_t prow = static_cast<int64_t>(mb) * BM + r;
    int pair = 0;
    float wrow = 1.0f;
    bool valid = false;
    if (!kGateUp) {
      pair = __ldg(p.sorted_ids + prow);
      valid = pair < p.numel;
      if (valid && p.topk_weights) wrow = __ldg(p.topk_weights + pair);
    }
    float acc[128];
#pragma unroll
    for (int i = 0; i < 128; ++i) acc[i] = 0.0f;
    for (int kb = 0; kb < p.num_kb; ++kb, ++kbg) {
      const int rs = kbg % SRING;
      const int b = kbg & 1;
      int ok = mbar_wait(&C->tfull[b], (kbg >> 1) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_EPILOGUE, abort);
      ok = ok && mbar_wait(&C->sfull[rs], (kbg / SRING) & 1, p.pipe_timeout_ns, p.status, B2M_STATUS_TIMEOUT_EPILOGUE,
                           abort);
      if (!__all_sync(0xffffffffu, ok)) {
        alive = false;
        break;
      }
      tc_fence_after();
      const float sa = C->as[rs][r];
      const float s_lo = sa * C->bs[rs][sidx_lo];
      const float s_hi = sa * C->bs[rs][sidx_hi];
      __syncwarp();
      if (lane == 0) mbar_arrive(&C->sempty[rs]);
      const uint32_t base = tmem_base + lane_off + static_cast<uint32_t>(b * BN);
      {
        float v0[32], v1[32];
        tmem_ld32(base + c0, v0);
        tmem_ld32(base + c1, v1);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; i += 2) fma2(acc[i], acc[i + 1], v0[i], v0[i + 1], s_lo);
#pragma unroll
        for (int i = 0; i < 32; i += 2) fma2(acc[32 + i], acc[33 + i], v1[i], v1[i + 1], s_lo);
      }
      {
        float v2[32], v3[32];
        tmem_ld32(base + c2, v2);
        tmem_ld32(base + c3, v3);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        // The loads of this buffer have returned (wait::ld), so the leader may overwrite it:
        // a relaxed arrive suffices and avoids a cluster-scope fence per K block.
        if (lane == 0) mbar_arrive_cluster_relaxed(b ? tempty_leader1 : tempty_leader0);
#pragma unroll
        for (int i = 0; i < 32; i += 2) fma2(acc[64 + i], acc[65 + i], v2[i], v2[i + 1], s_hi);
#pragma unroll
        for (int i = 0; i < 32; i += 2) fma2(acc[96 + i], acc[97 + i], v3[i], v3[i + 1], s_hi);
      }
    }
    if (!alive) break;
    if (mine) {
      if (!finish_tile<kGateUp>(p, C->amax, C->amax_bar, acc, prow, it.nt, h, r, pair, wrow, valid, tiles_done,
                                lane, abort))
        break;
      ++tiles_done;
    }
  }
}

template <bool kGateUp>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const __grid_constant__ GemmParams p, const int32_t* __restrict__ block_pairs) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairControl* C = reinterpret_cast<PairControl*>(smem + PSTAGES * PSTAGE_BYTES);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cr = cluster_ctarank();

  const int32_t ntpp = __ldg(p.ntpp);
  int num_pairs = __ldg(block_pairs);
  if (ntpp < 0 || ntpp % BM != 0 || ntpp / BM > p.max_blocks || num_pairs < 0 || num_pairs > p.max_blocks) {
    if (threadIdx.x == 0 && blockIdx.x == 0) set_status(p.status, B2M_STATUS_BAD_ROUTING);
    num_pairs = 0;
  }
  const PairWalk pw{block_pairs, num_pairs, p.num_nt, static_cast<int64_t>(num_pairs) * p.num_nt, p.nt_begin};

  if (threadIdx.x == 0) {
    for (int s = 0; s < PSTAGES; ++s) {
      mbar_init(&C->full[s], 1);
      mbar_init(&C->empty[s], 1);
    }
    for (int r = 0; r < SRING; ++r) {
      mbar_init(&C->sfull[r], 1);
      mbar_init(&C->sempty[r], NUM_EPI_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&C->tfull[b], 1);
      mbar_init(&C->tempty[b], 2 * NUM_EPI_WARPS);
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
  if (warp == 1) tmem_alloc_pair(&C->tmem_base, TMEM_COLS);
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before any cross-CTA arrive or TMA signal
  tc_fence_after();
  const uint32_t tmem_base = C->tmem_base;

  if (warp < 4) {
    reg_dealloc<56>();
    if (warp == 0) {
      pair_producer<kGateUp>(&map_a, &map_b, p, smem, C, pw, cr, lane);
    } else if (warp == 1) {
      if (lane == 0 && cr == 0) pair_mma_thread(p, smem, C, pw, tmem_base);
      __syncwarp();
    }
  } else {
    reg_alloc<224>();
    pair_epilogue<kGateUp>(p, C, pw, tmem_base, cr, warp, lane);
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the leader's MMAs and the peer's epilogue are done with both CTAs' memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
int encode_map_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                  uint32_t box_inner, uint32_t box_outer) {
  void* fn = nullptr;
  B2M_TRY(driver_entry("cuTensorMapEncodeTiled", &fn));
  const auto encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
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

// Per-device "dynamic shared memory attribute set" flags (the call is idempotent; the
// atomics only make concurrent first calls well defined).
template <typename Kernel>
int ensure_smem_attr(std::atomic<bool> (&done)[64], Kernel kernel, size_t bytes, const char* what) {
  int dev = 0;
  B2M_TRY(check_cuda(cudaGetDevice(&dev), "cudaGetDevice"));
  if (dev >= 0 && dev < 64 && done[dev].load(std::memory_order_acquire)) return B2M_OK;
  B2M_TRY(check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)),
                     what));
  if (dev >= 0 && dev < 64) done[dev].store(true, std::memory_order_release);
  return B2M_OK;
}

template <bool kGateUp, int S = STAGES>
int launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p, int num_sms, cudaStream_t s) {
  // num_sms here is the CTA budget (all SMs, or fewer when the caller keeps SMs for comm kernels)
  constexpr size_t SMEM_BYTES = smem_bytes<S>();
  static std::atomic<bool> attr_done[64];
  B2M_TRY(ensure_smem_attr(attr_done, moe_gemm_kernel<kGateUp, S>, SMEM_BYTES, "gemm: cudaFuncSetAttribute"));
  int64_t upper = static_cast<int64_t>(p.max_blocks) * p.num_nt;
  int grid = static_cast<int>(upper < num_sms ? upper : num_sms);
  if (grid < 1) grid = 1;
  if (p.push_world > 1) {
    // The grid both waits for the peers' flags (producer) and publishes this rank's flags
    // once every CTA's pusher warps are done: all CTAs must be resident together, or
    // resident CTAs could wait on peers whose flags need this rank's unscheduled CTAs.
    // A cooperative launch guarantees co-residency (one CTA per SM, grid <= SMs).
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return check_cuda(cudaLaunchKernelEx(&cfg, moe_gemm_kernel<kGateUp, S>, ma, mb, p),
                      "gemm1 push (cooperative) launch");
  }
  moe_gemm_kernel<kGateUp, S><<<grid, NUM_THREADS, SMEM_BYTES, s>>>(ma, mb, p);
  return check_cuda(cudaGetLastError(), kGateUp ? "gemm1 launch" : "gemm2 launch");
}

template <bool kGateUp>
int launch_gemm_pair(const CUtensorMap& ma, const CUtensorMap& mb, const GemmParams& p, const int32_t* block_pairs,
                     int num_sms, cudaStream_t s) {
  static std::atomic<bool> attr_done[64];
  B2M_TRY(ensure_smem_attr(attr_done, moe_gemm_pair_kernel<kGateUp>, PSMEM_BYTES, "gemm pair: cudaFuncSetAttribute"));
  int64_t upper = static_cast<int64_t>(p.max_blocks) * p.num_nt;  // pairs <= blocks
  int64_t clusters = num_sms / 2;
  if (upper < clusters) clusters = upper;
  if (clusters < 1) clusters = 1;
  moe_gemm_pair_kernel<kGateUp><<<static_cast<int>(2 * clusters), NUM_THREADS, PSMEM_BYTES, s>>>(ma, mb, p,
                                                                                                block_pairs);
  return check_cuda(cudaGetLastError(), kGateUp ? "gemm1 pair launch" : "gemm2 pair launch");
}

}  // namespace
}  // namespace b2m

namespace b2m {
namespace {

struct SourceWait {
  const int32_t* block_order;
  const int32_t* sorted_ids;
  int64_t numel;
  int32_t top_k;
  int64_t tokens_per_src;
  const uint32_t* flags;
  uint32_t epoch;
  const int32_t* push_pos;  // nullptr: no pushing
  int64_t push_pairs;
  void* const* push_a;
  void* const* push_s;
  uint32_t* const* push_flags;
  int32_t* push_counters;
  int32_t world;
  int32_t rank;
};

int gemm1_impl(const void* a_sorted, const float* a_scale_t, int64_t rows_cap, int64_t hidden, const void* w1,
               const float* w1_scale, int32_t num_experts, int32_t inter, const int32_t* expert_ids,
               const int32_t* num_tokens_post_padded, const int32_t* block_pairs, void* out_q, float* out_scale_t,
               const SourceWait* sw, int32_t* dev_status, void* stream) {
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128 || num_experts <= 0 || rows_cap <= 0 ||
      rows_cap % BM)
    return fail(B2M_ERR_ARG, "gemm1: need hidden%%128==0 (%lld), inter%%128==0 (%d), rows_cap%%128==0 (%lld), E>0",
                (long long)hidden, inter, (long long)rows_cap);
  if (!a_sorted || !a_scale_t || !w1 || !w1_scale || !expert_ids || !num_tokens_post_padded || !out_q ||
      !out_scale_t)
    return fail(B2M_ERR_ARG, "gemm1: null pointer");
  if (!aligned16(a_sorted) || !aligned16(a_scale_t) || !aligned16(w1) || !aligned16(out_q))
    return fail(B2M_ERR_ARG, "gemm1: A, A scales, W1 and out_q must be 16-byte aligned");
  if (rows_cap / BM > INT32_MAX) return fail(B2M_ERR_ARG, "gemm1: sizes overflow int32 indices");
  CUtensorMap ma, mb;
  B2M_TRY(encode_map_2d(&ma, a_sorted, hidden, rows_cap, hidden, BK, BM));
  B2M_TRY(encode_map_2d(&mb, w1, hidden, static_cast<uint64_t>(num_experts) * 2 * inter, hidden, BK,
                        block_pairs ? BH : BN));
  GemmParams p{};
  p.expert_ids = expert_ids;
  p.ntpp = num_tokens_post_padded;
  p.max_blocks = static_cast<int32_t>(rows_cap / BM);
  p.num_kb = static_cast<int32_t>(hidden / BK);
  p.num_nt = inter / 128;
  p.n_blocks = 2 * inter / 128;
  p.n_rows = 2 * inter;
  p.a_scale = a_scale_t;
  p.a_scale_ld = rows_cap;
  p.b_scale = w1_scale;
  p.rows_cap = rows_cap;
  p.out_q = static_cast<uint8_t*>(out_q);
  p.out_scale_t = out_scale_t;
  p.inter = inter;
  p.hidden = hidden;
  p.status = dev_status;
  p.timeout_ns = timeout_ns();
  p.pipe_timeout_ns = 2 * p.timeout_ns;
  if (sw) {
    if (block_pairs) return fail(B2M_ERR_UNSUPPORTED, "gemm1_wait: no paired-CTA variant");
    if (!sw->block_order || !sw->sorted_ids || !sw->flags || sw->top_k < 1 || sw->tokens_per_src < 1 ||
        sw->numel < 0 || sw->numel >= INT32_MAX)
      return fail(B2M_ERR_ARG, "gemm1_wait: block_order, sorted_ids and flags are required; top_k, tokens_per_src >= 1");
    // Every source rank of a row must have a flag the producer waits on (at most 8 ranks).
    const int64_t tokens = (sw->numel + sw->top_k - 1) / sw->top_k;
    if ((tokens + sw->tokens_per_src - 1) / sw->tokens_per_src > 8)
      return fail(B2M_ERR_ARG, "gemm1_wait: %lld tokens / %lld per source is more than 8 source ranks",
                  (long long)tokens, (long long)sw->tokens_per_src);
    p.block_order = sw->block_order;
    p.sorted_ids = sw->sorted_ids;
    p.numel = static_cast<int32_t>(sw->numel);
    p.top_k = sw->top_k;
    p.tokens_per_src = sw->tokens_per_src;
    p.src_flags = sw->flags;
    p.src_epoch = sw->epoch;
    if (sw->push_pos) {
      if (sw->world < 2 || sw->world > 8 || sw->rank < 0 || sw->rank >= sw->world || sw->push_pairs < 0 ||
          !sw->push_a || !sw->push_s || !sw->push_flags || !sw->push_counters)
        return fail(B2M_ERR_ARG, "gemm1_wait: push needs 2 <= world <= 8, 0 <= rank < world and every peer table");
      for (int r = 0; r < sw->world; ++r) {
        if (!sw->push_a[r] || !sw->push_s[r] || !sw->push_flags[r] || !aligned16(sw->push_a[r]))
          return fail(B2M_ERR_ARG, "gemm1_wait: bad push pointer %d", r);
        p.push_a[r] = static_cast<uint8_t*>(sw->push_a[r]);
        p.push_s[r] = static_cast<float*>(sw->push_s[r]);
        p.push_flag[r] = sw->push_flags[r];
      }
      p.push_pos = sw->push_pos;
      p.push_pairs = sw->push_pairs;
      p.push_src_a = static_cast<const uint8_t*>(a_sorted);
      p.push_src_s = a_scale_t;
      p.push_counters = sw->push_counters;
      p.push_world = sw->world;
      p.push_rank = sw->rank;
    }
  }
  if (block_pairs) return launch_gemm_pair<true>(ma, mb, p, block_pairs, num_sms, static_cast<cudaStream_t>(stream));
  return launch_gemm<true>(ma, mb, p, num_sms, static_cast<cudaStream_t>(stream));
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_gemm1(const void* a_sorted, const float* a_scale_t, int64_t rows_cap, int64_t hidden,
                         const void* w1, const float* w1_scale, int32_t num_experts, int32_t inter,
                         const int32_t* expert_ids, const int32_t* num_tokens_post_padded,
                         const int32_t* block_pairs, void* out_q, float* out_scale_t, int32_t* dev_status,
                         void* stream) {
  return b2m::gemm1_impl(a_sorted, a_scale_t, rows_cap, hidden, w1, w1_scale, num_experts, inter, expert_ids,
                         num_tokens_post_padded, block_pairs, out_q, out_scale_t, nullptr, dev_status, stream);
}

extern "C" int b2m_gemm1_wait(const void* a_sorted, const float* a_scale_t, int64_t rows_cap, int64_t hidden,
                              const void* w1, const float* w1_scale, int32_t num_experts, int32_t inter,
                              const int32_t* expert_ids, const int32_t* num_tokens_post_padded,
                              const int32_t* block_order, const int32_t* sorted_token_ids, int64_t numel,
                              int32_t top_k, int64_t tokens_per_src, const uint32_t* src_flags, uint32_t epoch,
                              const int32_t* push_pos, int64_t push_pairs, void* const* push_a,
                              void* const* push_s, uint32_t* const* push_flags, int32_t* push_counters,
                              int32_t world, int32_t rank, void* out_q, float* out_scale_t, int32_t* dev_status,
                              void* stream) {
  const b2m::SourceWait sw{block_order, sorted_token_ids, numel, top_k, tokens_per_src, src_flags, epoch,
                           push_pos, push_pairs, push_a, push_s, push_flags, push_counters, world, rank};
  return b2m::gemm1_impl(a_sorted, a_scale_t, rows_cap, hidden, w1, w1_scale, num_experts, inter, expert_ids,
                         num_tokens_post_padded, nullptr, out_q, out_scale_t, &sw, dev_status, stream);
}

namespace b2m {
namespace {

struct Scatter {
  void* const* dst;
  int32_t world;
  int64_t pairs_per_owner;
  int64_t row0;
};

int gemm2_impl(const void* a_fp8, const float* a_scale_t, int64_t rows_cap, int32_t inter, const void* w2,
               const float* w2_scale, int32_t num_experts, int64_t hidden, const int32_t* sorted_token_ids,
               const int32_t* expert_ids, const int32_t* num_tokens_post_padded, const int32_t* block_pairs,
               int64_t numel, const float* topk_weights, void* out_bf16, int64_t col_begin, int64_t col_end,
               int32_t max_ctas, const Scatter* sc, int32_t* dev_status, void* stream) {
  int num_sms = 0;
  B2M_TRY(require_sm100(&num_sms));
  if (hidden <= 0 || hidden % 128 || inter <= 0 || inter % 128 || num_experts <= 0 || rows_cap <= 0 ||
      rows_cap % BM || numel < 0)
    return fail(B2M_ERR_ARG, "gemm2: need hidden%%128==0 (%lld), inter%%128==0 (%d), rows_cap%%128==0 (%lld)",
                (long long)hidden, inter, (long long)rows_cap);
  if (!a_fp8 || !a_scale_t || !w2 || !w2_scale || !sorted_token_ids || !expert_ids || !num_tokens_post_padded ||
      (!sc && !out_bf16))
    return fail(B2M_ERR_ARG, "gemm2: null pointer");
  if (!aligned16(a_fp8) || !aligned16(a_scale_t) || !aligned16(w2) || (out_bf16 && !aligned16(out_bf16)))
    return fail(B2M_ERR_ARG, "gemm2: A, A scales, W2 and out must be 16-byte aligned");
  if (rows_cap / BM > INT32_MAX || numel >= INT32_MAX) return fail(B2M_ERR_ARG, "gemm2: sizes overflow int32");
  if (col_end <= 0) col_end = hidden;
  if (col_begin < 0 || col_begin % BN || col_end > hidden || col_begin >= col_end || (col_end % BN && col_end != hidden))
    return fail(B2M_ERR_ARG, "gemm2: column window [%lld, %lld) must be 256-aligned inside [0, %lld)",
                (long long)col_begin, (long long)col_end, (long long)hidden);
  if (max_ctas > 0 && max_ctas < num_sms) num_sms = max_ctas < 2 ? 2 : max_ctas;
  CUtensorMap ma, mb;
  B2M_TRY(encode_map_2d(&ma, a_fp8, inter, rows_cap, inter, BK, BM));
  B2M_TRY(encode_map_2d(&mb, w2, inter, static_cast<uint64_t>(num_experts) * hidden, inter, BK,
                        block_pairs ? BH : BN));
  GemmParams p{};
  p.sorted_ids = sorted_token_ids;
  p.expert_ids = expert_ids;
  p.ntpp = num_tokens_post_padded;
  p.max_blocks = static_cast<int32_t>(rows_cap / BM);
  p.numel = static_cast<int32_t>(numel);
  p.top_k = 1;
  p.num_kb = inter / BK;
  p.nt_begin = static_cast<int32_t>(col_begin / BN);
  p.num_nt = static_cast<int32_t>((col_end + BN - 1) / BN) - p.nt_begin;
  p.n_blocks = static_cast<int32_t>(hidden / 128);
  p.n_rows = static_cast<int32_t>(hidden);
  p.a_scale = a_scale_t;
  p.a_scale_ld = rows_cap;
  p.b_scale = w2_scale;
  p.rows_cap = rows_cap;
  p.out_bf16 = static_cast<__nv_bfloat16*>(out_bf16);
  p.topk_weights = topk_weights;
  p.hidden = hidden;
  p.status = dev_status;
  p.timeout_ns = timeout_ns();
  p.pipe_timeout_ns = 2 * p.timeout_ns;
  if (sc) {
    if (sc->world < 1 || sc->world > 8 || !sc->dst || sc->pairs_per_owner <= 0 || sc->row0 < 0 ||
        sc->pairs_per_owner * sc->world != numel)
      return fail(B2M_ERR_ARG, "gemm2_scatter: need 1 <= world <= 8, pairs_per_owner * world == numel (%lld), row0 >= 0",
                  (long long)numel);
    for (int r = 0; r < sc->world; ++r) {
      if (!sc->dst[r] || !aligned16(sc->dst[r])) return fail(B2M_ERR_ARG, "gemm2_scatter: bad owner buffer %d", r);
      p.rs_dst[r] = static_cast<__nv_bfloat16*>(sc->dst[r]);
    }
    p.rs_world = sc->world;
    p.rs_pairs_per_owner = sc->pairs_per_owner;
    p.rs_row0 = sc->row0;
  }
  if (block_pairs)
    return launch_gemm_pair<false>(ma, mb, p, block_pairs, num_sms, static_cast<cudaStream_t>(stream));
  if (sc)  // rows leave through the staging tile as whole-row bulk stores
    return launch_gemm<false, SCATTER_STAGES>(ma, mb, p, num_sms, static_cast<cudaStream_t>(stream));
  return launch_gemm<false>(ma, mb, p, num_sms, static_cast<cudaStream_t>(stream));
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_gemm2(const void* a_fp8, const float* a_scale_t, int64_t rows_cap, int32_t inter, const void* w2,
                         const float* w2_scale, int32_t num_experts, int64_t hidden, const int32_t* sorted_token_ids,
                         const int32_t* expert_ids, const int32_t* num_tokens_post_padded,
                         const int32_t* block_pairs, int64_t numel, const float* topk_weights, void* out_bf16,
                         int64_t col_begin, int64_t col_end, int32_t max_ctas, int32_t* dev_status, void* stream) {
  return b2m::gemm2_impl(a_fp8, a_scale_t, rows_cap, inter, w2, w2_scale, num_experts, hidden, sorted_token_ids,
                         expert_ids, num_tokens_post_padded, block_pairs, numel, topk_weights, out_bf16, col_begin,
                         col_end, max_ctas, nullptr, dev_status, stream);
}

extern "C" int b2m_gemm2_scatter(const void* a_fp8, const float* a_scale_t, int64_t rows_cap, int32_t inter,
                                 const void* w2, const float* w2_scale, int32_t num_experts, int64_t hidden,
                                 const int32_t* sorted_token_ids, const int32_t* expert_ids,
                                 const int32_t* num_tokens_post_padded, const int32_t* block_pairs, int64_t numel,
                                 const float* topk_weights, void* const* owner_dst, int32_t world,
                                 int64_t pairs_per_owner, int64_t row0, int32_t* dev_status, void* stream) {
  const b2m::Scatter sc{owner_dst, world, pairs_per_owner, row0};
  return b2m::gemm2_impl(a_fp8, a_scale_t, rows_cap, inter, w2, w2_scale, num_experts, hidden, sorted_token_ids,
                         expert_ids, num_tokens_post_padded, block_pairs, numel, topk_weights, nullptr, 0, 0, 0, &sc,
                         dev_status, stream);
}
