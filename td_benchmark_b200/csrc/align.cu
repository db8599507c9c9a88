// K2: moe_align_block_size — histogram, scan and deterministic scatter in one cluster.
//
// Contract: vLLM moe_align_block_size (moe_align_block_size.py:19-104), called by
// the reference at moe_bench/overlap/overlap_forward.py:420-422.  Pairs of one
// expert are emitted in ascending flat index, which makes the output unique.
//
// One cluster of 8 CTAs x 32 warps.  Global warp g = cta * 32 + w owns the contiguous
// pair range [g*chunk, (g+1)*chunk).  Pass A: per-warp per-expert counts (warp_cnt[w][e],
// shared atomics: a count does not depend on the order of the adds); each CTA sums its
// warps into ctot[e], and after a cluster barrier every CTA reads all eight ctot arrays
// through distributed shared memory (no global scratch): the expert totals and the
// counts of the lower CTAs.  Scan (redundant per CTA): padded counts -> expert segment
// starts; per-(warp, expert) bases are the segment start plus the counts of lower CTAs
// and lower warps.  Pass C: each warp walks its range
// again in order and places every pair at base + rank inside its match group; the
// optional inverse map pair_pos[pair] = sorted position (-1 for a non-local expert)
// drives the row dispatch into the sorted operand layout of the gate/up GEMM, and the
// optional block-pair list feeds the paired-CTA GEMMs.
#include "b2m_common.cuh"
#include "b2m_host.h"

namespace b2m {
namespace {

constexpr int kAlignCtas = 8;  // one portable cluster
constexpr int kAlignWarps = 32;  // per CTA
constexpr int kAlignThreads = kAlignWarps * 32;
constexpr int kAlignShared = kAlignWarps + 5;  // int32 arrays of E entries in shared memory
constexpr int kMaxExperts = 1024;
constexpr int kBatch = 8;
constexpr int BM_ORDER = 128;  // M block of the grouped GEMMs  // ids loaded per lane before use (keeps 8 loads in flight per warp)

__global__ void __cluster_dims__(kAlignCtas, 1, 1) __launch_bounds__(kAlignThreads, 1)
    align_kernel(const int32_t* __restrict__ topk_ids, int64_t numel, int32_t num_experts, int32_t bs,
                 const int32_t* __restrict__ expert_map, int32_t* __restrict__ sorted_ids, int64_t sorted_cap,
                 int32_t* __restrict__ expert_ids, int64_t expert_ids_cap, int32_t* __restrict__ ntpp_out,
                 int32_t* __restrict__ pair_pos, int32_t* __restrict__ block_pairs) {
  extern __shared__ int32_t sm[];
  int32_t* warp_cnt = sm;                                  // [32][E] counts, then bases
  int32_t* ctot = warp_cnt + kAlignWarps * num_experts;    // [E] this CTA's counts (read by the cluster)
  int32_t* counts = ctot + num_experts;                    // [E] totals
  int32_t* lower = counts + num_experts;                   // [E] counts of the lower CTAs
  int32_t* starts = lower + num_experts;                   // [E]
  int32_t* pstart = starts + num_experts;                  // [E] first pair index of each expert
  __shared__ int32_t s_total;
  __shared__ int32_t s_pairs;

  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int warp = tid >> 5;
  const uint32_t cta = cluster_ctarank();
  const int64_t gthread = static_cast<int64_t>(cta) * kAlignThreads + tid;
  constexpr int64_t kAllThreads = int64_t(kAlignCtas) * kAlignThreads;
  const int64_t chunk = (numel + kAlignCtas * kAlignWarps - 1) / (kAlignCtas * kAlignWarps);
  const int64_t lo_raw = (static_cast<int64_t>(cta) * kAlignWarps + warp) * chunk;
  const int64_t lo = lo_raw < numel ? lo_raw : numel;
  const int64_t hi = lo + chunk < numel ? lo + chunk : numel;

  for (int i = tid; i < kAlignWarps * num_experts; i += kAlignThreads) warp_cnt[i] = 0;
  __syncthreads();

  // Pass A: per-warp counts (shared-memory atomics; the count does not depend on order).
  int32_t* my_cnt = warp_cnt + warp * num_experts;
  for (int64_t i0 = lo; i0 < hi; i0 += 32 * kBatch) {
    int32_t ev[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = i < hi ? __ldg(topk_ids + i) : -1;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (ev[u] >= 0 && ev[u] < num_experts) atomicAdd(&my_cnt[ev[u]], 1);
  }
  __syncthreads();

  // This CTA's totals, then the cluster's: every CTA reads the eight ctot arrays.
  for (int e = tid; e < num_experts; e += kAlignThreads) {
    int32_t c = 0;
    for (int w = 0; w < kAlignWarps; ++w) c += warp_cnt[w * num_experts + e];
    ctot[e] = c;
  }
  cluster_sync();  // every CTA's ctot is complete and visible to the cluster
  for (int e = tid; e < num_experts; e += kAlignThreads) {
    const uint32_t local = smem_u32(&ctot[e]);
    int32_t all = 0, below = 0;
    for (uint32_t c = 0; c < kAlignCtas; ++c) {
      const int32_t v = c == cta ? ctot[e] : ld_dsmem_s32(mapa_shared(local, c));
      all += v;
      below += c < cta ? v : 0;
    }
    counts[e] = all;
    lower[e] = below;
  }
  cluster_sync();  // no CTA reads another's shared memory after this point

  // Exclusive scan of padded counts (warp 0, 32 experts per step).
  if (warp == 0) {
    int32_t carry = 0;
    for (int e0 = 0; e0 < num_experts; e0 += 32) {
      const int e = e0 + lane;
      const int32_t c = e < num_experts ? counts[e] : 0;
      const int32_t p = (c + bs - 1) / bs * bs;
      int32_t incl = p;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int32_t v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
      }
      if (e < num_experts) starts[e] = carry + incl - p;
      carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) s_total = carry;
    if (block_pairs) {  // pairs of consecutive blocks inside each local expert's segment
      int32_t pc = 0;
      for (int e0 = 0; e0 < num_experts; e0 += 32) {
        const int e = e0 + lane;
        int32_t np = 0;
        if (e < num_experts && (expert_map == nullptr || __ldg(expert_map + e) >= 0)) {
          const int32_t nb = (counts[e] + bs - 1) / bs;
          np = (nb + 1) / 2;
        }
        int32_t incl = np;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int32_t v = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += v;
        }
        if (e < num_experts) pstart[e] = pc + incl - np;
        pc += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) s_pairs = pc;
    }
  }
  __syncthreads();
  const int32_t total = s_total;

  // Per-(warp, expert) bases.
  for (int e = tid; e < num_experts; e += kAlignThreads) {
    int32_t run = starts[e] + lower[e];
    for (int w = 0; w < kAlignWarps; ++w) {
      const int32_t c = warp_cnt[w * num_experts + e];
      warp_cnt[w * num_experts + e] = run;
      run += c;
    }
  }
  __syncthreads();

  // Pass C: ordered scatter (ascending pair index inside every expert segment).
  for (int64_t i0 = lo; i0 < hi; i0 += 32 * kBatch) {
    int32_t ev[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      ev[u] = i < hi ? __ldg(topk_ids + i) : -1;
      if (ev[u] >= num_experts) ev[u] = -1;  // out-of-range ids take no slot
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int64_t i = i0 + u * 32 + lane;
      const int32_t e = ev[u];
      const uint32_t grp = __match_any_sync(0xffffffffu, e);
      const int leader = __ffs(grp) - 1;
      const int rank = __popc(grp & ((1u << lane) - 1u));
      if (e >= 0) sorted_ids[my_cnt[e] + rank] = static_cast<int32_t>(i);
      if (pair_pos && i < hi) {
        const bool local = e >= 0 && (expert_map == nullptr || __ldg(expert_map + e) >= 0);
        pair_pos[i] = local ? my_cnt[e] + rank : -1;
      }
      __syncwarp();
      if (e >= 0 && lane == leader) my_cnt[e] += __popc(grp);
      __syncwarp();
    }
  }

  // Pads inside segments, block -> expert table (each expert by one thread of the cluster).
  const int32_t pad_id = static_cast<int32_t>(numel);
  for (int64_t e64 = gthread; e64 < num_experts; e64 += kAllThreads) {
    const int e = static_cast<int>(e64);
    const int32_t c = counts[e];
    const int32_t st = starts[e];
    const int32_t p = (c + bs - 1) / bs * bs;
    for (int32_t s = st + c; s < st + p; ++s) sorted_ids[s] = pad_id;
    const int32_t mapped = expert_map ? __ldg(expert_map + e) : e;
    for (int32_t b = st / bs; b < (st + p) / bs; ++b) expert_ids[b] = mapped;
    if (block_pairs && mapped >= 0) {
      const int32_t nb = p / bs;
      for (int32_t j = 0; 2 * j < nb; ++j) {
        const int32_t first = st / bs + 2 * j;
        block_pairs[1 + 2 * (pstart[e] + j)] = first;
        block_pairs[2 + 2 * (pstart[e] + j)] = 2 * j + 1 < nb ? first + 1 : -1;
      }
    }
  }
  if (block_pairs && gthread == 0) block_pairs[0] = s_pairs;
  // Tails.
  for (int64_t s = total + gthread; s < sorted_cap; s += kAllThreads) sorted_ids[s] = pad_id;
  for (int64_t b = total / bs + gthread; b < expert_ids_cap; b += kAllThreads) expert_ids[b] = -1;
  if (gthread == 0) *ntpp_out = total;
}

// M-block visiting order of a gate/up GEMM whose rows arrive per source rank
// (b2m_quant_dispatch_push, which serves the own rank first, then rank-1, rank-2, ...; so
// source s reaches this rank at step (s - rank) mod world): block b's key is the latest
// step among its rows' sources, the source of pair p being (p / top_k) / tokens_per_src;
// blocks are listed by key, ascending block index within a key.  One CTA: a warp per block
// computes the key, then one stable compaction pass per key.
constexpr int kOrderThreads = 1024;
constexpr int kOrderMaxBlocks = 16384;

__global__ void __launch_bounds__(kOrderThreads, 1)
    block_order_kernel(const int32_t* __restrict__ sorted_ids, const int32_t* __restrict__ ntpp, int64_t numel,
                       int top_k, int64_t tokens_per_src, int world, int rank, int32_t* __restrict__ order,
                       int64_t order_cap, int32_t* status) {
  __shared__ uint8_t s_key[kOrderMaxBlocks];
  __shared__ int32_t s_warp[kOrderThreads / 32];
  __shared__ int32_t s_base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int64_t nblk = __ldg(ntpp) / BM_ORDER;
  if (nblk < 0 || nblk > order_cap || nblk > kOrderMaxBlocks) {
    if (tid == 0) set_status(status, B2M_STATUS_BAD_ROUTING);
    nblk = 0;
  }
  for (int64_t b = warp; b < nblk; b += kOrderThreads / 32) {
    int hi = -1;
    for (int i = lane; i < BM_ORDER; i += 32) {
      const int32_t id = __ldg(sorted_ids + b * BM_ORDER + i);
      if (id >= 0 && id < numel) {
        const int src = static_cast<int>((id / top_k) / tokens_per_src);
        hi = max(hi, ((src - rank) % world + world) % world);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) hi = max(hi, __shfl_xor_sync(0xffffffffu, hi, off));
    if (lane == 0) s_key[b] = static_cast<uint8_t>(hi < 0 ? 0 : hi);
  }
  if (tid == 0) s_base = 0;
  __syncthreads();
  for (int key = 0; key < world; ++key) {
    for (int64_t b0 = 0; b0 < nblk; b0 += kOrderThreads) {
      const int64_t b = b0 + tid;
      const int flag = (b < nblk && s_key[b] == key) ? 1 : 0;
      const uint32_t bal = __ballot_sync(0xffffffffu, flag);
      if (lane == 0) s_warp[warp] = __popc(bal);
      __syncthreads();
      int before = 0, total = 0;
      for (int w = 0; w < kOrderThreads / 32; ++w) {
        const int c = s_warp[w];
        before += w < warp ? c : 0;
        total += c;
      }
      if (flag) order[s_base + before + __popc(bal & ((1u << lane) - 1u))] = static_cast<int32_t>(b);
      __syncthreads();
      if (tid == 0) s_base += total;
      __syncthreads();
    }
  }
}

}  // namespace
}  // namespace b2m

extern "C" int b2m_align(const int32_t* topk_ids, int64_t numel, int32_t num_experts, int32_t block_size,
                         const int32_t* expert_map, int32_t* sorted_token_ids, int64_t sorted_cap,
                         int32_t* expert_ids, int64_t expert_ids_cap, int32_t* num_tokens_post_padded,
                         int32_t* pair_pos, int32_t* block_pairs, void* stream) {
  using namespace b2m;
  B2M_TRY(require_sm100(nullptr));
  if (num_experts <= 0 || num_experts > kMaxExperts)
    return fail(B2M_ERR_ARG, "align: num_experts=%d outside [1, %d]", num_experts, kMaxExperts);
  if (block_size <= 0 || numel < 0) return fail(B2M_ERR_ARG, "align: bad block_size/numel");
  if (numel >= (int64_t(1) << 31) - int64_t(num_experts) * block_size)
    return fail(B2M_ERR_ARG, "align: numel=%lld overflows int32 indices", (long long)numel);
  int64_t need = numel + int64_t(num_experts) * (block_size - 1);
  if (numel < num_experts && numel * block_size < need) need = numel * block_size;
  if (sorted_cap < need)
    return fail(B2M_ERR_ARG, "align: sorted_cap=%lld < required %lld", (long long)sorted_cap, (long long)need);
  if (expert_ids_cap < (sorted_cap + block_size - 1) / block_size)
    return fail(B2M_ERR_ARG, "align: expert_ids_cap=%lld < cdiv(sorted_cap, block_size)",
                (long long)expert_ids_cap);
  if ((sorted_cap > 0 && !sorted_token_ids) || (expert_ids_cap > 0 && !expert_ids) || !num_tokens_post_padded ||
      (numel > 0 && !topk_ids))
    return fail(B2M_ERR_ARG, "align: null pointer");
  const size_t smem = size_t(kAlignShared) * num_experts * sizeof(int32_t);
  if (smem > 48 * 1024)
    B2M_TRY(check_cuda(
        cudaFuncSetAttribute(align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)),
        "align: cudaFuncSetAttribute"));
  align_kernel<<<kAlignCtas, kAlignThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      topk_ids, numel, num_experts, block_size, expert_map, sorted_token_ids, sorted_cap, expert_ids,
      expert_ids_cap, num_tokens_post_padded, pair_pos, block_pairs);
  return check_cuda(cudaGetLastError(), "align launch");
}

extern "C" int b2m_block_order(const int32_t* sorted_token_ids, const int32_t* num_tokens_post_padded, int64_t numel,
                               int32_t top_k, int64_t tokens_per_src, int32_t world, int32_t rank, int32_t* order,
                               int64_t order_cap, int32_t* dev_status, void* stream) {
  using namespace b2m;
  B2M_TRY(require_sm100(nullptr));
  if (world < 1 || world > 255 || rank < 0 || rank >= world || top_k < 1 || tokens_per_src < 1 || numel < 0 ||
      order_cap < 0 || order_cap > kOrderMaxBlocks)
    return fail(B2M_ERR_ARG, "block_order: bad world/rank/top_k/tokens_per_src or order_cap > %d", kOrderMaxBlocks);
  if (!sorted_token_ids || !num_tokens_post_padded || (order_cap > 0 && !order))
    return fail(B2M_ERR_ARG, "block_order: null pointer");
  block_order_kernel<<<1, kOrderThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      sorted_token_ids, num_tokens_post_padded, numel, top_k, tokens_per_src, world, rank, order, order_cap,
      dev_status);
  return check_cuda(cudaGetLastError(), "block_order launch");
}
