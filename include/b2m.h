/* b2m — B200-native FP8 MoE FFN layer kernels, C ABI.
 *
 * The path these entry points implement is the one stmoonar/td_benchmark times as
 * scheme b2 (moe_bench/overlap/overlap_forward.py:348-622): token-sharded bf16
 * activations -> 1x128 FP8 group quant -> all-gather -> moe_align_block_size ->
 * gate/up grouped GEMM + SiLU*mul -> down grouped GEMM with top-k weights ->
 * top-k combine -> reduce-scatter.
 *
 * Conventions
 *  - Plain pointers and sizes only.  Every pointer is a device pointer unless its
 *    comment says "host".  Outputs are caller-allocated; no entry point allocates
 *    device memory except the b2m_symm_* set-up calls, which exist to allocate.
 *  - Work is enqueued on `stream` (a cudaStream_t passed as void*), asynchronously.
 *  - Return value: B2M_OK (0) or a positive error class; b2m_last_error() gives the
 *    message of the last failing call on the calling host thread.
 *  - Kernels that wait on the pipeline or on peers write a non-zero code into the
 *    caller's `dev_status` word (int32 on the device, may be NULL) instead of
 *    trapping; read it after the stream is synchronised.
 *  - sm_100a (B200) only.
 */
#ifndef B2M_H_
#define B2M_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes (host) */
#define B2M_OK 0
#define B2M_ERR_ARG 1         /* bad shape, stride, alignment or null pointer */
#define B2M_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define B2M_ERR_UNSUPPORTED 3 /* device is not sm_100 or a feature is missing */

/* ---- device status codes (written to dev_status by kernels; first error wins) */
#define B2M_STATUS_OK 0
#define B2M_STATUS_TIMEOUT_PRODUCER 0x101 /* TMA producer waited too long for a free stage */
#define B2M_STATUS_TIMEOUT_MMA 0x102      /* MMA issuer waited too long for operands/TMEM */
#define B2M_STATUS_TIMEOUT_EPILOGUE 0x103 /* epilogue waited too long for an accumulator */
#define B2M_STATUS_TIMEOUT_PEER 0x104     /* a peer rank's chunk flag never arrived */
#define B2M_STATUS_TIMEOUT_DRAIN 0x105    /* teardown could not drain in-flight copies */
#define B2M_STATUS_BAD_ROUTING 0x201      /* num_tokens_post_padded exceeds the block capacity */

/* Library version (major*10000 + minor*100 + patch). */
int b2m_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* b2m_last_error(void);

/* Upper bound for every bounded device-side wait, in nanoseconds (default 2e9).
 * Process-wide; applies to launches made after the call. */
int b2m_set_timeout_ns(uint64_t ns);

/* ---------------------------------------------------------------------------
 * K1  1x128 group FP8 (e4m3) quantisation of bf16 activations.
 * Replaces vLLM per_token_group_fp8_quant as called through
 * moe_kernel_quantize_input (moe_bench/overlap/overlap_forward.py:427-429) and
 * follows the repo oracle moe_bench/verify.py:108-117 exactly:
 *   scale[r,g] = max(amax(|x[r, 128g : 128g+128]|) / 448, 1e-12)   (IEEE division)
 *   q[r,c]     = e4m3_rne(clamp(x[r,c] / scale[r, c/128], -448, 448))
 * x: bf16 [rows, cols] with row stride ldx (elements); q: e4m3 bytes, row stride
 * ldq; scale: fp32 [rows, ceil(cols/128)] with row stride ld_scale.
 * Ragged cols (not a multiple of 128) are handled as if zero padded. */
int b2m_quant_g128(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq,
                   float* scale, int64_t ld_scale, void* stream);

/* Same rule with the scales written K-block-major: scale_t[g * ld_scale_t + r]
 * (the layout the grouped GEMMs read with one bulk copy per 128-row block). */
int b2m_quant_g128_t(const void* x, int64_t rows, int64_t cols, int64_t ldx, void* q, int64_t ldq,
                     float* scale_t, int64_t ld_scale_t, void* stream);

/* K1 + dispatch: quantise bf16 tokens [tokens, hidden] (rule of K1) and write each
 * token's codes and scales to the sorted rows of its top-k pairs:
 *   a_sorted[pair_pos[t*k + j], :] = q[t, :],  a_scale_t[g, pair_pos[t*k + j]] = scale[t, g]
 * (pairs with pair_pos < 0 are skipped).  This replaces the A-row gather the
 * reference's fused_moe_kernel does through sorted_token_ids // top_k
 * (moe_bench/overlap/kernels.py:123-125, :140-141) with one write pass, so the gate/up GEMM
 * reads A with tiled TMA.  q_tok / scale_tok_t (nullable, together) also receive the
 * token-order codes and K-block-major scales (ld_scale_tok_t >= tokens), as the
 * shared expert needs.  hidden % 128 == 0; x rows 16-byte aligned. */
int b2m_quant_dispatch(const void* x, int64_t tokens, int64_t hidden, int64_t ldx, const int32_t* pair_pos,
                       int32_t top_k, void* a_sorted, float* a_scale_t, int64_t rows_cap, void* q_tok,
                       float* scale_tok_t, int64_t ld_scale_tok_t, void* stream);

/* Dispatch of already-quantised token rows (after an all-gather): xq e4m3 [tokens,
 * hidden], xs fp32 [tokens, hidden/128] -> a_sorted / a_scale_t as b2m_quant_dispatch. */
int b2m_dispatch_rows(const void* xq, const float* xs, int64_t tokens, int64_t hidden, const int32_t* pair_pos,
                      int32_t top_k, void* a_sorted, float* a_scale_t, int64_t rows_cap, void* stream);

/* ---------------------------------------------------------------------------
 * K2  moe_align_block_size.
 * Replaces vllm.model_executor.layers.fused_moe.moe_align_block_size
 * (called at moe_bench/overlap/overlap_forward.py:420-422; contract in vLLM
 * moe_align_block_size.py:19-104).  topk_ids: int32 [numel] (flattened [T, k]).
 * Outputs: sorted_token_ids [sorted_cap] (pairs of each expert in ascending flat
 * index, each expert segment padded to a multiple of block_size with the pad id
 * `numel`, tail also `numel`); expert_ids [expert_ids_cap] (expert of each block,
 * remapped through expert_map when non-NULL, -1 for non-local experts and for the
 * tail); num_tokens_post_padded [1].  Required capacities: sorted_cap >=
 * numel + E*(block_size-1) (or numel*block_size when numel < E) and
 * expert_ids_cap >= cdiv(sorted_cap, block_size).  num_experts <= 1024.
 * pair_pos (nullable, int32 [numel]) additionally receives the inverse map: the
 * sorted position of every pair, or -1 when its expert is not local.
 * block_pairs (nullable, int32 [1 + 2*expert_ids_cap]) receives the work list of the
 * paired-CTA GEMMs: [0] = number of pairs P, then P entries (first block, second
 * block or -1) pairing consecutive blocks inside every local expert's segment. */
int b2m_align(const int32_t* topk_ids, int64_t numel, int32_t num_experts, int32_t block_size,
              const int32_t* expert_map, int32_t* sorted_token_ids, int64_t sorted_cap, int32_t* expert_ids,
              int64_t expert_ids_cap, int32_t* num_tokens_post_padded, int32_t* pair_pos, int32_t* block_pairs,
              void* stream);

/* M-block visiting order for b2m_gemm1_wait: block b (of *num_tokens_post_padded / 128)
 * gets key max over its rows of (source - rank) mod world (the step at which
 * b2m_quant_dispatch_push delivers that source here), source of pair p =
 * (p / top_k) / tokens_per_src; order lists the blocks by key, ascending block index
 * within a key.  order_cap <= 16384.  One CTA. */
int b2m_block_order(const int32_t* sorted_token_ids, const int32_t* num_tokens_post_padded, int64_t numel,
                    int32_t top_k, int64_t tokens_per_src, int32_t world, int32_t rank, int32_t* order,
                    int64_t order_cap, int32_t* dev_status, void* stream);

/* ---------------------------------------------------------------------------
 * Gate/up weight layout for K3.  The reference stores w1 as [E, 2I, H] with all
 * gate rows before all up rows (moe_bench/schemes/runtime.py:154-159).  K3 wants,
 * per expert, 128-row blocks interleaved gate0, up0, gate1, up1, ... so one
 * 256-row tile holds matching gate and up rows; its block scales [E, 2I/128, H/128]
 * are permuted the same way.  I (inter) must be a multiple of 128. */
int b2m_w1_interleave(const void* w1, const float* w1_scale, int32_t num_experts, int32_t inter,
                      int64_t hidden, void* w1_out, float* w1_scale_out, void* stream);

/* ---------------------------------------------------------------------------
 * K3  gate/up grouped GEMM with fused SiLU*mul and 1x128 requant (tcgen05 + TMEM + TMA).
 * Replaces invoke_moe_kernel_k_split/fused_moe_kernel_accumulate
 * (moe_bench/overlap/kernels.py:36-214, :317-452) + torch.ops._C.silu_and_mul +
 * the second moe_kernel_quantize_input (overlap_forward.py:530-561).
 * A is expert-sorted: row p of a_sorted holds the codes of the token of pair
 * sorted_token_ids[p] (b2m_quant_dispatch / b2m_dispatch_rows); pad rows are
 * don't-care (their outputs are never read back).  For each 128-row block b with
 * expert e = expert_ids[b] >= 0 and each row p of it:
 *   gu[p, n] = sum_kb (sum_k A[p,k] W1[e,n,k]) * a_scale_t[kb,p] * w1_scale[e,n/128,kb]
 *   h[p, j]  = silu(gu[p, j]) * gu[p, I + j]                      (fp32)
 *   out_q[p, j] / out_scale_t[j/128, p] = 1x128 e4m3 quant of h
 *     (scale rule of K1; codes from h * (1/scale), so a code can differ from the
 *      IEEE-division result by one step in the rare tie case)
 * Blocks with expert -1 are skipped.
 * a_sorted: e4m3 [rows_cap, hidden]; a_scale_t: fp32 [hidden/128, rows_cap];
 * w1: interleaved e4m3 [E, 2I, hidden]; w1_scale: interleaved fp32 [E, 2I/128, hidden/128];
 * out_q: e4m3 [rows_cap, I]; out_scale_t: fp32 [I/128, rows_cap].
 * hidden % 128 == 0, I % 128 == 0, rows_cap % 128 == 0, expert_ids holds
 * rows_cap/128 entries.
 * block_pairs (nullable): the pair list of b2m_align.  When given, the GEMM runs on
 * CTA pairs (cta_group::2, M = 256 over two consecutive blocks of one expert, half
 * of each B tile staged per CTA); otherwise one CTA per 128-row block. */
int b2m_gemm1(const void* a_sorted, const float* a_scale_t, int64_t rows_cap, int64_t hidden, const void* w1,
              const float* w1_scale, int32_t num_experts, int32_t inter, const int32_t* expert_ids,
              const int32_t* num_tokens_post_padded, const int32_t* block_pairs, void* out_q, float* out_scale_t,
              int32_t* dev_status, void* stream);

/* b2m_gemm1 for a tensor-parallel layer whose A rows are stored by the source ranks while
 * it runs, so the all-gather overlaps the GEMM (replaces the all-gather + gate/up GEMM of
 * overlap_forward.py:494-552): M blocks are visited in block_order (b2m_block_order: own
 * rows first), and before a block's loads the producer waits until src_flags[s] >= epoch
 * for every source s among its rows (source of pair p = (p / top_k) / tokens_per_src,
 * from sorted_token_ids; pads = numel).  With push_pos != NULL the GEMM also performs this
 * rank's part of the all-gather: two otherwise idle warps per CTA copy the rows
 * push_pos[0 .. push_pairs) of a_sorted (and their scales) to the same rows of push_a[d] /
 * push_s[d] for every peer d (rank-1, rank-2, ...) and set *push_flags[d] = epoch when
 * done (push_counters: world int32, zero before the first call).  The own rows must be in
 * a_sorted before the call (b2m_quant_dispatch_push with world 1).  Waits are bounded
 * (timeout -> B2M_STATUS_TIMEOUT_PEER in dev_status).  No paired-CTA variant. */
int b2m_gemm1_wait(const void* a_sorted, const float* a_scale_t, int64_t rows_cap, int64_t hidden, const void* w1,
                   const float* w1_scale, int32_t num_experts, int32_t inter, const int32_t* expert_ids,
                   const int32_t* num_tokens_post_padded, const int32_t* block_order,
                   const int32_t* sorted_token_ids, int64_t numel, int32_t top_k, int64_t tokens_per_src,
                   const uint32_t* src_flags, uint32_t epoch, const int32_t* push_pos, int64_t push_pairs,
                   void* const* push_a, void* const* push_s, uint32_t* const* push_flags, int32_t* push_counters,
                   int32_t world, int32_t rank, void* out_q, float* out_scale_t, int32_t* dev_status, void* stream);

/* ---------------------------------------------------------------------------
 * K4  down grouped GEMM with the routed top-k weight in the epilogue.
 * Replaces invoke_moe_kernel_n_split -> vLLM fused_moe_kernel with
 * MUL_ROUTED_WEIGHT=True (moe_bench/overlap/kernels.py:221-310,
 * overlap_forward.py:564-579):
 *   y[p, n] = w(pair) * sum_kb (sum_j Q[p,j] W2[e,n,j]) * a_scale_t[kb,p] * w2_scale[e,n/128,kb]
 *   out[pair, n] = bf16(y[p, n])       for every non-pad row p of a block with expert e >= 0
 * w(pair) = topk_weights[pair] (flat [T*k] fp32), or 1 when topk_weights is NULL.
 * a_fp8 / a_scale_t: K3's out_q / out_scale_t; w2: e4m3 [E, hidden, I];
 * w2_scale: fp32 [E, ceil(hidden/128), I/128]; out: bf16 [numel, hidden] indexed by pair.
 * hidden % 128 == 0, I % 128 == 0.  block_pairs as for b2m_gemm1.
 * Only output columns [col_begin, col_end) are computed (col_begin a multiple of 256,
 * col_end a multiple of 256 or hidden; col_end <= 0 means hidden): the reduce-scatter
 * of one column chunk can then overlap the GEMM of the next, as the reference's N-split
 * chunks do (overlap_forward.py:564-608).  max_ctas > 0 caps the persistent grid so
 * that SMs stay free for a concurrently running exchange kernel. */
int b2m_gemm2(const void* a_fp8, const float* a_scale_t, int64_t rows_cap, int32_t inter, const void* w2,
              const float* w2_scale, int32_t num_experts, int64_t hidden, const int32_t* sorted_token_ids,
              const int32_t* expert_ids, const int32_t* num_tokens_post_padded, const int32_t* block_pairs,
              int64_t numel, const float* topk_weights, void* out_bf16, int64_t col_begin, int64_t col_end,
              int32_t max_ctas, int32_t* dev_status, void* stream);

/* Down GEMM fused with the reduce-scatter push (replaces the down GEMM's bf16 output, the
 * top-k sum and reduce_scatter_tensor, overlap_forward.py:564-608): b2m_gemm2 whose
 * routed-weighted bf16 row of pair p is stored straight into its owner's receive buffer
 * (peer memory) as its tile finishes, so the NVLink transfer runs under the GEMM:
 * owner q = p / pairs_per_owner, row row0 + p - q * pairs_per_owner of owner_dst[q]
 * (bf16 rows of `hidden`).  pairs_per_owner * world == numel, world <= 8.  Tensor
 * parallel: every rank writes its partial of every pair, row0 = rank * pairs_per_owner
 * into owner buffers of world * pairs_per_owner rows; expert parallel: each pair is
 * computed by exactly one rank, row0 = 0 into buffers of pairs_per_owner rows.  The
 * owner sums with b2m_rs_combine once every source has published its flag (b2m_signal
 * after this kernel on the same stream). */
int b2m_gemm2_scatter(const void* a_fp8, const float* a_scale_t, int64_t rows_cap, int32_t inter, const void* w2,
                      const float* w2_scale, int32_t num_experts, int64_t hidden, const int32_t* sorted_token_ids,
                      const int32_t* expert_ids, const int32_t* num_tokens_post_padded, const int32_t* block_pairs,
                      int64_t numel, const float* topk_weights, void* const* owner_dst, int32_t world,
                      int64_t pairs_per_owner, int64_t row0, int32_t* dev_status, void* stream);

/* ---------------------------------------------------------------------------
 * Top-k combine (+ shared expert add).
 * Replaces the torch.sum over top-k and the shared add of
 * moe_bench/overlap/overlap_forward.py:581-597:
 *   out[t, :] = bf16( sum_j staged[t*k + j, :] + shared[t, :] )     (fp32 sum, j ascending)
 * A slot j is skipped when expert_map is non-NULL and expert_map[topk_ids[t*k+j]] < 0.
 * staged: bf16 [tokens*k, hidden]; shared: bf16 [tokens, hidden] or NULL;
 * out: bf16 [tokens, ld_out]. */
int b2m_combine(const void* staged, int64_t tokens, int32_t top_k, int64_t hidden, const int32_t* topk_ids,
                const int32_t* expert_map, const void* shared, void* out, int64_t ld_out, void* stream);

/* ---------------------------------------------------------------------------
 * Peer-memory exchange (fused all-gather / reduce-scatter over NVLink).
 * Replaces the NCCL all_gather_into_tensor of FP8 bytes + scales
 * (moe_bench/overlap/overlap_forward.py:494-505) and reduce_scatter_tensor
 * (:603-608).  Symmetric buffers are cudaMalloc blocks shared by CUDA IPC; flags
 * are uint32 epochs (only grow) published with system-scope release stores and
 * read with bounded acquire spins (timeout -> B2M_STATUS_TIMEOUT_PEER). */

/* Set-up only: zeroed device allocation / free for symmetric buffers. */
int b2m_symm_alloc(int64_t bytes, void** dev_ptr);
int b2m_symm_free(void* dev_ptr);
/* CUDA IPC: handle_out / handle are 64-byte host buffers. */
int b2m_ipc_handle(void* dev_ptr, void* handle_out);
int b2m_ipc_open(const void* handle, void** peer_ptr);
int b2m_ipc_close(void* peer_ptr);

/* Copy-engine transfers between own and peer (IPC-mapped) device memory or pinned host
 * memory, enqueued on `stream`: one cudaMemcpyAsync / cudaMemcpy2DAsync each (pitches
 * and width in bytes).  Used to push a rank's all-gather rows and reduce-scatter blocks
 * and their epoch flags without occupying SMs. */
int b2m_copy_async(void* dst, const void* src, int64_t bytes, void* stream);
int b2m_copy2d_async(void* dst, int64_t dpitch, const void* src, int64_t spitch, int64_t width, int64_t height,
                     void* stream);

/* All-gather push: quantise x [rows, hidden] (rule of K1) and store codes / scales
 * into rows [row0, row0+rows) of every rank's gather buffers q_dst[r] (e4m3
 * [T, hidden]) and s_dst[r] (fp32 [T, hidden/128]); then publish
 * *flag_dst[r] = epoch (flag_dst[r] = this source's flag on rank r).  q_dst, s_dst,
 * flag_dst are host arrays of `world` device pointers (own and peer).  counter: a
 * device int32, zero before the first call, left zero by every call. */
int b2m_quant_push(const void* x, int64_t rows, int64_t hidden, int64_t ldx, int32_t world, void* const* q_dst,
                   void* const* s_dst, int64_t row0, uint32_t* const* flag_dst, uint32_t epoch, int32_t* counter,
                   void* stream);

/* Sparse expert-parallel all-gather (the dispatch of moe_bench/tdx/function/ep_moe_fused.py:375-517:
 * a token goes only to the ranks that hold one of its experts): b2m_quant_push, except that
 * token row0 + i is stored on rank d only when expert_owner[e] == d for one of its experts
 * e = topk_ids[row0 + i, 0..top_k), and always on this rank (row0 / rows).  expert_owner
 * (int32 [num_experts], global expert -> rank) is the same on every rank.
 * topk_ids int32 [T, top_k] is the routing of all T tokens, the same on every rank; rows
 * a destination does not receive keep stale contents, which its dispatch never reads
 * (no pair of that token is local there).  row0 % rows == 0. */
int b2m_quant_push_sparse(const void* x, int64_t rows, int64_t hidden, int64_t ldx, int32_t world, void* const* q_dst,
                          void* const* s_dst, int64_t row0, uint32_t* const* flag_dst, uint32_t epoch, int32_t* counter,
                          const int32_t* topk_ids, int32_t top_k, const int32_t* expert_owner, int32_t num_experts,
                          void* stream);

/* b2m_quant_push for callers that cannot allocate device memory (a runtime that
 * owns every device byte through its own arena, or code that may not call
 * cudaMalloc): no counter argument; the completion counter lives in a static
 * 256-byte device array of this library (held on every GPU that loads it, until
 * exit).  No counterpart in the reference.  Limits: world <= 8 (B2M_ERR_ARG beyond);
 * the scratch need is one counter whatever rows/hidden are.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) and should
 * come before any stream capture.  Each call clears the counter on `stream` before
 * the launch; calls share it, so calls that overlap on the GPU race and must be
 * serialised by the caller.  Allocates nothing (no cudaMalloc/cudaFree). */
int b2m_quant_push_noalloc(const void* x, int64_t rows, int64_t hidden, int64_t ldx, int32_t world,
                           void* const* q_dst, void* const* s_dst, int64_t row0, uint32_t* const* flag_dst,
                           uint32_t epoch, void* stream);

/* All-gather straight into every rank's expert-sorted operand (tensor parallel: the
 * alignment, hence pair_pos [T*top_k], is identical on every rank; replaces the FP8
 * all_gather_into_tensor of overlap_forward.py:494-505 and the row dispatch): quantise
 * x [rows, hidden] (this rank's tokens token0 .. token0+rows-1) exactly as b2m_quant_g128
 * and store each token's codes at row pair_pos[t*top_k + j] of a_dst[d] (e4m3
 * [rows_cap, hidden]) and its scales at s_dst[d][kb * rows_cap + pos] for every j with
 * pos >= 0 and every rank d: the own rank first, then rank-1, rank-2, ...  When the grid
 * is done with destination d, *flag_dst[d] = epoch.  counters: world int32, zero before
 * the first call (calls leave them zero). */
int b2m_quant_dispatch_push(const void* x, int64_t rows, int64_t hidden, int64_t ldx, const int32_t* pair_pos,
                            int32_t top_k, int64_t token0, int32_t world, int32_t rank, void* const* a_dst,
                            void* const* s_dst, int64_t rows_cap, uint32_t* const* flag_dst, uint32_t epoch,
                            int32_t* counters, void* stream);

/* b2m_dispatch_rows on the gather buffer, reading source rank s's rows
 * (tokens [s*T/world, (s+1)*T/world)) only once flags[s] >= epoch (own rank first).
 * top_k <= 8. */
int b2m_dispatch_rows_wait(const void* xq, const float* xs, int64_t tokens, int64_t hidden, const int32_t* pair_pos,
                           int32_t top_k, void* a_sorted, float* a_scale_t, int64_t rows_cap, const uint32_t* flags,
                           int32_t world, int32_t rank, uint32_t epoch, int32_t* dev_status, void* stream);

/* Reduce-scatter push: the combine of b2m_combine over all T tokens for output columns
 * [col_begin, col_end) (8-aligned; col_end <= 0 means hidden); token t's bf16 partial
 * goes to owner q = t / (T/world), row rank*(T/world) + t - q*(T/world) of slot_dst[q]
 * (bf16 [world*T/world, hidden] on rank q); then *flag_dst[q] = epoch.  max_ctas > 0
 * caps the grid (the push shares the GPU with the next chunk's down GEMM).  With
 * counter == NULL nothing is published (flag_dst may be NULL): the partials are only
 * stored, e.g. into a local staging buffer that copy engines push afterwards.
 * sparse != 0 (expert parallel, needs expert_map): a token with no pair on this rank's
 * experts is not sent at all; the owner's sparse reduce does not read that slot (the
 * send-only-routed-rows combine of moe_bench/tdx/function/ep_moe_fused.py:375-517). */
int b2m_combine_push(const void* staged, int64_t tokens, int32_t top_k, int64_t hidden, int64_t col_begin,
                     int64_t col_end, const int32_t* topk_ids, const int32_t* expert_map, const void* shared,
                     int32_t world, int32_t rank, void* const* slot_dst, uint32_t* const* flag_dst, uint32_t epoch,
                     int32_t* counter, int32_t max_ctas, int32_t sparse, void* stream);

/* Publishes epoch to every flag_dst[r] (own, peer or host-mapped memory) as stream
 * memory operations (cuStreamWriteValue32): ordered after all earlier work on
 * `stream`, each preceded by a fence equivalent to __threadfence_system, executed
 * without an SM (so it cannot be starved by kernels that spin on flags). */
int b2m_signal(uint32_t* const* flag_dst, int32_t world, uint32_t epoch, void* stream);

/* Owner side of the scattered reduce-scatter (after b2m_gemm2_scatter on every source):
 * once flags[0..nflags) are all >= epoch,
 *   out[t, :] = bf16( sum_{s < nsrc} sum_{j < top_k} recv[(s*rows + t)*top_k + j, :] + add[t, :] )
 * in fp32 with one rounding (the top-k sum and the cross-rank sum of
 * overlap_forward.py:581-608 in one pass).  add (bf16 [rows, hidden]) may be NULL;
 * a flag wait that runs out records B2M_STATUS_TIMEOUT_PEER in dev_status. */
int b2m_rs_combine(const void* recv, int64_t rows, int32_t top_k, int64_t hidden, int32_t nsrc,
                   const uint32_t* flags, int32_t nflags, uint32_t epoch, const void* add, void* out,
                   int32_t* dev_status, void* stream);

/* Owner side of the reduce-scatter: once the nchunks*world flags (chunk-major) are all
 * >= epoch, out[t, :] = bf16( sum_{r=0..world-1} slots[r*rows + t, :] + add[t, :] )
 * (fp32, rank order).  add (bf16 [rows, hidden]) may be NULL.  With topk_ids (int32
 * [rows, top_k], the routing of this owner's tokens; expert parallel, nchunks == 1) only
 * the sources r holding one of token t's experts (expert_owner[expert] == r) are summed --
 * the slots a sparse b2m_combine_push wrote; the others are zero partials, so the result
 * is that of the dense sum. */
int b2m_rs_reduce(const void* slots, int64_t rows, int64_t hidden, int32_t world, int32_t nchunks,
                  const uint32_t* flags, uint32_t epoch, const void* add, void* out, const int32_t* topk_ids,
                  int32_t top_k, const int32_t* expert_owner, int32_t num_experts, int32_t* dev_status,
                  void* stream);

/* FP8 reduce-scatter push (replaces the b3 path's per-chunk rs_input quantisation +
 * all_to_all_single of codes and scales, moe_bench/overlap/overlap_forward.py:900-928).
 * Token t's partial -- its local top-k rows (+ shared row) summed in fp32, rounded to bf16 --
 * is quantised per 128 columns (scale = max(amax/448, 1e-12), IEEE division, clamp, RNE
 * e4m3) and stored at row rank*(T/world) + t - q*(T/world) of owner q = t / (T/world):
 * codes into code_dst[q] (u8 [T, hidden]), scales into scale_dst[q] (fp32 [T, hidden/128]).
 * Then *flag_dst[q] = epoch for every owner (counter == NULL: nothing published, e.g. when
 * a collective moves the slots afterwards).  hidden % 128 == 0.  sparse != 0: as for
 * b2m_combine_push (tokens without a local pair are not sent). */
int b2m_combine_push_fp8(const void* staged, int64_t tokens, int32_t top_k, int64_t hidden, const int32_t* topk_ids,
                         const int32_t* expert_map, const void* shared, int32_t world, int32_t rank,
                         void* const* code_dst, void* const* scale_dst, uint32_t* const* flag_dst, uint32_t epoch,
                         int32_t* counter, int32_t sparse, void* stream);

/* Owner side of the FP8 reduce-scatter (replaces the dequant-sum of overlap_forward.py:933-946):
 * once flags[0..world) are all >= epoch (flags == NULL: no wait),
 *   out[t, :] = bf16( sum_{r=0..world-1} e4m3(codes[r*rows + t, :]) * scales[r*rows + t, group] + add[t, :] )
 * in fp32, rank order, one rounding.  codes u8 [world*rows, hidden], scales fp32
 * [world*rows, hidden/128]; add (bf16 [rows, hidden]) may be NULL.  topk_ids / top_k /
 * expert_owner / num_experts: the sparse reduce, as for b2m_rs_reduce (NULL: dense). */
int b2m_rs_reduce_fp8(const void* codes, const float* scales, int64_t rows, int64_t hidden, int32_t world,
                      const uint32_t* flags, uint32_t epoch, const void* add, void* out, const int32_t* topk_ids,
                      int32_t top_k, const int32_t* expert_owner, int32_t num_experts, int32_t* dev_status,
                      void* stream);

/* On-device routing (replaces the host-side steps of moe_bench/data/routing.py:58-64 that
 * follow the gate GEMM): per token t, p = softmax(logits[t, :] + bias) (bias fp32 [E], may
 * be NULL; the reference adds strength * log(E * target) under imbalanced routing), the k
 * largest p in descending order (equal p: lower expert first) into topk_ids[t, :] (int32),
 * and p / sum(selected p) into topk_weights[t, :] (fp32).  logits fp32 [tokens, E],
 * 1 <= E <= 1024, 1 <= top_k <= min(32, E). */
int b2m_route_topk(const float* logits, int64_t tokens, int32_t experts, int32_t top_k, const float* bias,
                   int32_t* topk_ids, float* topk_weights, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B2M_H_ */
