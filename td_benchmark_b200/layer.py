"""FP8 MoE FFN layer on the b2m kernels (per rank).

``MoELayer`` owns the prepared weights and every buffer the forward needs, sized
once for the layer's token count, so the timed forward allocates nothing.  The
forward is the path of the reference's scheme b2
(``moe_bench/overlap/overlap_forward.py:348-622``) and its unfused twins a1/a2
(``moe_bench/schemes/vllm_tp.py:50-64``, ``vllm_ep.py:53-71``):

    align(topk_ids) -> quant(x_local) -> [all-gather] -> dispatch rows to expert order
      -> GEMM1(+SiLU*mul+requant) -> GEMM2(*w) -> combine over top-k (+shared) -> [reduce-scatter]

On one GPU the quant and the dispatch are one kernel (b2m_quant_dispatch).

The exchange steps are pluggable: ``NullExchange`` for one GPU, ``NcclExchange``
(torch.distributed all_gather_into_tensor / reduce_scatter_tensor, the unfused
comparison scheme) and ``P2PExchange`` (fused all-gather / reduce-scatter through
peer memory, ``csrc/symm.cu``).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import ops

BM = 128
# GEMMs on CTA pairs (cta_group::2, two 128-row blocks of one expert per work item).
# Off by default: with per-128-K promotion the TMEM hand-off per K block limits both
# variants alike, and the paired one loses the odd trailing block of every expert
# (measured on B200: equal on the Mixtral shape, slower on DeepSeek-V3).
PAIRED_GEMM = False


@dataclass
class ExpertWeights:
    """One set of expert weights in the kernels' layouts."""
    w1i: torch.Tensor        # e4m3 [E, 2I, H], 128-row interleaved gate/up
    w1i_scale: torch.Tensor  # fp32 [E, 2I/128, H/128] (same interleave)
    w2: torch.Tensor         # e4m3 [E, H, I]
    w2_scale: torch.Tensor   # fp32 [E, H/128, I/128]

    @property
    def num_experts(self) -> int:
        return self.w1i.shape[0]

    @property
    def inter(self) -> int:
        return self.w1i.shape[1] // 2

    @property
    def hidden(self) -> int:
        return self.w1i.shape[2]

    @classmethod
    def prepare(cls, w1: torch.Tensor, w1_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor
                ) -> "ExpertWeights":
        """From the reference layouts (``moe_bench/schemes/runtime.py:27-104``): w1 [E, 2I, H] gate-then-up."""
        w1 = w1.contiguous()
        w1i, w1i_s = ops.w1_interleave(w1, w1_scale.float().contiguous())
        return cls(w1i, w1i_s, w2.contiguous(), w2_scale.float().contiguous())


class _Routing:
    """Alignment buffers for one routing (sized for numel pairs)."""

    def __init__(self, numel: int, num_experts: int, device):
        self.numel = numel
        self.cap, self.nblk = ops.align_sizes(numel, num_experts, BM)
        self.rows_cap = self.nblk * BM
        self.sorted_ids = torch.empty(self.cap, dtype=torch.int32, device=device)
        self.expert_ids = torch.empty(self.nblk, dtype=torch.int32, device=device)
        self.ntpp = torch.empty(1, dtype=torch.int32, device=device)
        self.pair_pos = torch.empty(numel, dtype=torch.int32, device=device)
        self.block_pairs = torch.empty(1 + 2 * self.nblk, dtype=torch.int32, device=device)

    def pairs(self, paired: bool) -> torch.Tensor | None:
        return self.block_pairs if paired else None


class SharedExpert:
    """Dense SwiGLU FFN on the same kernels (one expert, every token routed to it).

    Mirrors ``moe_bench/schemes/shared_expert.py`` (StaticSharedExpert): the
    alignment (identity order) and all buffers are built once.  Its A operand is the
    token-order codes of the already-quantised input (``shared_expert.py:91-102``:
    an FP8 input is used directly with its scales); ``run`` returns bf16 [rows, H].
    """

    def __init__(self, weights: ExpertWeights, rows: int, device):
        self.w = weights
        self.rows = rows
        self.route = _Routing(rows, 1, device)
        nb = (rows + BM - 1) // BM
        ids = torch.full((self.route.cap,), rows, dtype=torch.int32)
        ids[:rows] = torch.arange(rows, dtype=torch.int32)
        self.route.sorted_ids.copy_(ids)
        eids = torch.full((self.route.nblk,), -1, dtype=torch.int32)
        eids[:nb] = 0
        self.route.expert_ids.copy_(eids)
        self.route.ntpp.fill_(nb * BM)
        self.route.pair_pos.copy_(torch.arange(rows, dtype=torch.int32))
        bp = torch.full((1 + 2 * self.route.nblk,), -1, dtype=torch.int32)
        npairs = (nb + 1) // 2
        bp[0] = npairs
        for i in range(npairs):
            bp[1 + 2 * i] = 2 * i
            bp[2 + 2 * i] = 2 * i + 1 if 2 * i + 1 < nb else -1
        self.route.block_pairs.copy_(bp)
        self.paired = PAIRED_GEMM and nb >= 2
        H = weights.hidden
        self.a = torch.empty((self.route.rows_cap, H), dtype=ops.FP8, device=device)
        self.as_t = torch.empty((H // 128, self.route.rows_cap), dtype=torch.float32, device=device)
        self.inter_q = torch.empty((self.route.rows_cap, weights.inter), dtype=ops.FP8, device=device)
        self.inter_st = torch.empty((weights.inter // 128, self.route.rows_cap), dtype=torch.float32, device=device)
        self.out = torch.empty((rows, H), dtype=torch.bfloat16, device=device)

    def load_rows(self, xq: torch.Tensor, xs: torch.Tensor) -> None:
        """Take quantised token rows (row-major scales) as this expert's A operand."""
        ops.dispatch_rows(xq, xs, self.route.pair_pos, 1, self.a, self.as_t)

    def run(self, status: torch.Tensor | None) -> torch.Tensor:
        r = self.route
        bp = r.pairs(self.paired)
        ops.gemm1(self.a, self.as_t, self.w.w1i, self.w.w1i_scale, r.expert_ids, r.ntpp, self.inter_q, self.inter_st,
                  status, block_pairs=bp)
        ops.gemm2(self.inter_q, self.inter_st, self.w.w2, self.w.w2_scale, r.sorted_ids, r.expert_ids, r.ntpp,
                  r.numel, None, self.out, status, block_pairs=bp)
        return self.out


class NullExchange:
    """One rank: quantisation and dispatch in one pass, combine straight into the output."""
    world_size = 1
    rank = 0
    name = "none"

    def setup(self, layer: "MoELayer") -> None:
        pass

    def gather_dispatch(self, layer: "MoELayer", x_local: torch.Tensor) -> None:
        sh = layer.shared
        ops.quant_dispatch(x_local, layer.route.pair_pos, layer.top_k, layer.a_sorted, layer.as_t,
                           None if sh is None else sh.a, None if sh is None else sh.as_t)

    def down_and_scatter(self, layer: "MoELayer", topk_weights, ids, shared_out) -> torch.Tensor:
        layer.gemm2(topk_weights)
        layer._event("gemm2_end")
        return ops.combine(layer.staged, layer.top_k, ids, layer.expert_map, shared_out, layer.out_local)

    def close(self) -> None:
        pass


class NcclExchange:
    """Unfused comparison: NCCL all-gather of FP8 bytes + fp32 scales, NCCL reduce-scatter.

    Same collectives as the reference's b2 (``overlap_forward.py:494-505``, ``:603-608``),
    issued as one call each instead of per chunk.  ``rs_dtype="fp8"`` is the b3 variant
    (``overlap_forward.py:900-946``): every token's partial is quantised per 128 columns
    into a send buffer ordered by owner (``b2m_combine_push_fp8`` with local destinations),
    codes and scales cross with ``all_to_all_single``, and ``b2m_rs_reduce_fp8``
    dequant-sums the received slots in rank order.
    """
    name = "nccl"

    def __init__(self, group=None, rs_dtype: str = "bf16"):
        import torch.distributed as dist
        if rs_dtype not in ("bf16", "fp8"):
            raise ValueError(f"rs_dtype must be 'bf16' or 'fp8', got {rs_dtype!r}")
        self.dist = dist
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rs_dtype = rs_dtype

    def setup(self, layer: "MoELayer") -> None:
        from .symm import ptr_array

        dev = layer.device
        layer.xq = torch.empty((layer.T, layer.H), dtype=ops.FP8, device=dev)
        layer.xs = torch.empty((layer.T, layer.H // 128), dtype=torch.float32, device=dev)
        if self.rs_dtype == "bf16":
            self.partial = torch.empty((layer.T, layer.H), dtype=torch.bfloat16, device=dev)
            return
        T, H, Tl, P = layer.T, layer.H, layer.T_local, self.world_size
        self.send_q = torch.empty((T, H), dtype=torch.uint8, device=dev)
        self.send_s = torch.empty((T, H // 128), dtype=torch.float32, device=dev)
        self.recv_q = torch.empty((T, H), dtype=torch.uint8, device=dev)
        self.recv_s = torch.empty((T, H // 128), dtype=torch.float32, device=dev)
        # destination r's rows start at row r*Tl of the send buffer: the push kernel stores
        # owner r's token i at row rank*Tl + i of destination r, so shift each base back
        # by (r - rank)*Tl rows (the addresses written all fall inside the buffer)
        qb, sb = self.send_q.data_ptr(), self.send_s.data_ptr()
        self._q_dst = ptr_array([qb + (r - self.rank) * Tl * H for r in range(P)])
        self._s_dst = ptr_array([sb + (r - self.rank) * Tl * (H // 128) * 4 for r in range(P)])

    def gather_dispatch(self, layer: "MoELayer", x_local: torch.Tensor) -> None:
        r0 = self.rank * layer.T_local
        xq_l, xs_l = layer.xq[r0:r0 + layer.T_local], layer.xs[r0:r0 + layer.T_local]
        ops.quant_g128(x_local, xq_l, xs_l)
        if layer.shared is not None and layer.ep:
            layer.shared.load_rows(xq_l, xs_l)
        self.dist.all_gather_into_tensor(layer.xq.view(torch.uint8), xq_l.view(torch.uint8), group=self.group)
        self.dist.all_gather_into_tensor(layer.xs, xs_l, group=self.group)
        ops.dispatch_rows(layer.xq, layer.xs, layer.route.pair_pos, layer.top_k, layer.a_sorted, layer.as_t)
        if layer.shared is not None and not layer.ep:
            layer.shared.load_rows(layer.xq, layer.xs)

    def down_and_scatter(self, layer: "MoELayer", topk_weights, ids, shared_out) -> torch.Tensor:
        from . import _lib

        layer.gemm2(topk_weights)
        if self.rs_dtype == "fp8":
            st = ops._stream(layer.device)
            _lib.call("b2m_combine_push_fp8", layer.staged.data_ptr(), layer.T, layer.top_k, layer.H,
                      None if ids is None else ids.data_ptr(),
                      None if layer.expert_map is None else layer.expert_map.data_ptr(),
                      None if shared_out is None else shared_out.data_ptr(), self.world_size, self.rank, self._q_dst,
                      self._s_dst, None, 0, None, 0, st)
            self.dist.all_to_all_single(self.recv_q, self.send_q, group=self.group)
            self.dist.all_to_all_single(self.recv_s, self.send_s, group=self.group)
            add = layer.shared.run(layer.status) if (layer.shared is not None and layer.ep) else None
            _lib.call("b2m_rs_reduce_fp8", self.recv_q.data_ptr(), self.recv_s.data_ptr(), layer.T_local, layer.H,
                      self.world_size, None, 0, None if add is None else add.data_ptr(), layer.out_local.data_ptr(),
                      None, 0, None, 0, layer.status.data_ptr(), st)
            return layer.out_local
        ops.combine(layer.staged, layer.top_k, ids, layer.expert_map, shared_out, self.partial)
        self.dist.reduce_scatter_tensor(layer.out_local, self.partial, group=self.group)
        if layer.shared is not None and layer.ep:
            ops.combine(layer.out_local, 1, None, None, layer.shared.run(layer.status), layer.out_local)
        return layer.out_local

    def close(self) -> None:
        pass


class P2PExchange:
    """Fused exchange over NVLink peer memory: no NCCL on the data path.

    All-gather (``ag_mode``):
      "sm" -- ``b2m_quant_push`` quantises the rank's tokens and stores them into every
           rank's gather buffer with SM stores, then publishes the flags.
      "ce" -- ``b2m_quant_g128`` quantises into the rank's own rows of its gather buffer;
           copy engines copy that contiguous block (codes, then scales) to each peer on
           side streams, and ``b2m_signal`` (a stream memory write, no SM) publishes each
           peer's flag right after its copies.
      "push" -- tensor parallel only: the all-gather runs inside the gate/up GEMM.  Every
           rank aligns the same routing, so the sorted row of each (token, expert) pair is
           the same on every rank.  ``b2m_quant_dispatch_push`` (world 1) quantises the own
           tokens into the own expert-sorted operand; then ``b2m_gemm1_wait`` visits its M
           blocks own-rows-first (``b2m_block_order``), waits per block for the flags of the
           sources the block holds, and two otherwise idle warps per CTA copy the own rows
           to the same rows of every peer (rank-1, rank-2, ...), publishing a flag per peer.
           No gather buffer and no dispatch kernel; top_k copies of each token cross NVLink.
           Measured on 2 B200s (Mixtral TP2): the exposed all-gather falls from 34 us to
           3 us, but the gate/up GEMM runs 5 % slower beside its pusher warps and the own-row
           kernel + block order cost 16 us more than quant + dispatch, so the layer is
           slower there (1030 vs 995 us); at 8 GPUs, where the all-gather + dispatch it
           hides take 63 us, it is expected to win but has not been measured.
      "auto" (default) -- "ce" when a rank's block of codes is at least
           ``AG_CE_MIN_BYTES``, else "sm".  On 8 B200s the copy engines won for the
           DeepSeek-V3 EP shape (7.3 MB per peer: 1648 vs 1683 us per layer) and lost for
           the Mixtral TP shape (2 MB per peer: 512 vs 457 us).
    Either way ``b2m_dispatch_rows_wait`` then moves rows into expert order as each
    source's flag arrives (own rows first).

    Reduce-scatter (``rs_mode``):
      "gemm" -- the down GEMM itself stores each pair's routed-weighted row into its
           owner's receive buffer as the tile finishes (``b2m_gemm2_scatter``), so the
           NVLink traffic runs under the GEMM; ``b2m_signal`` publishes the flags after it
           and the owner sums sources and top-k rows in one pass (``b2m_rs_combine``).  Not
           with a tensor-parallel shared expert (its partials must join before the push).
           The GEMM runs with 3 operand stages so that a 66 KB staging tile fits beside
           them: each finished tile's rows are written there, and one thread per row sends
           the row's 512 bytes to its owner with a bulk copy that drains under the next
           tile's MMAs.  (Storing 16 bytes of a different row per thread and instruction
           straight from registers stalled the GEMM: DeepSeek-V3 EP8 down GEMM 1424 us
           instead of 448.)  Under expert parallelism this is sparse by construction: only
           the pairs this rank computed cross, each to its token's owner.
      "auto" (default) -- "gemm" when a token's pair rows are at most twice the bytes of its
           partials (top_k <= 2 under TP, top_k <= 2P under EP) or with at least
           ``RS_GEMM_MIN_TOKENS`` local tokens; otherwise, and for a tensor-parallel layer with a
           shared expert, "sm".
      "sm" -- after the whole down GEMM, ``b2m_combine_push`` stores each
           token's partial into its owner's slot with SM stores and publishes the flags.
      "ce" -- the down GEMM runs in ``chunks`` column chunks on all SMs; after each chunk
           the combine writes the per-owner partials into a local staging buffer (own
           block straight into the own slot) and the copy engines push each owner's block
           of that chunk into its slot on side streams while the next chunk computes; one
           ``b2m_signal`` publishes the epoch after the last copy.  Measured slower than
           "sm" on 2 and 8 B200s for the Mixtral and DeepSeek-V3 shapes (the strided
           copy-engine pushes ran below the SM stores' NVLink rate and the column chunks
           cost the down GEMM time), kept as the alternative.
      "fp8" -- the b3 payload (``overlap_forward.py:900-946``): as "sm", but each token's
           partial is quantised per 128 columns and its e4m3 codes + fp32 scales are stored in
           the owner's FP8 slot (``b2m_combine_push_fp8``, H + H/32 bytes per row instead of
           2H); the owner dequantises and sums in rank order (``b2m_rs_reduce_fp8``).
    ``b2m_rs_reduce`` then sums the slots in rank order.  Flags are epochs.
    """
    name = "p2p"
    MAX_CHUNKS = 8
    AG_CE_MIN_BYTES = 6 << 20   # between the measured win (7 MiB blocks) and loss (2 MiB blocks)
    # rs_mode 'auto': the down GEMM sends a token's pair rows (top_k per token under TP, top_k / P
    # per rank under EP) where the SM-store path sends one partial.  It pays off when that is at
    # most twice the bytes, or with at least this many local tokens (DeepSeek-V3 shape, 4x the
    # bytes, on 2 B200s: 2-6 % slower than SM stores at 256 and 1024 local tokens, 0.4-2 % faster
    # at 4096; at 2x the bytes on 4 B200s 6 % faster at 2048).
    RS_GEMM_MIN_TOKENS = 2048

    def __init__(self, group=None, chunks: int = 4, rs_mode: str = "auto", ce_streams: int = 2, ag_mode: str = "auto",
                 sparse: bool = False):
        import torch.distributed as dist
        if rs_mode not in ("auto", "ce", "sm", "gemm", "fp8") or ag_mode not in ("ce", "sm", "auto", "push"):
            raise ValueError(f"rs_mode must be 'auto', 'gemm', 'ce', 'sm' or 'fp8' and ag_mode 'push', 'ce', 'sm' or "
                             f"'auto', got {rs_mode!r}, {ag_mode!r}")
        self.ag_mode = ag_mode
        self.sparse = sparse
        self.dist = dist
        self.group = group
        self.world_size = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.epoch = 0
        self.ws = None
        self._shared_out = None   # shared expert output of this forward (expert parallel), run early
        self.chunks_req = chunks if rs_mode == "ce" else 1
        self.rs_mode = rs_mode
        self.ce_streams = max(1, ce_streams)

    @classmethod
    def auto_rs_mode(cls, ep: bool, top_k: int, world: int, tokens_local: int, shared: bool) -> str:
        """The reduce-scatter that ``rs_mode='auto'`` picks: the down GEMM's own stores ('gemm')
        when a token's pair rows are at most twice the bytes of its partials or there are enough
        local tokens to hide them, else SM stores ('sm'); always 'sm' for a tensor-parallel
        layer with a shared expert, whose output must join the partials before they leave."""
        if shared and not ep:
            return "sm"
        rows_per_partial = top_k / world if ep else top_k
        return "gemm" if (rows_per_partial <= 2 or tokens_local >= cls.RS_GEMM_MIN_TOKENS) else "sm"

    def setup(self, layer: "MoELayer") -> None:
        from .symm import SymmetricWorkspace, ptr_array

        P, T, H, Tl = self.world_size, layer.T, layer.H, layer.T_local
        if self.rs_mode == "auto":
            self.rs_mode = self.auto_rs_mode(layer.ep, layer.top_k, P, Tl, layer.shared is not None)
        if self.sparse:
            # sends decided per (token, rank) by SM stores: no contiguous-block copies
            # (rs_mode 'gemm' is sparse already: each pair row goes only to its token's owner)
            if not layer.ep or self.ag_mode in ("ce", "push") or self.rs_mode == "ce":
                raise ValueError("sparse exchange needs expert parallelism, ag_mode 'sm'/'auto' and rs_mode "
                                 "'sm'/'fp8'/'gemm'")
            if layer.E % P:
                raise ValueError(f"sparse exchange needs E={layer.E} divisible by world_size={P}")
            self.ag_mode = "sm"
            if layer.expert_owner is None:   # the contiguous layout: expert e on rank e // (E/P)
                layer.expert_owner = (torch.arange(layer.E, device=layer.device) // (layer.E // P)).to(torch.int32)
        if self.ag_mode == "auto":
            self.ag_mode = "ce" if Tl * H >= self.AG_CE_MIN_BYTES else "sm"
        if self.rs_mode == "gemm" and layer.shared is not None and not layer.ep:
            raise ValueError("rs_mode='gemm' cannot add a tensor-parallel shared expert; use 'sm'")
        if self.ag_mode == "push" and (layer.ep or layer.shared is not None):
            raise ValueError("ag_mode='push' needs a tensor-parallel layer without a shared expert")
        # receive rows of the scattered reduce-scatter: one block of T/P*k rows per source (TP)
        # or a single block (EP: every pair has exactly one writer)
        self.rs_nsrc = (1 if layer.ep else P)
        layout = {"xq": T * H, "xs": T * (H // 128) * 4, "ag_flags": 4 * P, "rs_flags": 4 * P * self.MAX_CHUNKS,
                  "counters": 16}
        if self.rs_mode == "gemm":
            layout["recv"] = self.rs_nsrc * Tl * layer.top_k * H * 2
        elif self.rs_mode == "fp8":
            layout["slots_q"] = T * H                    # [P source blocks of T/P rows, H] e4m3
            layout["slots_s"] = T * (H // 128) * 4       # their fp32 group scales
        else:
            layout["slots"] = T * H * 2
        rows_cap = layer.route.rows_cap
        if self.ag_mode == "push":
            layout.update({"a_sorted": rows_cap * H, "as_t": (H // 128) * rows_cap * 4,
                           "push_counters": 4 * (P + 1)})
        self.ws = SymmetricWorkspace(layout, self.group, layer.device)
        ws = self.ws
        if self.ag_mode == "push":
            # the expert-sorted operand and its scales are written by every source rank
            layer.a_sorted = ws.tensor("a_sorted", (rows_cap, H), torch.uint8).view(ops.FP8)
            layer.as_t = ws.tensor("as_t", (H // 128, rows_cap), torch.float32)
            self._a_dst = ptr_array([ws.peer("a_sorted", r) for r in range(P)])
            self._as_dst = ptr_array([ws.peer("as_t", r) for r in range(P)])
            self.push_counters = ws.local("push_counters")
            self.block_order = torch.empty(layer.route.nblk, dtype=torch.int32, device=layer.device)
            self._own_a = ptr_array([ws.local("a_sorted")])
            self._own_as = ptr_array([ws.local("as_t")])
        layer.xq = ws.tensor("xq", (T, H), torch.uint8).view(ops.FP8)
        layer.xs = ws.tensor("xs", (T, H // 128), torch.float32)
        if self.rs_mode == "gemm":
            self._recv_dst = ptr_array([ws.peer("recv", r) for r in range(P)])
        elif self.rs_mode == "fp8":
            self._slotq_dst = ptr_array([ws.peer("slots_q", r) for r in range(P)])
            self._slots_dst = ptr_array([ws.peer("slots_s", r) for r in range(P)])
        else:
            self.slots = ws.tensor("slots", (T, H), torch.bfloat16)   # [P source blocks of T/P rows, H]
        self.ag_flags = ws.local("ag_flags")
        self.rs_flags = ws.local("rs_flags")
        self.counters = ws.local("counters")
        self._q_dst = ptr_array([ws.peer("xq", r) for r in range(P)])
        self._s_dst = ptr_array([ws.peer("xs", r) for r in range(P)])
        self._ag_dst = ptr_array([ws.peer("ag_flags", r) + 4 * self.rank for r in range(P)])
        self._ag_own = ptr_array([self.ag_flags + 4 * self.rank])
        if self.rs_mode in ("sm", "ce"):
            self._slot_dst = ptr_array([ws.peer("slots", r) for r in range(P)])
        self._rs_dst = ptr_array([ws.peer("rs_flags", r) + 4 * self.rank for r in range(P)])
        # column chunks of the down GEMM (multiples of its 256-column tile)
        ntiles = (H + 255) // 256
        n = max(1, min(self.chunks_req, ntiles, self.MAX_CHUNKS))
        bounds = [round(i * ntiles / n) * 256 for i in range(n + 1)]
        bounds[-1] = H
        self.chunk_cols = [(bounds[i], bounds[i + 1]) for i in range(n) if bounds[i] < bounds[i + 1]]
        if "ce" in (self.rs_mode, self.ag_mode):
            # side streams for the copy engines; peers are dealt round-robin, starting after
            # the own rank so that the ranks do not all copy to the same peer first
            peers = [(self.rank + i) % P for i in range(1, P)]
            ns = max(1, min(self.ce_streams, len(peers)))
            lo, hi = torch.cuda.Stream.priority_range()
            self.ce = [torch.cuda.Stream(layer.device, priority=hi) for _ in range(ns)]
            self._copies = [[] for _ in range(ns)]   # per stream: the peers it copies to
            for i, r in enumerate(peers):
                self._copies[i % ns].append(r)
            self.join_ev = [torch.cuda.Event() for _ in self.ce]
            self.ag_ev = torch.cuda.Event()
            self._ag_own = ptr_array([self.ag_flags + 4 * self.rank])
            self._ag_peer = {r: ptr_array([ws.peer("ag_flags", r) + 4 * self.rank]) for r in peers}
            self._pending_side = False
        if self.rs_mode == "ce":
            # staging rows: token t's partial at row t; the own block goes to the own slot
            self.partial = torch.empty((T, H), dtype=torch.bfloat16, device=layer.device)
            pb, own = self.partial.data_ptr(), ws.peer("slots", self.rank)
            self._stage_dst = ptr_array([own if r == self.rank else pb + (r - self.rank) * Tl * H * 2
                                         for r in range(P)])
            self.chunk_ev = [torch.cuda.Event() for _ in self.chunk_cols]
        self.dist.barrier(group=self.group)

    def gather_dispatch(self, layer: "MoELayer", x_local: torch.Tensor, with_shared: bool = True) -> None:
        from . import _lib

        self.epoch += 1
        st = ops._stream(layer.device)
        Tl, H = layer.T_local, layer.H
        if self.ag_mode == "push":
            self._push_own(layer, x_local, self.epoch)
            return
        if self.ag_mode == "sm" and self.sparse:
            _lib.call("b2m_quant_push_sparse", x_local.data_ptr(), Tl, H, x_local.stride(0), self.world_size,
                      self._q_dst, self._s_dst, self.rank * Tl, self._ag_dst, self.epoch, self.counters,
                      layer.cur_ids.data_ptr(), layer.top_k, layer.expert_owner.data_ptr(), layer.E, st)
        elif self.ag_mode == "sm":
            _lib.call("b2m_quant_push", x_local.data_ptr(), Tl, H, x_local.stride(0), self.world_size, self._q_dst,
                      self._s_dst, self.rank * Tl, self._ag_dst, self.epoch, self.counters, st)
        else:
            self._gather_ce(layer, x_local)
        self._shared_out = None
        if layer.shared is not None and layer.ep and with_shared:
            # Expert parallel: the shared expert works on this rank's own tokens, which are
            # already quantised here, so its GEMMs run now -- while the peers' rows are still
            # crossing NVLink -- instead of after the reduce-scatter (the overlap of the
            # reference's shared stream, overlap_forward.py:513-525).
            r0 = self.rank * Tl
            layer.shared.load_rows(layer.xq[r0:r0 + Tl], layer.xs[r0:r0 + Tl])
            self._shared_out = layer.shared.run(layer.status)
            layer._event("shared_end")
        r = layer.route
        _lib.call("b2m_dispatch_rows_wait", layer.xq.data_ptr(), layer.xs.data_ptr(), layer.T, H, r.pair_pos.data_ptr(),
                  layer.top_k, layer.a_sorted.data_ptr(), layer.as_t.data_ptr(), r.rows_cap, self.ag_flags,
                  self.world_size, self.rank, self.epoch, layer.status.data_ptr(), st)
        if layer.shared is not None and not layer.ep:
            sh = layer.shared
            _lib.call("b2m_dispatch_rows_wait", layer.xq.data_ptr(), layer.xs.data_ptr(), layer.T, H,
                      sh.route.pair_pos.data_ptr(), 1, sh.a.data_ptr(), sh.as_t.data_ptr(), sh.route.rows_cap,
                      self.ag_flags, self.world_size, self.rank, self.epoch, layer.status.data_ptr(), st)

    def _join_side(self, compute) -> None:
        """The compute stream waits for every copy issued on the side streams so far."""
        if getattr(self, "_pending_side", False):
            for s, ev in zip(self.ce, self.join_ev):
                ev.record(s)
                compute.wait_event(ev)
            self._pending_side = False

    def _gather_ce(self, layer: "MoELayer", x_local: torch.Tensor) -> None:
        from . import _lib

        compute = torch.cuda.current_stream(layer.device)
        self._join_side(compute)   # the previous call's copies read the own rows rewritten here
        Tl, H, ws = layer.T_local, layer.H, self.ws
        r0 = self.rank * Tl
        ops.quant_g128(x_local, layer.xq[r0:r0 + Tl], layer.xs[r0:r0 + Tl])
        _lib.call("b2m_signal", self._ag_own, 1, self.epoch, compute.cuda_stream)
        self.ag_ev.record(compute)
        qb, sb = Tl * H, Tl * (H // 128) * 4
        q_off, s_off = r0 * H, r0 * (H // 128) * 4
        for s, peers in zip(self.ce, self._copies):
            s.wait_event(self.ag_ev)
            for r in peers:
                _lib.call("b2m_copy_async", ws.peer("xq", r) + q_off, ws.local("xq") + q_off, qb, s.cuda_stream)
                _lib.call("b2m_copy_async", ws.peer("xs", r) + s_off, ws.local("xs") + s_off, sb, s.cuda_stream)
                _lib.call("b2m_signal", self._ag_peer[r], 1, self.epoch, s.cuda_stream)
        self._pending_side = True

    def _push_own(self, layer: "MoELayer", x_local: torch.Tensor, epoch: int) -> None:
        """Block order, then the own tokens quantised into the own sorted operand (own flag)."""
        from . import _lib

        r, st, Tl, P = layer.route, ops._stream(layer.device), layer.T_local, self.world_size
        _lib.call("b2m_block_order", r.sorted_ids.data_ptr(), r.ntpp.data_ptr(), layer.numel, layer.top_k, Tl, P,
                  self.rank, self.block_order.data_ptr(), self.block_order.numel(), layer.status.data_ptr(), st)
        _lib.call("b2m_quant_dispatch_push", x_local.data_ptr(), Tl, layer.H, x_local.stride(0), r.pair_pos.data_ptr(),
                  layer.top_k, self.rank * Tl, 1, 0, self._own_a, self._own_as, r.rows_cap, self._ag_own, epoch,
                  self.push_counters + 4 * P, st)

    def gemm1(self, layer: "MoELayer") -> bool:
        """Runs the gate/up GEMM when the rows arrive by push; False: the layer runs its own."""
        from . import _lib

        if self.ag_mode != "push":
            return False
        r, Tl, k, P = layer.route, layer.T_local, layer.top_k, self.world_size
        _lib.call("b2m_gemm1_wait", layer.a_sorted.data_ptr(), layer.as_t.data_ptr(), r.rows_cap, layer.H,
                  layer.w.w1i.data_ptr(), layer.w.w1i_scale.data_ptr(), layer.w.num_experts, layer.w.inter,
                  r.expert_ids.data_ptr(), r.ntpp.data_ptr(), self.block_order.data_ptr(), r.sorted_ids.data_ptr(),
                  layer.numel, k, Tl, self.ag_flags, self.epoch, r.pair_pos.data_ptr() + 4 * self.rank * Tl * k,
                  Tl * k, self._a_dst, self._as_dst, self._ag_dst, self.push_counters, P, self.rank,
                  layer.inter_q.data_ptr(), layer.inter_st.data_ptr(), layer.status.data_ptr(),
                  ops._stream(layer.device))
        return True

    def _gemm2_scatter(self, layer: "MoELayer", topk_weights, dst) -> None:
        from . import _lib

        r, P, Tl, k = layer.route, self.world_size, layer.T_local, layer.top_k
        bp = r.pairs(layer.paired)
        row0 = 0 if layer.ep else self.rank * Tl * k
        _lib.call("b2m_gemm2_scatter", layer.inter_q.data_ptr(), layer.inter_st.data_ptr(), r.rows_cap, layer.w.inter,
                  layer.w.w2.data_ptr(), layer.w.w2_scale.data_ptr(), layer.w.num_experts, layer.H,
                  r.sorted_ids.data_ptr(), r.expert_ids.data_ptr(), r.ntpp.data_ptr(),
                  None if bp is None else bp.data_ptr(), layer.numel, topk_weights.reshape(-1).data_ptr(), dst, P,
                  Tl * k, row0, layer.status.data_ptr(), ops._stream(layer.device))

    def _rs_combine(self, layer: "MoELayer", add, epoch: int) -> None:
        from . import _lib

        _lib.call("b2m_rs_combine", self.ws.local("recv"), layer.T_local, layer.top_k, layer.H, self.rs_nsrc,
                  self.rs_flags, self.world_size, epoch, None if add is None else add.data_ptr(),
                  layer.out_local.data_ptr(), layer.status.data_ptr(), ops._stream(layer.device))

    def down_and_scatter(self, layer: "MoELayer", topk_weights, ids, shared_out) -> torch.Tensor:
        from . import _lib

        compute = torch.cuda.current_stream(layer.device)
        P, Tl, H = self.world_size, layer.T_local, layer.H
        idsp = None if ids is None else ids.data_ptr()
        emap = None if layer.expert_map is None else layer.expert_map.data_ptr()
        shp = None if shared_out is None else shared_out.data_ptr()
        if self.rs_mode == "gemm":
            self._gemm2_scatter(layer, topk_weights, self._recv_dst)
            layer._event("gemm2_end")
            _lib.call("b2m_signal", self._rs_dst, P, self.epoch, compute.cuda_stream)
            layer._event("combine_end")
            self._rs_combine(layer, self._shared_out, self.epoch)
            return layer.out_local
        if self.rs_mode == "fp8":
            layer.gemm2(topk_weights)
            layer._event("gemm2_end")
            self._fp8_push_reduce(layer, idsp, emap, shp, self._shared_out, compute)
            return layer.out_local
        if self.rs_mode == "sm":
            layer.gemm2(topk_weights)
            layer._event("gemm2_end")
            _lib.call("b2m_combine_push", layer.staged.data_ptr(), layer.T, layer.top_k, H, 0, H, idsp, emap, shp,
                      P, self.rank, self._slot_dst, self._rs_dst, self.epoch, self.counters + 4, 0, int(self.sparse),
                      compute.cuda_stream)
        else:
            pb = self.partial.data_ptr()
            for c, (c0, c1) in enumerate(self.chunk_cols):
                layer.gemm2(topk_weights, cols=(c0, c1))
                _lib.call("b2m_combine_push", layer.staged.data_ptr(), layer.T, layer.top_k, H, c0, c1, idsp, emap,
                          shp, P, self.rank, self._stage_dst, None, 0, None, 0, 0, compute.cuda_stream)
                self.chunk_ev[c].record(compute)
                for s, peers in zip(self.ce, self._copies):
                    s.wait_event(self.chunk_ev[c])
                    for r in peers:
                        _lib.call("b2m_copy2d_async", self.ws.peer("slots", r) + (self.rank * Tl * H + c0) * 2, H * 2,
                                  pb + (r * Tl * H + c0) * 2, H * 2, (c1 - c0) * 2, Tl, s.cuda_stream)
            for s, ev in zip(self.ce[1:], self.join_ev[1:]):
                ev.record(s)
                self.ce[0].wait_event(ev)
            _lib.call("b2m_signal", self._rs_dst, P, self.epoch, self.ce[0].cuda_stream)
            self._pending_side = True
        layer._event("combine_end")
        add = self._shared_out
        if self.rs_mode == "ce":
            self._join_side(compute)   # staging buffer reuse by the next call
        _lib.call("b2m_rs_reduce", self.slots.data_ptr(), Tl, H, P, 1, self.rs_flags, self.epoch,
                  None if add is None else add.data_ptr(), layer.out_local.data_ptr(), *self._sparse_owner(layer),
                  layer.status.data_ptr(), compute.cuda_stream)
        return layer.out_local

    def _fp8_push_reduce(self, layer: "MoELayer", idsp, emap, shp, add, compute) -> None:
        """FP8 reduce-scatter: quantised partials to the owners' slots, then the owner dequant-sum."""
        from . import _lib

        _lib.call("b2m_combine_push_fp8", layer.staged.data_ptr(), layer.T, layer.top_k, layer.H, idsp, emap, shp,
                  self.world_size, self.rank, self._slotq_dst, self._slots_dst, self._rs_dst, self.epoch,
                  self.counters + 4, int(self.sparse), compute.cuda_stream)
        layer._event("combine_end")
        _lib.call("b2m_rs_reduce_fp8", self.ws.local("slots_q"), self.ws.local("slots_s"), layer.T_local, layer.H,
                  self.world_size, self.rs_flags, self.epoch, None if add is None else add.data_ptr(),
                  layer.out_local.data_ptr(), *self._sparse_owner(layer), layer.status.data_ptr(), compute.cuda_stream)

    def _sparse_owner(self, layer: "MoELayer") -> tuple:
        """(routing rows of this rank's tokens, top_k, expert -> rank table, E) for the sparse
        owner reduce, or the dense reduce's (None, 0, None, 0)."""
        if not self.sparse:
            return None, 0, None, 0
        return (layer.cur_ids.data_ptr() + 4 * self.rank * layer.T_local * layer.top_k, layer.top_k,
                layer.expert_owner.data_ptr(), layer.E)

    def exchange_alone(self, layer: "MoELayer", x_local: torch.Tensor, topk_ids: torch.Tensor) -> bool:
        """The all-gather and the reduce-scatter of one forward with no GEMM between them.

        Runs exactly the exchange kernels of ``forward`` -- quantise + push to every peer +
        dispatch as each source arrives, then combine + push of the staged rows to their
        owners + the owner reduce -- so a caller can time the communication of a step by
        itself (the reference's T_comm).  The staged rows are those of the last forward;
        the result lands in the layer's output buffer and is not meaningful.  Only for the
        SM / copy-engine all-gather with the SM reduce-scatter; returns False otherwise."""
        from . import _lib

        if self.ag_mode not in ("sm", "ce") or self.rs_mode not in ("sm", "fp8"):
            return False
        layer.cur_ids = topk_ids
        self.gather_dispatch(layer, x_local, with_shared=False)
        compute = torch.cuda.current_stream(layer.device)
        emap = None if layer.expert_map is None else layer.expert_map.data_ptr()
        idsp = topk_ids.data_ptr() if layer.ep else None
        if self.rs_mode == "fp8":
            self._fp8_push_reduce(layer, idsp, emap, None, None, compute)
            return True
        _lib.call("b2m_combine_push", layer.staged.data_ptr(), layer.T, layer.top_k, layer.H, 0, layer.H, idsp, emap,
                  None, self.world_size, self.rank, self._slot_dst, self._rs_dst, self.epoch, self.counters + 4, 0,
                  int(self.sparse), compute.cuda_stream)
        self._join_side(compute)
        _lib.call("b2m_rs_reduce", self.slots.data_ptr(), layer.T_local, layer.H, self.world_size, 1, self.rs_flags,
                  self.epoch, None, layer.out_local.data_ptr(), *self._sparse_owner(layer), layer.status.data_ptr(),
                  compute.cuda_stream)
        return True

    def extra_launches(self) -> int:
        """Kernels per forward beyond align, quant(+push), dispatch, GEMM1, GEMM2, combine(+push)."""
        if self.rs_mode == "gemm":
            return 0                                   # GEMM2 pushes, the owner combine replaces the combine
        return 1 + 2 * (len(self.chunk_cols) - 1)      # owner-side reduce; GEMM2/combine per extra chunk

    def close(self) -> None:
        if self.ws is not None:
            self.ws.close()
            self.ws = None


class MoELayer:
    """Per-rank FP8 MoE layer.

    ``tokens``: gathered token count T (= world_size * local tokens); ``top_k``;
    ``weights``: this rank's expert weights (TP: I/P columns of every expert; EP:
    the local experts); ``expert_map``: int32 [E_global] global->local id (-1 when
    not local) for EP, None for TP; ``shared``: shared-expert weights, applied on
    the gathered tokens before the reduce-scatter (TP, ``overlap_forward.py:513-525``)
    or on the local tokens after it (EP, ``vllm_ep.py:67-69``).
    """

    def __init__(self, weights: ExpertWeights, tokens: int, top_k: int, global_num_experts: int,
                 expert_map: torch.Tensor | None = None, shared: ExpertWeights | None = None,
                 exchange=None, device=None, expert_owner: torch.Tensor | None = None):
        self.w = weights
        self.exchange = exchange or NullExchange()
        self.P = self.exchange.world_size
        if tokens % self.P:
            raise ValueError(f"tokens={tokens} must be divisible by world_size={self.P}")
        self.T = tokens
        self.T_local = tokens // self.P
        self.top_k = top_k
        self.E = global_num_experts
        self.H = weights.hidden
        self.device = torch.device(device) if device is not None else weights.w1i.device
        self.expert_map = expert_map
        self.ep = expert_map is not None
        # int32 [E] global expert -> rank (expert parallel; None: the contiguous layout)
        self.expert_owner = None if expert_owner is None else expert_owner.to(self.device, torch.int32).contiguous()
        dev = self.device
        self.numel = tokens * top_k
        self.route = _Routing(self.numel, global_num_experts, dev)
        H = self.H
        self.xq = self.xs = None   # token-order all-gather target, owned by the exchange
        self.cur_ids = None        # routing of the current forward
        self.a_sorted = torch.empty((self.route.rows_cap, H), dtype=ops.FP8, device=dev)  # expert order
        self.as_t = torch.empty((H // 128, self.route.rows_cap), dtype=torch.float32, device=dev)
        self.inter_q = torch.empty((self.route.rows_cap, weights.inter), dtype=ops.FP8, device=dev)
        self.inter_st = torch.empty((weights.inter // 128, self.route.rows_cap), dtype=torch.float32, device=dev)
        self.staged = torch.empty((self.numel, H), dtype=torch.bfloat16, device=dev)
        self.out_local = torch.empty((self.T_local, H), dtype=torch.bfloat16, device=dev)
        self.status = ops.new_status(dev)
        self.events: list | None = None   # set to [] to record (name, cuda.Event) around the GEMMs
        # CTA pairs need two blocks of one expert; with under 2 blocks per expert on
        # average (decode shapes) a pair would mostly run with an idle partner.
        self.paired = PAIRED_GEMM and self.numel >= 2 * BM * global_num_experts
        self.shared = None
        self.shared_local = None
        if shared is not None:
            rows = self.T_local if self.ep else tokens
            self.shared = SharedExpert(shared, rows, dev)
        self.exchange.setup(self)

    # -- stages (exposed for tests and staged timing)
    def _event(self, name: str) -> None:
        if self.events is not None:
            ev = torch.cuda.Event(enable_timing=True)
            ev.record(torch.cuda.current_stream(self.device))
            self.events.append((name, ev))

    def route_and_dispatch(self, x_local: torch.Tensor, topk_ids: torch.Tensor) -> None:
        """Alignment, then quantisation + (all-gather) + row dispatch into expert order."""
        r = self.route
        self.cur_ids = topk_ids   # the routing of this forward (the sparse exchange reads it)
        ops.moe_align_block_size(topk_ids, BM, self.E, self.expert_map, out=(r.sorted_ids, r.expert_ids, r.ntpp),
                                 pair_pos=r.pair_pos, block_pairs=r.pairs(self.paired))
        self._event("align_end")
        self.exchange.gather_dispatch(self, x_local)

    def gemm1(self) -> None:
        r = self.route
        self._event("gemm1_start")
        hook = getattr(self.exchange, "gemm1", None)
        if hook is None or not hook(self):
            ops.gemm1(self.a_sorted, self.as_t, self.w.w1i, self.w.w1i_scale, r.expert_ids, r.ntpp, self.inter_q,
                      self.inter_st, self.status, block_pairs=r.pairs(self.paired))
        self._event("gemm1_end")

    def gemm2(self, topk_weights: torch.Tensor, cols: tuple[int, int] | None = None, max_ctas: int = 0) -> None:
        r = self.route
        ops.gemm2(self.inter_q, self.inter_st, self.w.w2, self.w.w2_scale, r.sorted_ids, r.expert_ids, r.ntpp,
                  self.numel, topk_weights.reshape(-1), self.staged, self.status, block_pairs=r.pairs(self.paired),
                  cols=cols, max_ctas=max_ctas)

    def kernel_launches(self) -> int:
        """b2m kernels one forward launches."""
        sh = self.shared is not None
        name = self.exchange.name
        if name == "none":
            return 5 + (2 if sh else 0)             # align, quant+dispatch, GEMM1, GEMM2, combine (+shared GEMMs)
        n = 6                                      # align, quant(+push), dispatch, GEMM1, GEMM2, combine(+push)
        if name == "p2p":
            n += self.exchange.extra_launches()
        if sh:
            n += 3 + (1 if (self.ep and name == "nccl") else 0)
        return n

    def forward(self, x_local: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                out: torch.Tensor | None = None) -> torch.Tensor:
        """x_local bf16 [T/P, H]; topk_ids int32 / topk_weights fp32 [T, k] (all tokens) -> bf16 [T/P, H].

        The result goes to ``out`` (contiguous bf16 [T/P, H] on this device) when given, else to
        the layer's own output buffer, which the next call overwrites."""
        if out is not None:
            if out.shape != self.out_local.shape or out.dtype != torch.bfloat16 or out.device != self.device or \
                    not out.is_contiguous():
                raise ValueError(f"out must be contiguous bf16 {tuple(self.out_local.shape)} on {self.device}")
            own, self.out_local = self.out_local, out
            try:
                return self.forward(x_local, topk_ids, topk_weights)
            finally:
                self.out_local = own
        self.route_and_dispatch(x_local, topk_ids)
        self.gemm1()
        shared_out = None
        if self.shared is not None and not self.ep:
            shared_out = self.shared.run(self.status)
            self._event("shared_end")
        out = self.exchange.down_and_scatter(self, topk_weights, topk_ids if self.ep else None, shared_out)
        self._event("scatter_end")
        return out

    def check(self) -> None:
        ops.check_status(self.status, "MoELayer")

    def close(self) -> None:
        self.exchange.close()
