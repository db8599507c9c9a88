"""torch-tensor wrappers over the b2m C ABI.

Each wrapper checks shapes/dtypes/devices, then enqueues the kernel on the
current CUDA stream of the tensors' device.  Outputs may be passed in (the layer
pre-allocates everything once); when omitted they are allocated here.
"""
from __future__ import annotations

import torch

from . import _lib

FP8 = torch.float8_e4m3fn
BLOCK = 128

STATUS_NAMES = {
    0x101: "TIMEOUT_PRODUCER", 0x102: "TIMEOUT_MMA", 0x103: "TIMEOUT_EPILOGUE", 0x104: "TIMEOUT_PEER",
    0x105: "TIMEOUT_DRAIN", 0x201: "BAD_ROUTING",
}


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda(t: torch.Tensor, name: str) -> None:
    _need(t.is_cuda, f"{name} must be a CUDA tensor")


def new_status(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def check_status(status: torch.Tensor, what: str = "b2m kernel") -> None:
    """Synchronise on the status word and raise if a kernel recorded an error."""
    code = int(status.item())
    if code:
        status.zero_()
        raise RuntimeError(f"{what}: device status 0x{code:x} ({STATUS_NAMES.get(code, 'unknown')})")


def quant_g128(x: torch.Tensor, q: torch.Tensor | None = None, scale: torch.Tensor | None = None
               ) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 [rows, cols] -> (e4m3 [rows, cols], fp32 [rows, ceil(cols/128)])."""
    _cuda(x, "x")
    _need(x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1, "x must be 2D bf16 with unit column stride")
    rows, cols = x.shape
    groups = (cols + BLOCK - 1) // BLOCK
    if q is None:
        q = torch.empty((rows, cols), dtype=FP8, device=x.device)
    if scale is None:
        scale = torch.empty((rows, groups), dtype=torch.float32, device=x.device)
    _need(q.shape == (rows, cols) and q.stride(1) == 1 and q.element_size() == 1, "bad q buffer")
    _need(scale.shape[0] == rows and scale.shape[1] >= groups and scale.stride(1) == 1 and
          scale.dtype == torch.float32, "bad scale buffer")
    _lib.call("b2m_quant_g128", x.data_ptr(), rows, cols, x.stride(0), q.data_ptr(), q.stride(0),
              scale.data_ptr(), scale.stride(0), _stream(x.device))
    return q, scale


def quant_g128_t(x: torch.Tensor, q: torch.Tensor, scale_t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 [rows, cols] -> e4m3 q [rows, cols] and K-block-major fp32 scale_t [cols/128, >= rows]."""
    _cuda(x, "x")
    _need(x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1, "x must be 2D bf16 with unit column stride")
    rows, cols = x.shape
    _need(scale_t.shape[0] == (cols + BLOCK - 1) // BLOCK and scale_t.shape[1] >= rows and scale_t.stride(1) == 1,
          "scale_t must be [cols/128, >= rows]")
    _lib.call("b2m_quant_g128_t", x.data_ptr(), rows, cols, x.stride(0), q.data_ptr(), q.stride(0),
              scale_t.data_ptr(), scale_t.stride(0), _stream(x.device))
    return q, scale_t


def quant_dispatch(x: torch.Tensor, pair_pos: torch.Tensor, top_k: int, a_sorted: torch.Tensor,
                   a_scale_t: torch.Tensor, q_tok: torch.Tensor | None = None,
                   scale_tok_t: torch.Tensor | None = None) -> None:
    """Quantise bf16 tokens and write codes/scales to the sorted rows of their pairs (+ optional token order)."""
    _cuda(x, "x")
    tokens, hidden = x.shape
    rows_cap = a_sorted.shape[0]
    _need(x.dtype == torch.bfloat16 and x.stride(1) == 1, "x must be bf16 with unit column stride")
    _need(pair_pos.dtype == torch.int32 and pair_pos.numel() == tokens * top_k, "pair_pos must be int32 [T*k]")
    _need(a_sorted.shape[1] == hidden and tuple(a_scale_t.shape) == (hidden // BLOCK, rows_cap),
          "a_sorted [rows_cap, H] / a_scale_t [H/128, rows_cap] mismatch")
    ld_tok = 0
    if q_tok is not None:
        _need(q_tok.shape[1] == hidden and q_tok.shape[0] >= tokens and scale_tok_t.shape[1] >= tokens,
              "bad token-order outputs")
        ld_tok = scale_tok_t.stride(0)
    _lib.call("b2m_quant_dispatch", x.data_ptr(), tokens, hidden, x.stride(0), pair_pos.data_ptr(), top_k,
              a_sorted.data_ptr(), a_scale_t.data_ptr(), rows_cap, _ptr(q_tok), _ptr(scale_tok_t), ld_tok,
              _stream(x.device))


def dispatch_rows(xq: torch.Tensor, xs: torch.Tensor, pair_pos: torch.Tensor, top_k: int, a_sorted: torch.Tensor,
                  a_scale_t: torch.Tensor) -> None:
    """Quantised token rows (+ row-major scales) -> sorted rows of their pairs."""
    _cuda(xq, "xq")
    tokens, hidden = xq.shape
    rows_cap = a_sorted.shape[0]
    _need(xq.is_contiguous() and xs.is_contiguous() and tuple(xs.shape) == (tokens, hidden // BLOCK),
          "xq / xs must be contiguous [T, H] / [T, H/128]")
    _need(pair_pos.dtype == torch.int32 and pair_pos.numel() == tokens * top_k, "pair_pos must be int32 [T*k]")
    _lib.call("b2m_dispatch_rows", xq.data_ptr(), xs.data_ptr(), tokens, hidden, pair_pos.data_ptr(), top_k,
              a_sorted.data_ptr(), a_scale_t.data_ptr(), rows_cap, _stream(xq.device))


def align_sizes(numel: int, num_experts: int, block_size: int) -> tuple[int, int]:
    """Buffer sizes of moe_align_block_size (vLLM moe_align_block_size.py:74-88)."""
    max_padded = numel + num_experts * (block_size - 1)
    if numel < num_experts:
        max_padded = min(numel * block_size, max_padded)
    return max_padded, (max_padded + block_size - 1) // block_size


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int,
                         expert_map: torch.Tensor | None = None,
                         out: tuple[torch.Tensor, torch.Tensor, torch.Tensor] | None = None,
                         pair_pos: torch.Tensor | None = None, block_pairs: torch.Tensor | None = None
                         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Same signature and outputs as vLLM's ``moe_align_block_size`` (without the padding flags).

    ``pair_pos`` (int32 [numel], optional) also receives each pair's sorted position (-1: non-local);
    ``block_pairs`` (int32 [1 + 2*nblk], optional) the block-pair work list of the paired-CTA GEMMs."""
    _cuda(topk_ids, "topk_ids")
    _need(topk_ids.dtype == torch.int32 and topk_ids.is_contiguous(), "topk_ids must be contiguous int32")
    numel = topk_ids.numel()
    cap, nblk = align_sizes(numel, num_experts, block_size)
    if out is None:
        sorted_ids = torch.empty(cap, dtype=torch.int32, device=topk_ids.device)
        expert_ids = torch.empty(nblk, dtype=torch.int32, device=topk_ids.device)
        ntpp = torch.empty(1, dtype=torch.int32, device=topk_ids.device)
    else:
        sorted_ids, expert_ids, ntpp = out
    if expert_map is not None:
        _need(expert_map.dtype == torch.int32 and expert_map.numel() >= num_experts, "expert_map must be int32 [E]")
    if pair_pos is not None:
        _need(pair_pos.dtype == torch.int32 and pair_pos.numel() == numel, "pair_pos must be int32 [numel]")
    if block_pairs is not None:
        _need(block_pairs.dtype == torch.int32 and block_pairs.numel() >= 1 + 2 * expert_ids.numel(),
              "block_pairs must be int32 [1 + 2*len(expert_ids)]")
    _lib.call("b2m_align", topk_ids.data_ptr(), numel, num_experts, block_size, _ptr(expert_map),
              sorted_ids.data_ptr(), sorted_ids.numel(), expert_ids.data_ptr(), expert_ids.numel(),
              ntpp.data_ptr(), _ptr(pair_pos), _ptr(block_pairs), _stream(topk_ids.device))
    return sorted_ids, expert_ids, ntpp


def w1_interleave(w1: torch.Tensor, w1_scale: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """[E, 2I, H] gate-then-up -> 128-row interleaved gate/up layout (+ scales)."""
    _cuda(w1, "w1")
    e, n2, h = w1.shape
    _need(n2 % 256 == 0 and h % 128 == 0 and w1.is_contiguous() and w1_scale.is_contiguous(),
          "w1 must be contiguous [E, 2I, H] with I % 128 == 0 and H % 128 == 0")
    _need(tuple(w1_scale.shape) == (e, n2 // 128, h // 128), "w1_scale must be [E, 2I/128, H/128]")
    out = torch.empty_like(w1)
    out_s = torch.empty_like(w1_scale)
    _lib.call("b2m_w1_interleave", w1.data_ptr(), w1_scale.data_ptr(), e, n2 // 2, h, out.data_ptr(),
              out_s.data_ptr(), _stream(w1.device))
    return out, out_s


def gemm1(a_sorted: torch.Tensor, a_scale_t: torch.Tensor, w1i: torch.Tensor, w1i_scale: torch.Tensor,
          expert_ids: torch.Tensor, ntpp: torch.Tensor, out_q: torch.Tensor | None = None,
          out_scale_t: torch.Tensor | None = None, status: torch.Tensor | None = None,
          block_pairs: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Gate/up grouped GEMM + SiLU*mul + 1x128 requant on expert-sorted A.

    a_sorted e4m3 [rows_cap, H], a_scale_t fp32 [H/128, rows_cap] -> (q [rows_cap, I], scale_t [I/128, rows_cap])."""
    _cuda(a_sorted, "a_sorted")
    rows_cap, hidden = a_sorted.shape
    e, n2, h2 = w1i.shape
    inter = n2 // 2
    _need(h2 == hidden and a_sorted.is_contiguous() and w1i.is_contiguous(), "A / W1 shape mismatch")
    _need(a_scale_t.is_contiguous() and tuple(a_scale_t.shape) == (hidden // 128, rows_cap),
          "a_scale_t must be [H/128, rows_cap]")
    _need(expert_ids.numel() * 128 >= rows_cap, "expert_ids shorter than rows_cap/128")
    if out_q is None:
        out_q = torch.empty((rows_cap, inter), dtype=FP8, device=a_sorted.device)
    if out_scale_t is None:
        out_scale_t = torch.empty((inter // 128, rows_cap), dtype=torch.float32, device=a_sorted.device)
    _lib.call("b2m_gemm1", a_sorted.data_ptr(), a_scale_t.data_ptr(), rows_cap, hidden, w1i.data_ptr(),
              w1i_scale.data_ptr(), e, inter, expert_ids.data_ptr(), ntpp.data_ptr(), _ptr(block_pairs),
              out_q.data_ptr(), out_scale_t.data_ptr(), _ptr(status), _stream(a_sorted.device))
    return out_q, out_scale_t


def gemm2(a_q: torch.Tensor, a_scale_t: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor,
          sorted_ids: torch.Tensor, expert_ids: torch.Tensor, ntpp: torch.Tensor, numel: int,
          topk_weights: torch.Tensor | None, out: torch.Tensor | None = None,
          status: torch.Tensor | None = None, block_pairs: torch.Tensor | None = None,
          cols: tuple[int, int] | None = None, max_ctas: int = 0) -> torch.Tensor:
    """Down grouped GEMM, routed weight in the epilogue.  Returns bf16 [numel, H] indexed by flat pair."""
    _cuda(a_q, "a_q")
    rows_cap, inter = a_q.shape
    e, hidden, i2 = w2.shape
    _need(i2 == inter and w2.is_contiguous() and a_q.is_contiguous(), "A / W2 shape mismatch")
    _need(tuple(a_scale_t.shape) == (inter // 128, rows_cap), "a_scale_t must be [I/128, rows_cap]")
    if topk_weights is not None:
        _need(topk_weights.dtype == torch.float32 and topk_weights.is_contiguous() and
              topk_weights.numel() == numel, "topk_weights must be contiguous fp32 with numel entries")
    if out is None:
        out = torch.empty((numel, hidden), dtype=torch.bfloat16, device=a_q.device)
    _lib.call("b2m_gemm2", a_q.data_ptr(), a_scale_t.data_ptr(), rows_cap, inter, w2.data_ptr(), w2_scale.data_ptr(),
              e, hidden, sorted_ids.data_ptr(), expert_ids.data_ptr(), ntpp.data_ptr(), _ptr(block_pairs), numel,
              _ptr(topk_weights), out.data_ptr(), 0 if cols is None else cols[0], 0 if cols is None else cols[1],
              max_ctas, _ptr(status), _stream(a_q.device))
    return out


def combine(staged: torch.Tensor, top_k: int, topk_ids: torch.Tensor | None = None,
            expert_map: torch.Tensor | None = None, shared: torch.Tensor | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [T*k, H] -> bf16 [T, H]: fp32 sum over the k slots (+ shared), one rounding."""
    _cuda(staged, "staged")
    pairs, hidden = staged.shape
    tokens = pairs // top_k
    if out is None:
        out = torch.empty((tokens, hidden), dtype=torch.bfloat16, device=staged.device)
    _need(out.shape[0] >= tokens and out.stride(1) == 1, "bad combine output")
    _lib.call("b2m_combine", staged.data_ptr(), tokens, top_k, hidden, _ptr(topk_ids), _ptr(expert_map),
              _ptr(shared), out.data_ptr(), out.stride(0), _stream(staged.device))
    return out


def route_topk(logits: torch.Tensor, top_k: int, bias: torch.Tensor | None = None,
               out: tuple[torch.Tensor, torch.Tensor] | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 router logits [T, E] (+ per-expert bias [E]) -> (int32 ids [T, k], fp32 weights [T, k]):
    softmax, top-k in descending order, renormalised (``moe_bench/data/routing.py:58-64``)."""
    _cuda(logits, "logits")
    _need(logits.dtype == torch.float32 and logits.dim() == 2 and logits.is_contiguous(),
          "logits must be contiguous fp32 [T, E]")
    tokens, experts = logits.shape
    if bias is not None:
        _need(bias.dtype == torch.float32 and bias.numel() == experts and bias.is_contiguous(), "bias must be fp32 [E]")
    if out is None:
        ids = torch.empty((tokens, top_k), dtype=torch.int32, device=logits.device)
        wts = torch.empty((tokens, top_k), dtype=torch.float32, device=logits.device)
    else:
        ids, wts = out
        _need(ids.dtype == torch.int32 and wts.dtype == torch.float32 and ids.is_contiguous() and wts.is_contiguous()
              and tuple(ids.shape) == (tokens, top_k) and tuple(wts.shape) == (tokens, top_k),
              "out must be contiguous int32 / fp32 [T, k]")
    _lib.call("b2m_route_topk", logits.data_ptr(), tokens, experts, top_k, _ptr(bias), ids.data_ptr(), wts.data_ptr(),
              _stream(logits.device))
    return ids, wts
