"""Overlap-level entry points — the reference's ``moe_bench.overlap`` contract.

``MoEOverlapState(n_chunks_gateup, n_chunks_down, tp_group)`` and
``moe_forward_overlap_fp8ag(state, hidden_states, w1, w2, topk_weights, topk_ids,
top_k, global_num_experts, expert_map=None, shared_mlp=None, M_valid=None,
w1_scale=None, w2_scale=None, w2_zp=None, a1_scale=None, a2_scale=None,
block_shape=None) -> [M_local, K] bf16`` keep the reference signature
(``moe_bench/overlap/overlap_forward.py:61-97``, ``:348-366``) and run the b2m path.

Weights arrive in the reference layout (w1 [E, 2I_r, K] gate-then-up, block scales
[E, 2I_r/128, K/128]); the interleaved copy and all buffers are prepared on the
first call for a given (weights, token count, expert map) and cached in the state.
``shared_mlp`` may be an ``ExpertWeights`` or any object exposing
``w1_fp8, w1_scale, w2_fp8, w2_scale`` (the fields of the reference's
``StaticSharedExpert``, ``moe_bench/schemes/shared_expert.py:15-30``).
Only 128x128 block scales and group-128 activations are supported, as in the
reference's FP8 contract (``moe_bench/worker.py:117-121``).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Optional

import torch

from ..layer import ExpertWeights, MoELayer, NcclExchange, NullExchange, P2PExchange

__all__ = ["MoEOverlapState", "moe_forward_overlap_fp8ag", "moe_forward_overlap_fp8ag_fp8rs"]


@dataclass
class MoEOverlapState:
    """Per-model state of the overlap entry points (``overlap_forward.py:61-97``).

    ``exchange`` picks how the ranks of ``tp_group`` exchange tokens and partials:
    ``"p2p"`` (default) the fused all-gather / reduce-scatter through NVLink peer memory
    (``P2PExchange``), ``"nccl"`` NCCL collectives (the unfused comparison).  With one
    rank there is no exchange.  ``n_chunks_*`` are kept for interface parity: the b2m
    path does not split the GEMMs into stream-level chunks."""
    n_chunks_gateup: int = 4
    n_chunks_down: int = 4
    tp_group: Any = field(default=None, repr=False)
    exchange: str = "p2p"
    _layers: dict = field(default_factory=dict, repr=False, init=False)

    def __post_init__(self) -> None:
        if self.exchange not in ("p2p", "nccl"):
            raise ValueError(f"exchange={self.exchange!r} must be 'p2p' or 'nccl'")

    @property
    def tp_size(self) -> int:
        import torch.distributed as dist

        if not dist.is_available() or not dist.is_initialized():
            return 1
        return dist.get_world_size(self.tp_group)

    def ensure_streams(self, device) -> None:
        """Kept for interface parity; the b2m path orders all work on the caller's stream."""

    def release(self) -> None:
        """Free every prepared layer (collective with P2P exchanges: all ranks call it)."""
        for layer in self._layers.values():
            layer.close()
        self._layers.clear()

    def make_exchange(self, rs_fp8: bool = False):
        if self.tp_size == 1:
            return NullExchange()
        if self.exchange == "p2p":
            return P2PExchange(self.tp_group, rs_mode="fp8" if rs_fp8 else "auto")
        return NcclExchange(self.tp_group, rs_dtype="fp8" if rs_fp8 else "bf16")


def _as_expert_weights(shared_mlp: Any) -> Optional[ExpertWeights]:
    if shared_mlp is None or isinstance(shared_mlp, ExpertWeights):
        return shared_mlp
    try:
        return ExpertWeights.prepare(shared_mlp.w1_fp8, shared_mlp.w1_scale, shared_mlp.w2_fp8, shared_mlp.w2_scale)
    except AttributeError as exc:
        raise TypeError("shared_mlp must be ExpertWeights or expose w1_fp8/w1_scale/w2_fp8/w2_scale") from exc


def _forward(state: MoEOverlapState, rs_fp8: bool, hidden_states: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
             topk_weights: torch.Tensor, topk_ids: torch.Tensor, top_k: int, global_num_experts: int,
             expert_map: Optional[torch.Tensor], shared_mlp: Any, M_valid: Optional[int],
             w1_scale: Optional[torch.Tensor], w2_scale: Optional[torch.Tensor], w2_zp: Optional[torch.Tensor],
             a1_scale: Optional[torch.Tensor], a2_scale: Optional[torch.Tensor],
             block_shape: Optional[list[int]]) -> torch.Tensor:
    if w1_scale is None or w2_scale is None:
        raise ValueError("moe_forward_overlap_fp8ag needs w1_scale and w2_scale (block FP8 weights)")
    if block_shape is not None and list(block_shape) != [128, 128]:
        raise ValueError(f"block_shape={block_shape} unsupported: the b2m kernels use 128x128 weight blocks")
    if w2_zp is not None or a1_scale is not None or a2_scale is not None:
        raise ValueError("zero points and static activation scales are not part of the FP8 group-128 contract")
    P = state.tp_size
    m_local = hidden_states.shape[0]
    tokens = m_local * P
    if M_valid is not None and M_valid < tokens:
        raise ValueError("M_valid < gathered tokens is not supported: pad routing to the full token count")
    key = (w1.data_ptr(), w2.data_ptr(), tokens, top_k, global_num_experts,
           None if expert_map is None else expert_map.data_ptr(), id(shared_mlp), rs_fp8)
    layer = state._layers.get(key)
    if layer is None:
        weights = ExpertWeights.prepare(w1, w1_scale, w2, w2_scale)
        layer = MoELayer(weights, tokens, top_k, global_num_experts, expert_map=expert_map,
                         shared=_as_expert_weights(shared_mlp), exchange=state.make_exchange(rs_fp8),
                         device=hidden_states.device)
        state._layers[key] = layer
    ids = topk_ids[:tokens].to(torch.int32).contiguous()
    wts = topk_weights[:tokens].to(torch.float32).contiguous()
    return layer.forward(hidden_states.contiguous(), ids, wts)


def moe_forward_overlap_fp8ag(state: MoEOverlapState, hidden_states: torch.Tensor, w1: torch.Tensor,
                              w2: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor, top_k: int,
                              global_num_experts: int, expert_map: Optional[torch.Tensor] = None,
                              shared_mlp: Any = None, M_valid: Optional[int] = None,
                              w1_scale: Optional[torch.Tensor] = None, w2_scale: Optional[torch.Tensor] = None,
                              w2_zp: Optional[torch.Tensor] = None, a1_scale: Optional[torch.Tensor] = None,
                              a2_scale: Optional[torch.Tensor] = None,
                              block_shape: Optional[list[int]] = None) -> torch.Tensor:
    """FP8 all-gather, bf16 reduce-scatter (the reference's b2, ``overlap_forward.py:348-622``)."""
    return _forward(state, False, hidden_states, w1, w2, topk_weights, topk_ids, top_k, global_num_experts,
                    expert_map, shared_mlp, M_valid, w1_scale, w2_scale, w2_zp, a1_scale, a2_scale, block_shape)


def moe_forward_overlap_fp8ag_fp8rs(state: MoEOverlapState, hidden_states: torch.Tensor, w1: torch.Tensor,
                                    w2: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                                    top_k: int, global_num_experts: int, expert_map: Optional[torch.Tensor] = None,
                                    shared_mlp: Any = None, M_valid: Optional[int] = None,
                                    w1_scale: Optional[torch.Tensor] = None,
                                    w2_scale: Optional[torch.Tensor] = None,
                                    w2_zp: Optional[torch.Tensor] = None, a1_scale: Optional[torch.Tensor] = None,
                                    a2_scale: Optional[torch.Tensor] = None,
                                    block_shape: Optional[list[int]] = None) -> torch.Tensor:
    """FP8 all-gather and FP8 reduce-scatter payload (the reference's b3,
    ``overlap_forward.py:625-953``): each rank's partials cross as 1x128 e4m3 codes +
    fp32 scales and the owner dequant-sums them in rank order.  With one rank it is the
    same computation as ``moe_forward_overlap_fp8ag`` (nothing is exchanged)."""
    return _forward(state, True, hidden_states, w1, w2, topk_weights, topk_ids, top_k, global_num_experts,
                    expert_map, shared_mlp, M_valid, w1_scale, w2_scale, w2_zp, a1_scale, a2_scale, block_shape)
