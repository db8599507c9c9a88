"""Seeded synthetic inputs for the BASELINE workloads (set-up, outside timing).

The objects keep the field names of the reference's data bundle
(``moe_bench/data/bundle.py:21-40``, ``checkpoint.py:11-25``, ``routing.py:11-25``),
so the scheme builders read either.  Values follow the BASELINE configs:

* activations ``hidden ~ N(0, 1)`` (seed + 17), fp32, sliced per rank, cast to bf16;
* expert weights ``~ N(0, weight_std)`` fp32, generated expert by expert with a
  per-expert seed (so every world size sees the same experts), 128x128 block FP8;
* router logits ``~ N(0, 1)`` [T, E] (seed + 1); under Zipf routing the logits get
  ``strength * log(E * p)`` with p the shuffled Zipf target (the steps of
  ``moe_bench/data/routing.py:28-38, 58-64``); softmax -> top-k -> renormalise,
  fp32 weights and int32 ids.

No dataset is involved: shapes are the model shapes named by the configs.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from .configs import RoutingCfg, RunCfg
from .weights import dequantize_block128, quantize_block128


@dataclass
class QuantizedTensor:
    fp8: torch.Tensor
    scale: torch.Tensor
    bf16: torch.Tensor | None = None   # dequantised view, only built when asked for (tests)


@dataclass
class WeightCheckpoint:
    w1: QuantizedTensor
    w2: QuantizedTensor
    shared_w1: QuantizedTensor | None
    shared_w2: QuantizedTensor | None
    gate_weight: Any = None


@dataclass
class RoutingBundle:
    topk_ids_local: torch.Tensor
    topk_weights_local: torch.Tensor
    topk_ids_full: torch.Tensor
    topk_weights_full: torch.Tensor
    stats: Any = None


@dataclass
class DataBundle:
    hidden_local: torch.Tensor            # bf16 [T/P, H]
    ckpt: WeightCheckpoint
    routing: RoutingBundle
    golden: Any = None
    hidden_full: torch.Tensor | None = None   # bf16 [T, H]


def _gen(device, seed: int) -> torch.Generator:
    return torch.Generator(device=device).manual_seed(int(seed) & 0x7FFFFFFFFFFF)


def expert_stack(n: int, rows: int, cols: int, std: float, seed: int, device) -> QuantizedTensor:
    """n experts of [rows, cols], each ~N(0, std) from its own seed, block-quantised one at a time."""
    fp8 = torch.empty((n, rows, cols), dtype=torch.float8_e4m3fn, device=device)
    scale = torch.empty((n, (rows + 127) // 128, (cols + 127) // 128), dtype=torch.float32, device=device)
    for e in range(n):
        w = torch.randn((1, rows, cols), generator=_gen(device, seed * 1_000_003 + e), device=device,
                        dtype=torch.float32) * std
        q, s = quantize_block128(w)
        fp8[e] = q[0]
        scale[e] = s[0]
    return QuantizedTensor(fp8, scale)


def target_distribution(cfg: RoutingCfg, experts: int) -> torch.Tensor:
    if cfg.imbalance_kind == "none":
        return torch.full((experts,), 1.0 / experts, dtype=torch.float32)
    ranks = torch.arange(1, experts + 1, dtype=torch.float32)
    probs = ranks.pow(-cfg.zipf_s)
    perm = torch.randperm(experts, generator=_gen("cpu", cfg.gate_seed))
    shuffled = torch.empty_like(probs)
    shuffled[perm] = probs
    return shuffled / shuffled.sum()


def route(logits: torch.Tensor, top_k: int, cfg: RoutingCfg) -> tuple[torch.Tensor, torch.Tensor]:
    """softmax -> top-k -> renormalise (``moe_bench/data/routing.py:58-64``) on given logits."""
    logits = logits.float()
    if cfg.imbalance_kind != "none":
        probs = target_distribution(cfg, logits.shape[-1]).to(logits.device)
        logits = logits + cfg.strength * torch.log(logits.shape[-1] * probs)
    w, ids = torch.topk(torch.softmax(logits, dim=-1), top_k, dim=-1)
    w = (w / w.sum(dim=-1, keepdim=True)).to(torch.float32).contiguous()
    return ids.to(torch.int32).contiguous(), w


def build_bundle(cfg: RunCfg, rank: int = 0, world_size: int = 1, device="cpu", with_bf16: bool = False,
                 with_weights: bool = True) -> DataBundle:
    s = cfg.shape
    T = s.M_aligned(world_size)
    hidden_f32 = torch.randn((T, s.K), generator=_gen(device, cfg.seed + 17), device=device, dtype=torch.float32)
    hidden_full = hidden_f32.to(torch.bfloat16)
    local = T // world_size
    hidden_local = hidden_full[rank * local:(rank + 1) * local].contiguous()
    logits = torch.randn((T, s.E), generator=_gen(device, cfg.seed + 1), device=device, dtype=torch.float32)
    ids, wts = route(logits, s.top_k, cfg.routing)
    routing = RoutingBundle(ids[rank * local:(rank + 1) * local].contiguous(),
                            wts[rank * local:(rank + 1) * local].contiguous(), ids, wts)
    ckpt = None
    if with_weights:
        w1 = expert_stack(s.E, s.n_gateup, s.K, cfg.weight_std, cfg.seed + 101, device)
        w2 = expert_stack(s.E, s.K, s.n_down, cfg.weight_std, cfg.seed + 202, device)
        sw1 = sw2 = None
        if s.shared_experts:
            sw1 = expert_stack(1, 2 * s.shared_intermediate, s.K, cfg.weight_std, cfg.seed + 303, device)
            sw2 = expert_stack(1, s.K, s.shared_intermediate, cfg.weight_std, cfg.seed + 404, device)
        if with_bf16:
            for qt in (w1, w2, sw1, sw2):
                if qt is not None:
                    qt.bf16 = dequantize_block128(qt.fp8, qt.scale)
        ckpt = WeightCheckpoint(w1, w2, sw1, sw2)
    return DataBundle(hidden_local=hidden_local, ckpt=ckpt, routing=routing, hidden_full=hidden_full)
