"""Weight preparation (set-up, outside the timed forward), in torch.

* ``quantize_block128`` / ``dequantize_block128``: the 128x128 block FP8 rule of
  ``moe_bench/data/checkpoint.py:28-52`` (scale = max(amax/448, 1e-12), codes
  e4m3 of clamp(w/scale)); the dequantised view is rounded to bf16.
* ``tp_views`` / ``ep_views``: the shard views of ``moe_bench/schemes/runtime.py:27-104``.
  TP rank r takes gate and up rows [r*I/P, (r+1)*I/P) and the matching columns of
  w2.  When I/P is a multiple of 128 the block codes are sliced directly; otherwise
  (Qwen3: 96 or 192) the bf16 view is sliced, zero padded to the next multiple of
  128 and re-quantised, as the reference's "L2" level does (``runtime.py:46-55``).
  EP rank r takes experts [r*E/P, (r+1)*E/P) with the global->local expert map
  (``runtime.py:162-167``).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

FP8 = torch.float8_e4m3fn
FP8_MAX = 448.0


def _ceil_to(v: int, b: int) -> int:
    return (v + b - 1) // b * b


def quantize_block128(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 [E, N, K] -> (e4m3 [E, N, K], fp32 [E, ceil(N/128), ceil(K/128)])."""
    e, n, k = w.shape
    npad, kpad = _ceil_to(n, 128), _ceil_to(k, 128)
    wp = F.pad(w.float(), (0, kpad - k, 0, npad - n))
    blocks = wp.view(e, npad // 128, 128, kpad // 128, 128)
    scale = (blocks.abs().amax(dim=(2, 4)) / FP8_MAX).clamp(min=1e-12)
    q = (blocks / scale[:, :, None, :, None]).clamp(-FP8_MAX, FP8_MAX)
    return q.view(e, npad, kpad)[:, :n, :k].to(FP8).contiguous(), scale.contiguous()


def dequantize_block128(fp8: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    e, n, k = fp8.shape
    npad, kpad = _ceil_to(n, 128), _ceil_to(k, 128)
    wp = F.pad(fp8.float(), (0, kpad - k, 0, npad - n))
    blocks = wp.view(e, npad // 128, 128, kpad // 128, 128) * scale[:, :, None, :, None].float()
    return blocks.view(e, npad, kpad)[:, :n, :k].to(torch.bfloat16).contiguous()


def tp_views(w1: torch.Tensor, w1_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor,
             rank: int, world_size: int) -> dict:
    """TP shard of full-layer block-quantised weights.  Returns fp8/scale tensors and the shard level."""
    if world_size == 1:
        return {"w1": w1, "w1_scale": w1_scale, "w2": w2, "w2_scale": w2_scale, "shard_level": "L0", "inter": w2.shape[2]}
    e, n2, h = w1.shape
    inter = n2 // 2
    if inter % world_size:
        raise ValueError(f"intermediate {inter} not divisible by world_size {world_size}")
    ir = inter // world_size
    lo, hi = rank * ir, (rank + 1) * ir
    if ir % 128 == 0:
        w1r = torch.cat([w1[:, lo:hi], w1[:, inter + lo:inter + hi]], dim=1).contiguous()
        s1r = torch.cat([w1_scale[:, lo // 128:hi // 128],
                         w1_scale[:, inter // 128 + lo // 128:inter // 128 + hi // 128]], dim=1).contiguous()
        return {"w1": w1r, "w1_scale": s1r, "w2": w2[:, :, lo:hi].contiguous(),
                "w2_scale": w2_scale[:, :, lo // 128:hi // 128].contiguous(), "shard_level": "L0", "inter": ir}
    # L2: slice the bf16 view, zero pad to a multiple of 128, re-quantise.
    irp = _ceil_to(ir, 128)
    w1b = dequantize_block128(w1, w1_scale)
    w2b = dequantize_block128(w2, w2_scale)
    gate = F.pad(w1b[:, lo:hi].float(), (0, 0, 0, irp - ir))
    up = F.pad(w1b[:, inter + lo:inter + hi].float(), (0, 0, 0, irp - ir))
    w1q, s1q = quantize_block128(torch.cat([gate, up], dim=1))
    w2q, s2q = quantize_block128(F.pad(w2b[:, :, lo:hi].float(), (0, irp - ir)))
    return {"w1": w1q, "w1_scale": s1q, "w2": w2q, "w2_scale": s2q, "shard_level": "L2", "inter": irp}


def contiguous_placement(num_experts: int, world_size: int) -> list[list[int]]:
    """The reference's expert-parallel layout: rank r owns experts [r*E/P, (r+1)*E/P)
    (``moe_bench/schemes/runtime.py:86-93``)."""
    le = num_experts // world_size
    return [list(range(r * le, (r + 1) * le)) for r in range(world_size)]


def balanced_placement(topk_ids: torch.Tensor, num_experts: int, world_size: int) -> list[list[int]]:
    """Experts per rank balanced by routed (token, expert) pairs, E/P experts on every rank.

    Greedy longest-first: experts in descending pair count (ties: lower id first) each go
    to the rank with the fewest pairs so far among those with room (ties: lower rank).
    Expert placement does not enter the layer's math -- the output is the same sum over
    the same experts -- only which rank computes which expert, so under skewed routing
    (Zipf) it removes the load imbalance the contiguous layout has (DeepSeek-V3 EP8 at
    Zipf 1.2: the most-loaded rank holds 2.24x the mean pairs contiguous, 1.0x balanced).
    Returns each rank's experts in ascending id order."""
    if num_experts % world_size:
        raise ValueError(f"E={num_experts} not divisible by world_size {world_size}")
    cap = num_experts // world_size
    counts = torch.bincount(topk_ids.reshape(-1).long().cpu(), minlength=num_experts)[:num_experts].tolist()
    order = sorted(range(num_experts), key=lambda e: (-counts[e], e))
    load = [0] * world_size
    owned: list[list[int]] = [[] for _ in range(world_size)]
    for e in order:
        r = min((r for r in range(world_size) if len(owned[r]) < cap), key=lambda r: (load[r], r))
        owned[r].append(e)
        load[r] += counts[e]
    return [sorted(x) for x in owned]


def expert_owner(placement: list[list[int]], device=None) -> torch.Tensor:
    """int32 [E]: the rank that holds each global expert."""
    n = sum(len(x) for x in placement)
    owner = torch.empty(n, dtype=torch.int32)
    for r, es in enumerate(placement):
        owner[es] = r
    return owner.to(device) if device is not None else owner


def ep_views(w1: torch.Tensor, w1_scale: torch.Tensor, w2: torch.Tensor, w2_scale: torch.Tensor,
             rank: int, world_size: int, placement: list[list[int]] | None = None) -> dict:
    """Expert-parallel shard: this rank's experts (contiguous layout unless ``placement`` gives
    every rank's expert list) and the global -> local expert map (-1: not local)."""
    e = w1.shape[0]
    if e % world_size:
        raise ValueError(f"E={e} not divisible by world_size {world_size}")
    if placement is None:
        placement = contiguous_placement(e, world_size)
    mine = placement[rank]
    emap = torch.full((e,), -1, dtype=torch.int32, device=w1.device)
    emap[mine] = torch.arange(len(mine), dtype=torch.int32, device=w1.device)
    lo = mine[0]
    if mine == list(range(lo, lo + len(mine))):   # a contiguous range: slice
        sel = slice(lo, lo + len(mine))
        views = [t[sel].contiguous() for t in (w1, w1_scale, w2, w2_scale)]
    else:
        idx = torch.tensor(mine, dtype=torch.long, device=w1.device)
        views = [t.index_select(0, idx).contiguous() for t in (w1, w1_scale, w2, w2_scale)]
    return {"w1": views[0], "w1_scale": views[1], "w2": views[2], "w2_scale": views[3],
            "expert_map": emap if world_size > 1 else None, "expert_owner": expert_owner(placement, w1.device),
            "shard_level": "L0", "inter": w2.shape[2]}
