"""Output verification of the layer: the reference worker's fp32 golden and gates, on the device.

The reference verifies every scheme after timing (``moe_bench/worker.py:108-146``):
it computes ``golden_moe`` (``moe_bench/verify.py:14-47``) in fp32, slices the rank's
rows and applies three gates -- cosine >= 0.995, masked relative p99 <= 5.0 and
|least-squares scale - 1| <= 0.05 (``verify.py:50-105``).  This module is that step in
torch on the GPU, for shapes where a host restatement would take minutes:

* ``golden_rows`` -- the fp32 golden of a token slice: per expert, the routed rows
  group-128 quant-dequantised (``verify.py:108-117``), ``gate, up = x @ w1[e].T``,
  ``h = silu(gate) * up``, quant-dequant ``h``, ``y = h @ w2[e].T``, times the routing
  weight, summed into the output; plus the dense shared expert.  Weights are the
  block-128 dequantised values rounded to bf16 (``moe_bench/data/bundle.py:59-62``).
  ``act_quant=False`` drops the two activation QDQ steps: the difference of the two is
  the calibration measure of ``tests/calibrate_tolerance.py:17-25``.
* ``compare_outputs`` -- the gate metrics.
* ``check_layer`` -- the gates plus max-abs <= 1.5 x calibration (the calibration
  script's tight-atol rule), as one report;
* ``rank_partials`` / ``rs_fp8_error`` -- the golden split into each rank's partial sum
  (its experts under EP, its intermediate slice under TP) and the extra error of the FP8
  reduce-scatter payload (``overlap_forward.py:900-946``): max |sum_r p_r - sum_r QDQ(bf16(p_r))|,
  the calibration term added to the bound when the partials cross as FP8.

It is a checker: nothing on the layer's forward path calls it.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.nn.functional as F

GATES = {"cos_threshold": 0.995, "rel_p99_threshold": 5.0, "scale_tolerance": 0.05}
MAX_ABS_FACTOR = 1.5


def qdq128(x: torch.Tensor) -> torch.Tensor:
    """Group-128 FP8 e4m3 quant-dequant per row: scale = max(amax / 448, 1e-12)."""
    r, c = x.shape
    cp = (c + 127) // 128 * 128
    g = F.pad(x.float(), (0, cp - c)).view(r, cp // 128, 128)
    s = (g.abs().amax(-1, keepdim=True) / 448.0).clamp(min=1e-12)
    q = (g / s).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).float() * s
    return q.view(r, cp)[:, :c]


def dequant_bf16(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """[N, K] e4m3 codes x [N/128, K/128] block scales -> fp32 values rounded to bf16."""
    n, k = q.shape
    w = q.float().view(n // 128, 128, k // 128, 128) * s.float()[:, None, :, None]
    return w.view(n, k).to(torch.bfloat16).float()


def _ffn(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, act_quant: bool) -> torch.Tensor:
    if act_quant:
        x = qdq128(x)
    gu = x @ w1.T
    i = gu.shape[1] // 2
    h = F.silu(gu[:, :i]) * gu[:, i:]
    if act_quant:
        h = qdq128(h)
    return h @ w2.T


@torch.no_grad()
def golden_rows(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, ckpt: Any,
                act_quant: bool = True) -> torch.Tensor:
    """fp32 golden [rows, H] of the given token rows (hidden [rows, H], routing [rows, k]).

    ``ckpt`` holds the full checkpoint: ``w1/w2`` (and optionally ``shared_w1/shared_w2``)
    with ``.fp8`` codes [E, N, K] and ``.scale`` block scales."""
    x = hidden.float()
    out = torch.zeros((x.shape[0], ckpt.w2.fp8.shape[1]), dtype=torch.float32, device=x.device)
    ids = topk_ids.long()
    for e in torch.unique(ids).tolist():
        rows, slots = torch.nonzero(ids == e, as_tuple=True)
        w1 = dequant_bf16(ckpt.w1.fp8[e].to(x.device), ckpt.w1.scale[e].to(x.device))
        w2 = dequant_bf16(ckpt.w2.fp8[e].to(x.device), ckpt.w2.scale[e].to(x.device))
        y = _ffn(x[rows], w1, w2, act_quant)
        out.index_add_(0, rows, y * topk_weights[rows, slots].float()[:, None])
    if getattr(ckpt, "shared_w1", None) is not None and getattr(ckpt, "shared_w2", None) is not None:
        sw1 = dequant_bf16(ckpt.shared_w1.fp8[0].to(x.device), ckpt.shared_w1.scale[0].to(x.device))
        sw2 = dequant_bf16(ckpt.shared_w2.fp8[0].to(x.device), ckpt.shared_w2.scale[0].to(x.device))
        out += _ffn(x, sw1, sw2, act_quant)
    return out


@torch.no_grad()
def rank_partials(hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, ckpt: Any, world: int,
                  parallel: str, owner: list[int] | None = None) -> torch.Tensor:
    """fp32 [world, rows, H]: rank r's share of the golden of these rows before the reduce-scatter.

    EP: the routed pairs of the experts rank r holds (``owner[e]``, default the contiguous layout
    [r*E/world, (r+1)*E/world)); the shared expert is added after the reduce-scatter and is not
    part of any partial.  TP: every routed pair restricted to
    intermediate columns [r*I/world, (r+1)*I/world) (and the same slice of the shared expert);
    needs I/world to be a multiple of 128 so the slices align with the quantisation groups."""
    x = hidden.float()
    E, H, I = ckpt.w1.fp8.shape[0], ckpt.w2.fp8.shape[1], ckpt.w2.fp8.shape[2]
    out = torch.zeros((world, x.shape[0], H), dtype=torch.float32, device=x.device)
    ids = topk_ids.long()

    def tp_split(xr: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, scale: torch.Tensor | None, rows):
        inter = w2.shape[1]
        if inter % world or (inter // world) % 128:
            raise ValueError(f"TP slices of I={inter} over {world} ranks are not 128-aligned")
        gu = qdq128(xr) @ w1.T
        h = qdq128(F.silu(gu[:, :inter]) * gu[:, inter:])
        for r in range(world):
            sl = slice(r * inter // world, (r + 1) * inter // world)
            y = h[:, sl] @ w2[:, sl].T
            out[r].index_add_(0, rows, y if scale is None else y * scale)

    for e in torch.unique(ids).tolist():
        rows, slots = torch.nonzero(ids == e, as_tuple=True)
        w1 = dequant_bf16(ckpt.w1.fp8[e].to(x.device), ckpt.w1.scale[e].to(x.device))
        w2 = dequant_bf16(ckpt.w2.fp8[e].to(x.device), ckpt.w2.scale[e].to(x.device))
        wt = topk_weights[rows, slots].float()[:, None]
        if parallel == "EP":
            r = owner[e] if owner is not None else e // (E // world)
            out[r].index_add_(0, rows, _ffn(x[rows], w1, w2, True) * wt)
        else:
            tp_split(x[rows], w1, w2, wt, rows)
    if parallel != "EP" and getattr(ckpt, "shared_w1", None) is not None:
        sw1 = dequant_bf16(ckpt.shared_w1.fp8[0].to(x.device), ckpt.shared_w1.scale[0].to(x.device))
        sw2 = dequant_bf16(ckpt.shared_w2.fp8[0].to(x.device), ckpt.shared_w2.scale[0].to(x.device))
        tp_split(x, sw1, sw2, None, torch.arange(x.shape[0], device=x.device))
    return out


@torch.no_grad()
def rs_fp8_error(partials: torch.Tensor) -> float:
    """max |sum_r p_r - sum_r QDQ128(bf16(p_r))| over the rows: the error the FP8 payload adds."""
    exact = partials.sum(0)
    q = torch.stack([qdq128(p.to(torch.bfloat16).float()) for p in partials]).sum(0)
    return float((exact - q).abs().max())


@torch.no_grad()
def compare_outputs(actual: torch.Tensor, expected: torch.Tensor, cos_threshold: float = 0.995,
                    rel_p99_threshold: float = 5.0, scale_tolerance: float = 0.05) -> dict:
    """Gate metrics of ``moe_bench/verify.py:50-105`` (float64 on the device)."""
    a = actual.double().reshape(-1)
    e = expected.double().reshape(-1)
    diff = (a - e).abs()
    if diff.numel() == 0:
        return {"max_abs": 0.0, "cos_sim": 1.0, "rel_p99": 0.0, "scale": 1.0, "pass": True}
    na, ne = torch.linalg.vector_norm(a), torch.linalg.vector_norm(e)
    cos = float(a @ e / (na * ne)) if float(na) > 0 and float(ne) > 0 else 0.0
    abs_e = e.abs()
    mask = abs_e > 1e-3 * abs_e.max()
    rel_p99 = 0.0
    if bool(mask.any()):
        rel = torch.sort(diff[mask] / abs_e[mask]).values
        k = max(1, int(0.99 * rel.numel()))
        rel_p99 = float(rel[k - 1])
    denom = float(e @ e)
    scale = float(a @ e) / denom if denom > 0 else 1.0
    passed = cos >= cos_threshold and rel_p99 <= rel_p99_threshold and abs(scale - 1.0) <= scale_tolerance
    return {"max_abs": float(diff.max()), "cos_sim": cos, "rel_p99": rel_p99, "scale": scale, "pass": bool(passed)}


@torch.no_grad()
def check_layer(out: torch.Tensor, hidden: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
                ckpt: Any, extra_calib: float = 0.0) -> dict:
    """Layer output rows vs the fp32 golden of the same tokens: the worker's gates plus
    max-abs <= 1.5 x (the activation-quantisation error calibrated on these rows +
    ``extra_calib``, e.g. ``rs_fp8_error`` when the partials crossed as FP8)."""
    g = golden_rows(hidden, topk_ids, topk_weights, ckpt, act_quant=True)
    g_plain = golden_rows(hidden, topk_ids, topk_weights, ckpt, act_quant=False)
    calib = float((g - g_plain).abs().max()) + extra_calib
    rep = compare_outputs(out.float(), g, **GATES)
    rep["calib"] = calib
    rep["max_abs_bound"] = MAX_ABS_FACTOR * calib
    rep["gates_pass"] = rep["pass"]
    rep["pass"] = bool(rep["pass"] and rep["max_abs"] <= rep["max_abs_bound"])
    return rep
