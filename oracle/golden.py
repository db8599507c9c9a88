"""fp32 MoE layer oracle and verification gates (test oracle).

``golden_moe`` restates ``moe_bench/verify.py:14-47``: for each expert, gather the
rows routed to it, group-128 quant-dequant them, ``gate, up = x @ w1[e].T`` split
in half, ``h = silu(gate) * up``, quant-dequant ``h``, ``y = h @ w2[e].T``, scale by
the routing weight and scatter-add into the output.  An optional dense shared
expert is added on every token (``:42-46``).  The weights are the bf16 dequantised
block-128 views (``moe_bench/data/bundle.py:59-62``).

``compare_outputs`` restates ``moe_bench/verify.py:50-105`` and ``GATES`` the
worker's defaults (``moe_bench/worker.py:108-110``).
"""
from __future__ import annotations

import numpy as np

from .fp8 import bf16_bits_to_f32
from .quant import quant_dequant_g128

GATES = {"cos_threshold": 0.995, "rel_p99_threshold": 5.0, "scale_tolerance": 0.05}


def silu(x: np.ndarray) -> np.ndarray:
    x = x.astype(np.float32)
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def _f32(w: np.ndarray) -> np.ndarray:
    """Weights may be held as bf16 bit patterns (uint16) and widened per expert, as the
    reference does with ``w1_bf16[expert].float()`` inside its loop (``verify.py:33``)."""
    return bf16_bits_to_f32(w) if w.dtype == np.uint16 else w.astype(np.float32, copy=False)


def _ffn(x: np.ndarray, w1: np.ndarray, w2: np.ndarray, act_quant: bool) -> np.ndarray:
    if act_quant:
        x = quant_dequant_g128(x)
    gu = x @ _f32(w1).T
    half = gu.shape[-1] // 2
    h = silu(gu[:, :half]) * gu[:, half:]
    if act_quant:
        h = quant_dequant_g128(h)
    return (h @ _f32(w2).T).astype(np.float32)


def golden_moe(hidden: np.ndarray, topk_ids: np.ndarray, topk_weights: np.ndarray,
               w1: np.ndarray, w2: np.ndarray,
               shared_w1: np.ndarray | None = None, shared_w2: np.ndarray | None = None,
               act_quant: bool = True) -> np.ndarray:
    """hidden [T, H]; topk_ids/weights [T, k]; w1 [E, 2I, H]; w2 [E, H, I] (fp32 values or
    bf16 bit patterns) -> [T, H] fp32."""
    hidden = np.asarray(hidden, dtype=np.float32)
    ids = np.asarray(topk_ids)
    wts = np.asarray(topk_weights, dtype=np.float32)
    out = np.zeros((hidden.shape[0], w2.shape[1]), dtype=np.float32)
    for e in range(w1.shape[0]):
        rows, slots = np.nonzero(ids == e)
        if rows.size == 0:
            continue
        y = _ffn(hidden[rows], w1[e], w2[e], act_quant)
        np.add.at(out, rows, y * wts[rows, slots][:, None])
    if shared_w1 is not None and shared_w2 is not None:
        out = out + _ffn(hidden, shared_w1[0], shared_w2[0], act_quant)
    return out


def golden_moe_threads(hidden: np.ndarray, topk_ids: np.ndarray, topk_weights: np.ndarray,
                       w1: np.ndarray, w2: np.ndarray,
                       shared_w1: np.ndarray | None = None, shared_w2: np.ndarray | None = None,
                       workers: int = 1) -> np.ndarray:
    """``golden_moe`` with the per-expert work spread over ``workers`` host threads.

    Same steps as ``golden_moe`` (the expert loop of ``moe_bench/verify.py:29-41``,
    including the per-expert widening of bf16 weights); each worker computes whole
    experts and the results are added into the output in ascending expert order, as
    the serial loop does.  numpy releases the GIL inside its array kernels and BLAS,
    so the threads run in parallel.  Used to time the reference algorithm on all host
    cores (with BLAS itself single-threaded per worker by the caller)."""
    from concurrent.futures import ThreadPoolExecutor

    hidden = np.asarray(hidden, dtype=np.float32)
    ids = np.asarray(topk_ids)
    wts = np.asarray(topk_weights, dtype=np.float32)
    experts = [e for e in range(w1.shape[0]) if np.any(ids == e)]

    def one(e: int):
        rows, slots = np.nonzero(ids == e)
        return rows, _ffn(hidden[rows], w1[e], w2[e], True) * wts[rows, slots][:, None]

    out = np.zeros((hidden.shape[0], w2.shape[1]), dtype=np.float32)
    with ThreadPoolExecutor(max_workers=max(1, workers)) as pool:
        for rows, y in pool.map(one, experts):
            np.add.at(out, rows, y)
    if shared_w1 is not None and shared_w2 is not None:
        out = out + _ffn(hidden, shared_w1[0], shared_w2[0], True)
    return out


def compare_outputs(actual: np.ndarray, expected: np.ndarray, atol: float = 0.2, rtol: float = 0.0,
                    cos_threshold: float | None = None, rel_p99_threshold: float | None = None,
                    scale_tolerance: float | None = None) -> dict:
    a = np.asarray(actual, dtype=np.float64).ravel()
    e = np.asarray(expected, dtype=np.float64).ravel()
    diff = np.abs(a - e)
    if diff.size == 0:
        return {"max_abs": 0.0, "max_rel": 0.0, "cos_sim": 1.0, "rel_p99": 0.0,
                "rel_masked_max": 0.0, "scale": 1.0, "pass": True}
    max_abs = float(diff.max())
    max_rel = float((diff / np.maximum(np.abs(e), 1e-12)).max())
    na, ne = np.linalg.norm(a), np.linalg.norm(e)
    cos = float(a @ e / max(na * ne, 1e-8 ** 2)) if na > 0 and ne > 0 else 0.0
    abs_e = np.abs(e)
    mask = abs_e > 1e-3 * abs_e.max()
    rel_p99 = rel_masked_max = 0.0
    if mask.any():
        rel = np.sort(diff[mask] / abs_e[mask])
        k = max(1, int(0.99 * rel.size))
        rel_p99 = float(rel[k - 1])
        rel_masked_max = float(rel[-1])
    denom = float(e @ e)
    scale = float(a @ e / denom) if denom > 0 else 1.0
    if cos_threshold is None and rel_p99_threshold is None and scale_tolerance is None:
        passed = bool(np.all(diff <= atol + rtol * abs_e))
    else:
        passed = True
        if cos_threshold is not None:
            passed = passed and cos >= cos_threshold
        if rel_p99_threshold is not None:
            passed = passed and rel_p99 <= rel_p99_threshold
        if scale_tolerance is not None:
            passed = passed and abs(scale - 1.0) <= scale_tolerance
    return {"max_abs": max_abs, "max_rel": max_rel, "cos_sim": cos, "rel_p99": rel_p99,
            "rel_masked_max": rel_masked_max, "scale": scale, "pass": bool(passed)}
