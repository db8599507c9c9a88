"""Top-k combine and the FP8 reduce-scatter of the b3 path (test oracle).

Restates, in numpy:

* the per-token combine of ``moe_bench/overlap/overlap_forward.py:581-597``: a token's
  top-k down-projection rows summed (fp32, ascending j), plus the shared expert's row,
  rounded once to bf16 -- the reduce-scatter input;
* the b3 FP8 reduce-scatter (``overlap_forward.py:900-946``): each source rank's bf16
  partial rows quantised per 128 columns by the activation rule (``quant.quant_g128``,
  ``moe_bench/verify.py:108-117``), exchanged as codes + fp32 scales, and on the owner
  dequantised (``e4m3 * scale`` in fp32) and summed over the sources in rank order, plus an
  optional bf16 row (the expert-parallel shared expert), rounded once to bf16.
"""
from __future__ import annotations

import numpy as np

from .fp8 import bf16_bits_to_f32, decode_e4m3, f32_to_bf16_bits
from .quant import quant_g128


def combine_rows(staged: np.ndarray, top_k: int, shared: np.ndarray | None = None,
                 mask: np.ndarray | None = None) -> np.ndarray:
    """staged fp32 [T*k, H] (bf16 values) -> bf16 bit patterns [T, H]; mask [T, k] bool selects pairs."""
    t = staged.shape[0] // top_k
    s3 = np.asarray(staged, dtype=np.float32).reshape(t, top_k, -1)
    acc = np.zeros((t, s3.shape[2]), np.float32)
    for j in range(top_k):
        row = s3[:, j] if mask is None else np.where(mask[:, j:j + 1], s3[:, j], np.float32(0))
        acc = (acc + row).astype(np.float32)
    if shared is not None:
        acc = (acc + np.asarray(shared, dtype=np.float32)).astype(np.float32)
    return f32_to_bf16_bits(acc)


def rs_fp8_push(partial_bits: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """bf16 bit patterns [rows, H] -> (e4m3 codes [rows, H], fp32 scales [rows, H/128])."""
    return quant_g128(bf16_bits_to_f32(partial_bits))


def rs_fp8_reduce(codes: np.ndarray, scales: np.ndarray, add_bits: np.ndarray | None = None) -> np.ndarray:
    """codes [P, rows, H], scales [P, rows, H/128] (+ bf16 bits [rows, H]) -> bf16 bits [rows, H]."""
    p, rows, h = codes.shape
    acc = np.zeros((rows, h), np.float32)
    for r in range(p):
        deq = (decode_e4m3(codes[r]) * np.repeat(scales[r], 128, axis=-1)[:, :h]).astype(np.float32)
        acc = (acc + deq).astype(np.float32)
    if add_bits is not None:
        acc = (acc + bf16_bits_to_f32(add_bits)).astype(np.float32)
    return f32_to_bf16_bits(acc)
