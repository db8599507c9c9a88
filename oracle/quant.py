"""Group-128 activation quant and 128x128 weight block quant (test oracle).

Restates, in numpy:

* ``moe_bench/verify.py:108-117`` (``_group_quant_dequant``): per row and per
  128-column group, ``scale = clamp(amax / 448, min=1e-12)`` (IEEE fp32 division),
  ``q = e4m3(clamp(x / scale, -448, 448))``; the dequantised value is
  ``float(q) * scale``.  Ragged tails are zero padded before the amax.
* ``moe_bench/data/checkpoint.py:28-52`` (``quantize_block128`` /
  ``dequantize_block128``): the same rule over 128x128 blocks of ``[E, N, K]``
  weights; the dequantised view is rounded to bf16.
"""
from __future__ import annotations

import numpy as np

from .fp8 import FP8_MAX, bf16_round, decode_e4m3, encode_e4m3

SCALE_MIN = np.float32(1e-12)


def _ceil_to(v: int, b: int) -> int:
    return (v + b - 1) // b * b


def quant_g128(x: np.ndarray, block: int = 128) -> tuple[np.ndarray, np.ndarray]:
    """[..., C] fp32/bf16-valued array -> (uint8 codes [..., C], fp32 scales [..., ceil(C/128)])."""
    x = np.asarray(x, dtype=np.float32)
    cols = x.shape[-1]
    cpad = _ceil_to(cols, block)
    pad = np.zeros(x.shape[:-1] + (cpad,), dtype=np.float32)
    pad[..., :cols] = x
    blocks = pad.reshape(x.shape[:-1] + (cpad // block, block))
    amax = np.abs(blocks).max(axis=-1)
    scale = np.maximum(amax / FP8_MAX, SCALE_MIN).astype(np.float32)
    q = np.clip(blocks / scale[..., None], -FP8_MAX, FP8_MAX).astype(np.float32)
    codes = encode_e4m3(q).reshape(x.shape[:-1] + (cpad,))[..., :cols]
    return np.ascontiguousarray(codes), scale


def dequant_g128(codes: np.ndarray, scale: np.ndarray, block: int = 128) -> np.ndarray:
    cols = codes.shape[-1]
    vals = decode_e4m3(codes)
    s = np.repeat(scale, block, axis=-1)[..., :cols]
    return (vals * s).astype(np.float32)


def quant_dequant_g128(x: np.ndarray) -> np.ndarray:
    """``_group_quant_dequant(x, 128)`` (``moe_bench/verify.py:108-117``)."""
    q, s = quant_g128(x)
    return dequant_g128(q, s)


def quant_block128(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """``quantize_block128`` (``moe_bench/data/checkpoint.py:28-40``): [E, N, K] -> codes, scales [E, N/128, K/128]."""
    w = np.asarray(w, dtype=np.float32)
    e, n, k = w.shape
    npad, kpad = _ceil_to(n, 128), _ceil_to(k, 128)
    pad = np.zeros((e, npad, kpad), dtype=np.float32)
    pad[:, :n, :k] = w
    blocks = pad.reshape(e, npad // 128, 128, kpad // 128, 128)
    amax = np.abs(blocks).max(axis=(2, 4))
    scale = np.maximum(amax / FP8_MAX, SCALE_MIN).astype(np.float32)
    q = np.clip(blocks / scale[:, :, None, :, None], -FP8_MAX, FP8_MAX).astype(np.float32)
    codes = encode_e4m3(q.reshape(e, npad, kpad))[:, :n, :k]
    return np.ascontiguousarray(codes), scale


def dequant_block128(codes: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """``dequantize_block128`` (``moe_bench/data/checkpoint.py:43-52``): fp32 product rounded to bf16 (as fp32)."""
    e, n, k = codes.shape
    s = np.repeat(np.repeat(scale, 128, axis=1), 128, axis=2)[:, :n, :k]
    return bf16_round(decode_e4m3(codes) * s)
