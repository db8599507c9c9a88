"""float8_e4m3fn encode/decode in numpy (test oracle).

The reference converts with ``tensor.to(torch.float8_e4m3fn)`` after clamping to
+-448 (``moe_bench/verify.py:116``, ``moe_bench/data/checkpoint.py:45-46``).  That
cast rounds to nearest, ties to even, with gradual underflow down to 2**-9.  This
module restates it from the format definition: 1 sign bit, 4 exponent bits (bias
7), 3 mantissa bits, no infinities, 0x7F/0xFF are NaN, max finite 448.
"""
from __future__ import annotations

import numpy as np

FP8_MAX = np.float32(448.0)


def _decode_table() -> np.ndarray:
    table = np.empty(256, dtype=np.float32)
    for code in range(256):
        sign = -1.0 if code & 0x80 else 1.0
        exp = (code >> 3) & 0xF
        man = code & 0x7
        if exp == 0xF and man == 0x7:
            table[code] = np.nan
        elif exp == 0:
            table[code] = sign * man * 2.0 ** -9
        else:
            table[code] = sign * (1.0 + man / 8.0) * 2.0 ** (exp - 7)
    return table


DECODE = _decode_table()


def encode_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 array -> uint8 e4m3fn codes, round-to-nearest-even.

    Inputs must already be finite and within [-448, 448] (the reference clamps
    before casting); larger magnitudes raise instead of silently producing NaN.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32)
    sign = ((bits >> 24) & 0x80).astype(np.uint8)
    mag_bits = bits & np.uint32(0x7FFFFFFF)
    mag = mag_bits.view(np.float32)
    if not np.all(np.isfinite(mag)) or np.any(mag > FP8_MAX):
        raise ValueError("encode_e4m3 expects finite inputs clamped to +-448")
    out = np.empty(x.shape, dtype=np.uint8)

    small = mag < np.float32(2.0 ** -6)
    # Subnormal range: code = m, value m * 2**-9 (m = 8 lands exactly on 2**-6).
    # mag * 512 is exact in fp32, np.rint rounds half to even.
    out[small] = np.rint(mag[small] * np.float32(512.0)).astype(np.uint8)

    normal = ~small
    nb = mag_bits[normal]
    # Round the 23-bit fp32 mantissa to 3 bits, ties to even, carrying into the exponent.
    lsb = (nb >> 20) & np.uint32(1)
    rounded = (nb + np.uint32(0x7FFFF) + lsb) >> 20          # (exp8 << 3) | mant3
    code = rounded.astype(np.int64) - ((127 - 7) << 3)        # rebias 127 -> 7
    if np.any(code > 0x7E):
        raise ValueError("value rounds above 448")
    out[normal] = code.astype(np.uint8)
    return out | sign


def decode_e4m3(codes: np.ndarray) -> np.ndarray:
    return DECODE[np.asarray(codes, dtype=np.uint8)]


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 (round to nearest even) -> fp32, for finite inputs."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    bits = x.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    r = ((bits + 0x7FFF + lsb) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> fp32 values."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)
