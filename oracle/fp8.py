"""e4m3fn and bf16 bit-level helpers (numpy).  Test infrastructure only.

The e4m3fn encoder restates the round-to-nearest-even conversion PyTorch
applies in ``tensor.to(torch.float8_e4m3fn)`` (called by the reference at
kernels/triton_kernels/fp8_flash_attn_hopper.py:398): sign kept, |x| >= 480
(the first value that rounds past 448) and NaN map to 0x7F | sign, values
below 2^-6 round to a multiple of 2^-9 (subnormals), normal values round
their 23-bit mantissa to 3 bits, ties to even.
"""

from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
_F32_480_BITS = 1087 << 20          # bit pattern of 480.0f
_F32_MIN_NORMAL_E4M3 = 121 << 23    # bit pattern of 2^-6


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 to bf16 (nearest, ties to even); NaN -> 0x7FC0."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, np.uint16(0x7FC0), rounded)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def e4m3_encode(y: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn bytes (see module docstring)."""
    y = np.ascontiguousarray(y, dtype=np.float32)
    u = y.view(np.uint32)
    sign = ((u >> 24) & 0x80).astype(np.uint8)
    a = (u & 0x7FFFFFFF).astype(np.int64)
    out = np.zeros(y.shape, dtype=np.uint8)

    big = a >= _F32_480_BITS  # includes inf and NaN
    small = (a < _F32_MIN_NORMAL_E4M3) & ~big
    normal = ~big & ~small

    out[big] = 0x7F
    mag = np.abs(y[small]).astype(np.float64)
    out[small] = np.rint(mag * 512.0).astype(np.uint8)  # multiples of 2^-9, ties even
    an = a[normal]
    mant_odd = (an >> 20) & 1
    an = an + ((7 - 127) << 23) + 0x7FFFF + mant_odd
    out[normal] = (an >> 20).astype(np.uint8)
    return out | sign


def _decode_table() -> np.ndarray:
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * m * 2.0**-9
        else:
            t[b] = s * (1 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_TABLE = _decode_table()


def e4m3_decode(b: np.ndarray) -> np.ndarray:
    return E4M3_TABLE[np.asarray(b, dtype=np.uint8)]
