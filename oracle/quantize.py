"""bf16 -> e4m3 quantisation, restated in numpy.  Test infrastructure only.

Follows kernels/triton_kernels/fp8_flash_attn_hopper.py:
  * ``_per_bh_scale`` (:374-385): amax |x| over (S, D) of each (b,h) in bf16,
    clamp(min=1e-6) in bf16, divided by 0.95 * 448 with the quotient rounded
    to bf16, widened to fp32 -> dequant scale;
  * ``_quantize`` (:388-398): x (fp32) * (1 / scale) -> clamp(+-448) -> e4m3fn.

Inputs are bf16 bit patterns (uint16 arrays shaped (B, H, S, D)), or fp16
bit patterns with ``fmt="f16"``: the reference's functions run the same steps
in the input's dtype, so for fp16 the amax, its clamp (fp16(1e-6) is the
subnormal 0x0011) and the rounded scale are fp16.  The per-128-token-block
mode (no reference code; an extension of the same formula) computes one
scale per block of 128 tokens of each (b,h); the last block of a ragged S is
short.
"""

from __future__ import annotations

import numpy as np

from .fp8 import bf16_bits_to_f32, e4m3_encode, round_to_bf16

BLOCK = 128
AMAX_FLOOR_BITS = 0x3586  # bf16 nearest to 1e-6 (clamp(min=1e-6) on a bf16 tensor)
SCALE_DIV = np.float32(0.95 * 448)  # float(0.95 * 448) == 425.6f

# per input format: (amax floor bits, +inf bits, bits -> f32, f32 -> rounded f32)
_FORMATS = {
    "bf16": (AMAX_FLOOR_BITS, 0x7F80, bf16_bits_to_f32, round_to_bf16),
    "f16": (
        0x0011,  # fp16 nearest to 1e-6
        0x7C00,
        lambda b: np.asarray(b, dtype=np.uint16).view(np.float16).astype(np.float32),
        lambda x: np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32),
    ),
}

SCALE_PER_BH = 0
SCALE_PER_BLOCK128 = 1


def absmax_bits(x_bits: np.ndarray, axis) -> np.ndarray:  # type: ignore[no-untyped-def]
    """max |x| as bf16 bits; NaN (bits > 0x7F80) wins like torch.amax."""
    return (np.asarray(x_bits, dtype=np.uint16) & 0x7FFF).max(axis=axis)


def scale_from_amax_bits(amax_bits: np.ndarray, fmt: str = "bf16") -> np.ndarray:
    floor, inf, decode, rnd = _FORMATS[fmt]
    b = np.asarray(amax_bits, dtype=np.uint16)
    b = np.where((b <= inf) & (b < floor), np.uint16(floor), b)
    a = decode(b)
    with np.errstate(invalid="ignore", over="ignore"):
        s = a / SCALE_DIV
    return rnd(s).astype(np.float32)


def per_bh_scale(x_bits: np.ndarray, fmt: str = "bf16") -> np.ndarray:
    """(B,H,S,D) 16-bit float bits -> (B*H,) fp32 dequant scales."""
    B, H, S, D = x_bits.shape
    return scale_from_amax_bits(absmax_bits(x_bits.reshape(B * H, S * D), axis=1), fmt)


def per_block_scale(x_bits: np.ndarray, fmt: str = "bf16") -> np.ndarray:
    """(B,H,S,D) 16-bit float bits -> (B*H, ceil(S/128)) fp32 dequant scales."""
    B, H, S, D = x_bits.shape
    nblk = (S + BLOCK - 1) // BLOCK
    flat = x_bits.reshape(B * H, S, D)
    out = np.empty((B * H, nblk), dtype=np.float32)
    for i in range(nblk):
        seg = flat[:, i * BLOCK : (i + 1) * BLOCK, :].reshape(B * H, -1)
        out[:, i] = scale_from_amax_bits(absmax_bits(seg, axis=1), fmt)
    return out


def expand_scales(scales: np.ndarray, S: int) -> np.ndarray:
    """(B*H,) or (B*H, nblk) -> per-row (B*H, S) scales."""
    scales = np.asarray(scales, dtype=np.float32)
    if scales.ndim == 1:
        return np.repeat(scales[:, None], S, axis=1)
    return np.repeat(scales, BLOCK, axis=1)[:, :S]


def quantize(x_bits: np.ndarray, scales: np.ndarray, fmt: str = "bf16") -> np.ndarray:
    """(B,H,S,D) 16-bit float bits + scales -> (B,H,S,D) e4m3 bytes."""
    B, H, S, D = x_bits.shape
    x = _FORMATS[fmt][2](x_bits).reshape(B * H, S, D)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        q_mul = np.float32(1.0) / expand_scales(scales, S)
        y = x * q_mul[:, :, None]
    y = np.where(y > 448.0, np.float32(448.0), y)
    y = np.where(y < -448.0, np.float32(-448.0), y).astype(np.float32)
    return e4m3_encode(y).reshape(B, H, S, D)


def quantize_with_scales(
    x_bits: np.ndarray, scale_mode: int, fmt: str = "bf16"
) -> tuple[np.ndarray, np.ndarray]:
    if scale_mode == SCALE_PER_BH:
        s = per_bh_scale(x_bits, fmt)
    elif scale_mode == SCALE_PER_BLOCK128:
        s = per_block_scale(x_bits, fmt)
    else:
        raise ValueError(f"unknown scale mode {scale_mode}")
    return quantize(x_bits, s, fmt), s
