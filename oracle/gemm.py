"""FP8 GEMM and FP8 linear, restated in numpy.  Test infrastructure only.

Follows the reference's proof-of-life FP8 GEMM,
kernels/hip/fp8_attn/fp8_gemm.hip:
  * ``fp8_gemm_kernel`` (:79-156): acc = sum_k A[m, k] * B[k, n] in fp32 over
    e4m3 operands, A (M, K) and B (K, N) row-major;
  * the write-back (:145-153): scale = a_scale * b_scale (fp32), then
    C[m, n] = bf16(acc * scale), round to nearest even.
The reference's operands are gfx942 e4m3fnuz; B200 computes in OCP e4m3fn,
so the bytes here decode as e4m3fn.

Accumulation is in float64 and rounded once to fp32.  For the reference's
own known-answer cases (tests/test_mfma_fragment_layout.py:262-318: all-ones
operands, small integers in [-2, 2]) every partial sum is an integer below
2^24, so any accumulation order gives the same fp32 value and the bf16
output is exact.  Otherwise a kernel's fp32 sum may differ from this one in
the last bits, and tests compare with a tolerance.

The per-channel form (no reference kernel; the FP8 DiT linears the reference
plans for its GEMM, docs/OPTIMIZATION.md:161-162) applies the same steps with
per-row activation scales sa[m] and per-column weight scales sb[n]:
C = out(acc * (sa[m] * sb[n]) + bias[n]).  Its operands come from the
row-wise quantizer: each row of an (rows, cols) matrix is one scale group of
the reference's attention quantizer (fp8_flash_attn_hopper.py:374-398).
"""

from __future__ import annotations

import numpy as np

from . import quantize as oq
from .fp8 import bf16_bits_to_f32, e4m3_decode, f32_to_bf16_bits


def _f16_bits(y: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return np.asarray(y, dtype=np.float32).astype(np.float16).view(np.uint16)


def _out_bits(y: np.ndarray, out_fmt: str) -> np.ndarray:
    if out_fmt == "bf16":
        return f32_to_bf16_bits(np.asarray(y, dtype=np.float32))
    if out_fmt == "f16":
        return _f16_bits(y)
    raise ValueError(f"unknown output format {out_fmt!r}")


def _bits_to_f32(bits: np.ndarray, fmt: str) -> np.ndarray:
    if fmt == "bf16":
        return bf16_bits_to_f32(bits)
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def accumulate(a8: np.ndarray, b8: np.ndarray, b_layout: str = "kn") -> np.ndarray:
    """fp32 acc[m, n] = sum_k A[m, k] * B(k, n) of e4m3 byte matrices.

    ``b_layout`` "kn": B is (K, N) (the reference's layout); "nk": (N, K)."""
    a = e4m3_decode(np.asarray(a8, dtype=np.uint8)).astype(np.float64)
    b = e4m3_decode(np.asarray(b8, dtype=np.uint8)).astype(np.float64)
    if b_layout == "nk":
        b = b.T
    elif b_layout != "kn":
        raise ValueError(f"unknown b_layout {b_layout!r}")
    return (a @ b).astype(np.float32)


def fp8_gemm(a8: np.ndarray, b8: np.ndarray, a_scale: float, b_scale: float) -> np.ndarray:
    """bf16 bits of C = bf16(acc * (a_scale * b_scale)) (fp8_gemm.hip:145-153)."""
    acc = accumulate(a8, b8, "kn")
    scale = np.float32(a_scale) * np.float32(b_scale)
    return f32_to_bf16_bits((acc * scale).astype(np.float32))


def gemm_ex(
    a8: np.ndarray,
    b8: np.ndarray,
    sa: np.ndarray | float,
    sb: np.ndarray | float,
    bias_bits: np.ndarray | None = None,
    out_fmt: str = "bf16",
    b_layout: str = "nk",
) -> np.ndarray:
    """Output bits of C = out(acc * (sa[m] * sb[n]) + bias[n]).

    ``sa`` / ``sb``: per-row / per-column fp32 scales, or scalars.
    ``bias_bits``: (N,) bits in the output format, or None."""
    acc = accumulate(a8, b8, b_layout)
    M, N = acc.shape
    sa_v = np.broadcast_to(np.asarray(sa, dtype=np.float32).reshape(-1, 1), (M, 1))
    sb_v = np.broadcast_to(np.asarray(sb, dtype=np.float32).reshape(1, -1), (1, N))
    with np.errstate(over="ignore", invalid="ignore"):
        y = (acc * (sa_v * sb_v).astype(np.float32)).astype(np.float32)
        if bias_bits is not None:
            y = (y + _bits_to_f32(np.asarray(bias_bits), out_fmt)[None, :]).astype(np.float32)
    return _out_bits(y, out_fmt)


def quantize_rows(x_bits: np.ndarray, fmt: str = "bf16") -> tuple[np.ndarray, np.ndarray]:
    """(rows, cols) 16-bit float bits -> e4m3 bytes (rows, cols), scales (rows,).

    One scale group per row, the attention quantizer's per-(b,h) steps."""
    rows, cols = x_bits.shape
    x4 = np.asarray(x_bits, dtype=np.uint16).reshape(1, rows, 1, cols)
    s = oq.per_bh_scale(x4, fmt)
    return oq.quantize(x4, s, fmt).reshape(rows, cols), s


def linear(
    x_bits: np.ndarray,
    w_bits: np.ndarray,
    bias_bits: np.ndarray | None = None,
    fmt: str = "bf16",
) -> np.ndarray:
    """FP8 linear y = x W^T + b: x (M, K) and W (N, K) quantized per row, one
    GEMM with both scales and the bias in its epilogue; output bits in fmt."""
    x8, xs = quantize_rows(x_bits, fmt)
    w8, ws = quantize_rows(w_bits, fmt)
    return gemm_ex(x8, w8, xs, ws, bias_bits, fmt, "nk")


def dequant_matmul(
    a8: np.ndarray, b8: np.ndarray, sa, sb, b_layout: str = "nk"  # type: ignore[no-untyped-def]
) -> np.ndarray:
    """float64 (A * sa) @ (B * sb): the exact product the kernel rounds."""
    a = e4m3_decode(np.asarray(a8, dtype=np.uint8)).astype(np.float64)
    b = e4m3_decode(np.asarray(b8, dtype=np.uint8)).astype(np.float64)
    if b_layout == "nk":
        b = b.T
    M, N = a.shape[0], b.shape[1]
    sa_v = np.broadcast_to(np.asarray(sa, dtype=np.float64).reshape(-1, 1), (M, 1))
    sb_v = np.broadcast_to(np.asarray(sb, dtype=np.float64).reshape(1, -1), (1, N))
    return (a @ b) * sa_v * sb_v
