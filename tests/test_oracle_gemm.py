"""The FP8 GEMM / linear oracle, pinned to the reference's known answers.

The reference's GEMM tests (tests/test_mfma_fragment_layout.py:262-318) hold
two known-answer cases: all-ones operands give C == K everywhere, and small
integers in [-2, 2] give the bf16 rounding of the exact integer product.  The
row-wise quantizer is pinned through the attention quantizer, whose steps it
reuses one row at a time (that quantizer is pinned bit for bit to the
reference's fixtures in tests/golden/).
"""

from __future__ import annotations

import numpy as np

from helpers import bits, gen_bf16
from oracle import gemm as og
from oracle import quantize as oq
from oracle.fp8 import bf16_bits_to_f32, e4m3_decode, e4m3_encode, f32_to_bf16_bits

E4M3_ONE = 0x38  # 1.0 in e4m3fn


def _ints(rng: np.random.Generator, shape: tuple[int, int]) -> tuple[np.ndarray, np.ndarray]:
    v = rng.integers(-2, 3, size=shape).astype(np.float32)
    return v, e4m3_encode(v)


def test_all_ones_sums_to_k():
    for M, N, K in ((16, 16, 32), (3, 5, 4096)):
        a = np.full((M, K), E4M3_ONE, np.uint8)
        b = np.full((K, N), E4M3_ONE, np.uint8)
        c = og.fp8_gemm(a, b, 1.0, 1.0)
        assert (bf16_bits_to_f32(c) == float(K)).all()


def test_small_integers_are_exact():
    rng = np.random.default_rng(0)
    for M, N, K in ((32, 32, 64), (37, 300, 1000)):
        ai, a8 = _ints(rng, (M, K))
        bi, b8 = _ints(rng, (K, N))
        assert (e4m3_decode(a8) == ai).all() and (e4m3_decode(b8) == bi).all()
        ref = f32_to_bf16_bits((ai.astype(np.float64) @ bi).astype(np.float32))
        assert (og.fp8_gemm(a8, b8, 1.0, 1.0) == ref).all()


def test_scale_product_is_formed_before_the_accumulator_multiply():
    # C = bf16(acc * fl(a_scale * b_scale)), the reference's write-back order
    a = np.full((1, 32), E4M3_ONE, np.uint8)
    b = np.full((32, 1), E4M3_ONE, np.uint8)
    sa, sb = np.float32(0.1), np.float32(3.3)
    want = f32_to_bf16_bits(np.float32(32.0) * (sa * sb))
    assert og.fp8_gemm(a, b, float(sa), float(sb))[0, 0] == want


def test_layouts_agree():
    rng = np.random.default_rng(1)
    a8 = rng.integers(0, 256, size=(20, 48), dtype=np.uint8) & 0xF7  # no NaN bytes
    b8 = rng.integers(0, 256, size=(48, 24), dtype=np.uint8) & 0xF7
    kn = og.gemm_ex(a8, b8, 0.5, 2.0, None, "bf16", "kn")
    nk = og.gemm_ex(a8, np.ascontiguousarray(b8.T), 0.5, 2.0, None, "bf16", "nk")
    assert (kn == nk).all()
    assert (kn == og.fp8_gemm(a8, b8, 0.5, 2.0)).all()


def test_quantize_rows_is_the_group_quantizer_per_row():
    x = bits(gen_bf16((7, 96), "n1_outlier", seed=5))
    q, s = og.quantize_rows(x)
    for r in range(7):
        qr, sr = oq.quantize_with_scales(x[r].reshape(1, 1, 1, 96), oq.SCALE_PER_BH)
        assert (q[r] == qr.reshape(96)).all()
        assert s[r] == sr[0]


def test_linear_is_the_dequantized_product_rounded_once():
    x = bits(gen_bf16((33, 160), "n1", seed=6))
    w = bits(gen_bf16((48, 160), "n05", seed=7))
    bias = bits(gen_bf16((48,), "n05", seed=8))
    y = bf16_bits_to_f32(og.linear(x, w, bias)).astype(np.float64)
    x8, xs = og.quantize_rows(x)
    w8, ws = og.quantize_rows(w)
    ref = og.dequant_matmul(x8, w8, xs, ws, "nk") + bf16_bits_to_f32(bias)[None, :]
    # one bf16 rounding (2^-9 relative) plus fp32 rounding of the scale steps
    assert (np.abs(y - ref) <= 2.0**-8 * np.abs(ref) + 1e-6).all()
    # and it tracks the unquantized linear to FP8 accuracy
    full = bf16_bits_to_f32(x).astype(np.float64) @ bf16_bits_to_f32(w).astype(np.float64).T
    full += bf16_bits_to_f32(bias)[None, :]
    cos = (y * full).sum() / np.sqrt((y * y).sum() * (full * full).sum())
    assert cos > 0.998
