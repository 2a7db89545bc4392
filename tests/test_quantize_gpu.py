"""Bit-exact parity of the CUDA quantizer with the oracle (and so with the
reference's ``_per_bh_scale`` / ``_quantize``, which the oracle is pinned to
by tests/test_oracle_golden.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import bits, bytes_equal_nan_aware, fp8_bytes, gen_bf16, scales_equal
from oracle import quantize as oq

pytestmark = pytest.mark.gpu

CASES = [
    # (B, H, S, D, dist)
    (1, 2, 256, 128, "n1"),
    (2, 3, 300, 128, "n05"),      # ragged S (last block 44 rows)
    (1, 1, 77, 64, "n1_outlier"),  # S < one block
    (1, 2, 128, 32, "qk_div8"),
    (1, 1, 200, 256, "n1"),
    (1, 2, 130, 128, "zeros"),
    (1, 1, 256, 128, "tiny"),
    (1, 1, 256, 128, "huge"),
]


def _run(x_dev: torch.Tensor, mode: int, layout: str):
    from repercep_runtime_b200 import ops

    (res,) = ops.quantize_fp8([x_dev], scale_mode=mode, layout=layout)
    torch.cuda.synchronize()
    return fp8_bytes(res.data), res.scales.cpu().numpy()


@pytest.mark.parametrize("mode", [oq.SCALE_PER_BH, oq.SCALE_PER_BLOCK128])
@pytest.mark.parametrize("case", CASES, ids=lambda c: "x".join(map(str, c)))
def test_quantize_bit_exact(case, mode):
    B, H, S, D, dist = case
    x = gen_bf16((B, H, S, D), dist, seed=11)
    ref_bytes, ref_scales = oq.quantize_with_scales(bits(x), mode)
    got_bytes, got_scales = _run(x.cuda(), mode, "bhsd")
    assert scales_equal(got_scales.reshape(ref_scales.shape), ref_scales).all()
    eq = bytes_equal_nan_aware(got_bytes.reshape(ref_bytes.shape), ref_bytes)
    assert eq.all(), f"{(~eq).sum()} of {eq.size} bytes differ"


@pytest.mark.parametrize("mode", [oq.SCALE_PER_BH, oq.SCALE_PER_BLOCK128])
def test_quantize_bshd_strided_input(mode):
    """A (B,S,H,D) diffusers tensor is read in place (no transposing copy)."""
    B, H, S, D = 2, 4, 333, 128
    x_bhsd = gen_bf16((B, H, S, D), "n1", seed=3)
    x_bshd = x_bhsd.permute(0, 2, 1, 3).contiguous()
    ref_bytes, ref_scales = oq.quantize_with_scales(bits(x_bhsd), mode)
    got_bytes, got_scales = _run(x_bshd.cuda(), mode, "bshd")
    assert scales_equal(got_scales.reshape(ref_scales.shape), ref_scales).all()
    assert bytes_equal_nan_aware(got_bytes.reshape(ref_bytes.shape), ref_bytes).all()


def test_quantize_three_tensors_one_call():
    from repercep_runtime_b200 import ops

    xs = [gen_bf16((1, 2, 257, 128), "n1_outlier", seed=s) for s in (1, 2, 3)]
    res = ops.quantize_fp8([x.cuda() for x in xs], scale_mode=oq.SCALE_PER_BH)
    for x, r in zip(xs, res):
        ref_bytes, ref_scales = oq.quantize_with_scales(bits(x), oq.SCALE_PER_BH)
        assert scales_equal(r.scales.cpu().numpy(), ref_scales).all()
        assert bytes_equal_nan_aware(fp8_bytes(r.data).reshape(ref_bytes.shape), ref_bytes).all()


def test_quantize_nan_and_inf():
    """NaN poisons its (b,h) like torch.amax; inf gives scale inf -> NaN/0 bytes."""
    x = gen_bf16((1, 2, 128, 128), "n1", seed=5)
    x[0, 0, 3, 7] = float("nan")
    x[0, 1, 9, 1] = float("inf")
    for mode in (oq.SCALE_PER_BH, oq.SCALE_PER_BLOCK128):
        ref_bytes, ref_scales = oq.quantize_with_scales(bits(x), mode)
        got_bytes, got_scales = _run(x.cuda(), mode, "bhsd")
        assert scales_equal(got_scales.reshape(ref_scales.shape), ref_scales).all()
        assert bytes_equal_nan_aware(got_bytes.reshape(ref_bytes.shape), ref_bytes).all()


def test_quantize_rounding_boundaries():
    """Inputs that land on e4m3 rounding midpoints (ties) and the subnormal range."""
    # Scale fixed by one element at 425.6 -> scale == 1.0 exactly, q_mul == 1.0.
    vals = []
    for e in range(-9, 9):
        for m in range(16):
            v = (1 + m / 16.0) * 2.0**e  # every e4m3 midpoint and grid point
            vals += [v, -v]
    vals = np.array(vals, dtype=np.float32)
    n = 128 * 128
    x = torch.zeros(n, dtype=torch.float32)
    x[: len(vals)] = torch.from_numpy(vals)
    x[-1] = 425.6
    x = x.to(torch.bfloat16).reshape(1, 1, 128, 128)
    ref_bytes, ref_scales = oq.quantize_with_scales(bits(x), oq.SCALE_PER_BH)
    got_bytes, got_scales = _run(x.cuda(), oq.SCALE_PER_BH, "bhsd")
    assert scales_equal(got_scales, ref_scales).all()
    assert (got_bytes.reshape(ref_bytes.shape) == ref_bytes).all()


def test_quantize_full_cfg2_sampled():
    """cfg2 shape (B=2, H=32, S=8192, outliers): bytes of sampled (b,h) slices."""
    from repercep_runtime_b200 import ops

    B, H, S, D = 2, 32, 8192, 128
    x = gen_bf16((B, H, S, D), "n1_outlier", seed=21)
    (r,) = ops.quantize_fp8([x.cuda()], scale_mode=oq.SCALE_PER_BH)
    got = fp8_bytes(r.data).reshape(B * H, S, D)
    sc = r.scales.cpu().numpy()
    xb = bits(x).reshape(B * H, 1, S, D)
    for bh in (0, 37, 63):
        ref_bytes, ref_scales = oq.quantize_with_scales(xb[bh : bh + 1], oq.SCALE_PER_BH)
        assert scales_equal(sc[bh : bh + 1], ref_scales).all()
        assert bytes_equal_nan_aware(got[bh], ref_bytes.reshape(S, D)).all()


F16_CASES = [
    (1, 2, 300, 64, "n1"),
    (1, 1, 257, 128, "n1_outlier"),
    (1, 2, 128, 32, "qk_div8"),
    (1, 2, 64, 256, "tiny"),    # amax under the fp16 1e-6 floor (subnormals)
    (1, 1, 64, 128, "huge"),    # overflows fp16 to inf
    (1, 1, 130, 128, "zeros"),
]


@pytest.mark.parametrize("mode", [oq.SCALE_PER_BH, oq.SCALE_PER_BLOCK128])
@pytest.mark.parametrize("case", F16_CASES, ids=lambda c: "x".join(map(str, c)))
def test_quantize_f16_bit_exact(case, mode):
    """fp16 inputs: bytes and scales equal the oracle's fp16 restatement."""
    B, H, S, D, dist = case
    x = gen_bf16((B, H, S, D), dist, seed=12, dtype=torch.float16)
    ref_bytes, ref_scales = oq.quantize_with_scales(bits(x), mode, fmt="f16")
    got_bytes, got_scales = _run(x.cuda(), mode, "bhsd")
    assert scales_equal(got_scales.reshape(ref_scales.shape), ref_scales).all()
    eq = bytes_equal_nan_aware(got_bytes.reshape(ref_bytes.shape), ref_bytes)
    assert eq.all(), f"{(~eq).sum()} of {eq.size} bytes differ"


@pytest.mark.parametrize("D", [32, 64])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_quantize_padded_rows(D, dtype):
    """Rows widened to the attention kernel's 128 bytes: data as unpadded, zeros after."""
    from repercep_runtime_b200 import ops

    x = gen_bf16((2, 3, 200, D), "n1", seed=13, dtype=dtype)
    fmt = "f16" if dtype == torch.float16 else "bf16"
    ref_bytes, ref_scales = oq.quantize_with_scales(bits(x), oq.SCALE_PER_BLOCK128, fmt=fmt)
    (res,) = ops.quantize_fp8([x.cuda()], scale_mode=oq.SCALE_PER_BLOCK128, row_bytes=128)
    torch.cuda.synchronize()
    got = fp8_bytes(res.data).reshape(2, 3, 200, 128)
    assert res.d == D
    assert scales_equal(res.scales.cpu().numpy().reshape(ref_scales.shape), ref_scales).all()
    assert bytes_equal_nan_aware(got[..., :D], ref_bytes).all()
    assert (got[..., D:] == 0).all()
