"""Parity records beside the tolerance relaxations, the reference's own FP8
regression anchor, and the diffusers bridge on CUDA tensors.

Two configurations cannot meet an absolute max-abs bound of 2e-2 against fp32
attention on the dequantised inputs, and neither can the reference kernel's
own algorithm (P rounded once to e4m3 against 448,
kernels/triton_kernels/fp8_flash_attn_hopper.py:280-329, output rounded to
bf16, :586), run here as the tile-loop oracle pinned bit for bit to the
reference's kernel (tests/golden/attention_cases.npz):

* cfg2 (N(0,1) with 1 % x20 outliers): outputs reach |o| ~ 69 where one bf16
  ulp is 0.25-0.5, so rounding the exact result to bf16 alone costs up to 0.25;
* causal, P in e4m3: rows near the diagonal average a handful of keys, so P's
  rounding is not averaged out.

For both, these tests measure the absolute error of the B200 kernel and of the
reference algorithm on the same inputs and rows, print both, and require the
kernel's to be within 1.5x the reference algorithm's own (cos >= 0.999).
Run with ``-s`` to see the records.
"""

from __future__ import annotations

import functools
import json
import math

import numpy as np
import pytest
import torch

from helpers import fp8_bytes, gen_bf16
from oracle import attention as oa
from oracle import quantize as oq

pytestmark = pytest.mark.gpu

SM = 1 / math.sqrt(128)


def _bf16(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.bfloat16).float().numpy()


def _record(name: str, kernel: dict, ref_alg: dict, extra: dict | None = None) -> None:
    rec = {"case": name, "kernel_vs_fp32": kernel, "reference_algorithm_vs_fp32": ref_alg, **(extra or {})}
    print("PARITY_RECORD " + json.dumps(rec, sort_keys=True))


def _quantized(B, H, S, dist, seeds, mode):  # type: ignore[no-untyped-def]
    from repercep_runtime_b200 import ops

    dev = [gen_bf16((B, H, S, 128), dist, seed=s).cuda() for s in seeds]
    qq, kq, vq = ops.quantize_fp8(dev, scale_mode=mode)
    q8, k8, v8 = (fp8_bytes(t.data).reshape(B * H, S, 128) for t in (qq, kq, vq))
    qs, ks, vs = (t.scales.cpu().numpy() for t in (qq, kq, vq))
    return (qq, kq, vq), (q8, k8, v8, qs, ks, vs)


def _metrics(out: np.ndarray, ref: np.ndarray) -> dict:
    return {k: float(v) for k, v in oa.parity_metrics(out, ref).items()}


def test_cfg2_absolute_error_is_the_reference_algorithms_own():
    from repercep_runtime_b200 import ops

    B, H, S = 2, 32, 8192
    bhs = [0, 33, 63]
    rows = np.r_[0:64, 4000:4064, 8128:8192]
    (qq, kq, vq), (q8, k8, v8, qs, ks, vs) = _quantized(B, H, S, "n1_outlier", (31, 32, 33), oq.SCALE_PER_BH)
    out = ops.attention_fp8_quantized(qq, kq, vq, p_mode=0)
    torch.cuda.synchronize()
    got = out.reshape(B * H, S, 128)[bhs][:, rows].float().cpu().numpy()
    fp32 = oa.attention_dequant(q8, k8, v8, qs, ks, vs, SM, bh_index=bhs, rows=rows)
    alg = np.stack([
        oa.reference_tile_loop(q8[b : b + 1][:, rows], k8[b : b + 1], v8[b : b + 1], qs[b : b + 1],
                               ks[b : b + 1], vs[b : b + 1], SM)[0]
        for b in bhs
    ])
    mk, mr = _metrics(got, fp32), _metrics(_bf16(alg), fp32)
    floor = _metrics(_bf16(fp32), fp32)
    _record("cfg2 B2 H32 S8192 n1+1%x20, per-(b,h), p e4m3, bh 0/33/63 x 192 rows", mk, mr,
            {"bf16_rounding_of_fp32": floor})
    assert mr["max_abs"] > 2e-2  # the reference itself cannot meet the absolute bound here
    assert mk["cos"] >= 0.999
    assert mk["max_abs"] <= 1.5 * mr["max_abs"], (mk, mr)
    assert mk["mean_abs"] <= 1.5 * mr["mean_abs"], (mk, mr)


@pytest.mark.parametrize("S", [384, 1024])
def test_causal_absolute_error_is_the_reference_algorithms_own(S):
    from repercep_runtime_b200 import ops

    B, H = 1, 2
    (qq, kq, vq), (q8, k8, v8, qs, ks, vs) = _quantized(B, H, S, "n1", (14, 15, 16), oq.SCALE_PER_BH)
    out = ops.attention_fp8_quantized(qq, kq, vq, causal=True, p_mode=0)
    torch.cuda.synchronize()
    got = out.reshape(B * H, S, 128).float().cpu().numpy()
    fp32 = oa.attention_dequant(q8, k8, v8, qs, ks, vs, SM, causal=True)
    alg = oa.reference_tile_loop(q8, k8, v8, qs, ks, vs, SM, causal=True)
    mk, mr = _metrics(got, fp32), _metrics(_bf16(alg), fp32)
    _record(f"causal B1 H2 S{S} n1, per-(b,h), p e4m3", mk, mr)
    assert mk["cos"] >= 0.999
    assert mk["max_abs"] <= 1.5 * mr["max_abs"], (mk, mr)


@pytest.mark.parametrize("scale_mode", ["bh", "block128"])
def test_reference_fp8_anchor_b1_h8_s4096(scale_mode, monkeypatch):
    """The reference's own FP8 regression anchor (tests/test_attention_cuda.py:142-170):
    B1 H8 S4096 D128, torch.manual_seed(0), q and k drawn on the device / 8,
    v unscaled, against bf16 SDPA; mean relative difference < 0.10 (the
    reference measured 3.4 % for its Hopper kernel)."""
    from repercep_runtime_b200.attention import B200FP8Attention

    monkeypatch.setenv("REPERCEP_B200_SCALE_MODE", scale_mode)
    op = B200FP8Attention()
    assert op.available, op.unavailable_reason
    torch.manual_seed(0)
    q = torch.randn(1, 8, 4096, 128, device="cuda", dtype=torch.bfloat16) / 8.0
    k = torch.randn_like(q) / 8.0
    v = torch.randn_like(q)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    out = op(q, k, v)
    rel = float((out - ref).abs().mean() / ref.abs().mean())
    print("PARITY_RECORD " + json.dumps({"case": f"reference anchor, scale {scale_mode}", "mean_rel": rel}))
    assert out.dtype == torch.bfloat16 and out.shape == q.shape
    assert rel < 0.10, rel


@pytest.mark.parametrize("guard", ["1", "deferred"])
def test_diffusers_bridge_on_cuda_bshd(guard, monkeypatch):
    """The bridge function diffusers calls, on (B, S, H, D) CUDA tensors past
    the 4096-token crossover: it runs the B200 kernel (strided BSHD in and
    out) and matches fp32 attention on the dequantised inputs."""
    from repercep_runtime_b200 import ops
    from repercep_runtime_b200.attention import diffusers_backend as db

    monkeypatch.setenv("REPERCEP_B200_FINITE_GUARD", guard)
    monkeypatch.delenv("REPERCEP_FP8_ATTENTION", raising=False)
    B, S, H = 1, 4352, 4
    x = [gen_bf16((B, S, H, 128), "n05", seed=s).cuda() for s in (71, 72, 73)]
    assert db._route_should_use_fp8(*x)
    db.nonfinite_calls(reset=True)
    out = db._repercep_fp8_attention(*x)
    torch.cuda.synchronize()
    op = getattr(db._repercep_fp8_attention, "_op", None)
    assert op is not None and op.available
    assert out.shape == (B, S, H, 128) and out.dtype == torch.bfloat16
    # the same quantisation the bridge applies (the op's scale mode, BSHD strides)
    qq, kq, vq = ops.quantize_fp8(x, scale_mode=op.scale_mode, layout="bshd")
    q8, k8, v8 = (fp8_bytes(t.data).reshape(B * H, S, 128) for t in (qq, kq, vq))
    qs, ks, vs = (t.scales.cpu().numpy() for t in (qq, kq, vq))
    rows = np.r_[0:64, 2000:2064, 4288:4352]
    fp32 = oa.attention_dequant(q8, k8, v8, qs, ks, vs, SM, bh_index=list(range(B * H)), rows=rows)
    got = out.permute(0, 2, 1, 3).reshape(B * H, S, 128)[:, rows].float().cpu().numpy()
    m = _metrics(got, fp32)
    assert m["max_abs"] <= 2e-2 and m["cos"] >= 0.999, m
    if guard == "deferred":
        assert db.nonfinite_calls() == 0
