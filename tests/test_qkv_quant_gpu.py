"""The QKV projection with the attention quantizer fused into the GEMM epilogue
(rp_fp8_gemm_qkv_quant) against the two separate launches it replaces: the
FP8 GEMM with a bf16 output (rp_fp8_gemm_ex), then the per-128-token-block
quantizer (rp_quant_fp8_e4m3) on the (B, S, 3, H, 128) view of that output.
The e4m3 bytes and the scales must be identical.

Cases cover ragged sequence lengths (blocks and CTA row tiles cut by the end
of a batch; a batch's tail rows overlap the next batch's rows in the A
operand), an odd head count (the last column tile half past N), K not a
multiple of the 128-byte K block, per-row / per-column / scalar scales, a bias,
and infinite values (a bias of +inf makes a block's amax and scale infinite,
the quantizer's special-value path).  Both GEMM forms (CTA pairs and single
CTAs) run through the variants test of the GEMM suite.
"""

from __future__ import annotations

import pytest
import torch

from repercep_runtime_b200 import linear, ops

pytestmark = pytest.mark.gpu

CASES = [
    # B, S, H, K, scales, bias
    (2, 1000, 4, 512, "rowcol", "bias"),
    (1, 256, 3, 192, "rowcol", None),
    (3, 300, 2, 256, "scalar", "bias"),
    (2, 128, 2, 128, "rowcol", "inf"),
    (1, 4096, 8, 1024, "rowcol", "bias"),
]


def _operands(B, S, H, K, scales, bias, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    N = 3 * H * 128
    x = torch.randn(B * S, K, device="cuda", generator=g, dtype=torch.float32).to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    x8, xs = linear.quantize_rows(x)
    w8, ws = linear.quantize_rows(w)
    if scales == "scalar":
        xs, ws = 0.75, 1.5
    b = None
    if bias is not None:
        b = (torch.randn(N, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
        if bias == "inf":
            b[5] = float("inf")       # Q head 0, one column: that head's blocks have amax inf
            b[3 * 128 + 7] = float("-inf")
    return x8, xs, w8, ws, b


def _separate(x8, xs, w8, ws, b, B, S, H):
    c = linear.gemm_ex(x8, w8, xs, ws, bias=b)            # (B*S, 3*H*128) bf16
    c5 = c.view(B, S, 3, H, 128)
    views = [c5[:, :, i] for i in range(3)]                # (B, S, H, 128), BSHD strides
    return ops.quantize_fp8(views, scale_mode=ops.SCALE_PER_BLOCK128, layout="bshd")


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(map(str, c)))
def test_fused_qkv_quantize_matches_gemm_then_quantize(case):
    B, S, H, K, scales, bias = case
    x8, xs, w8, ws, b = _operands(B, S, H, K, scales, bias, seed=B * 1000 + S + H)
    fused = linear.gemm_qkv_quant(x8, w8, xs, ws, H, S, bias=b)
    ref = _separate(x8, xs, w8, ws, b, B, S, H)
    torch.cuda.synchronize()
    for name, f, r in zip("qkv", fused, ref):
        assert f.data.shape == (B, H, S, 128) and f.scales.shape == (B * H, (S + 127) // 128)
        fb, rb = f.data.view(torch.uint8), r.data.view(torch.uint8).reshape(B, H, S, 128)
        mism = (fb != rb).sum().item()
        assert mism == 0, f"{name}: {mism} e4m3 bytes differ"
        fs, rs = f.scales.view(torch.int32), r.scales.view(torch.int32)
        assert torch.equal(fs, rs), f"{name}: scales differ"
    from repercep_runtime_b200 import _lib

    assert _lib.device_status() == 0


def test_fused_qkv_feeds_the_attention_kernel():
    """The fused outputs drive the attention kernel directly, and give the
    same result as attention on the separately quantized tensors."""
    B, S, H, K = 1, 1024, 2, 256
    x8, xs, w8, ws, b = _operands(B, S, H, K, "rowcol", "bias", seed=7)
    q, k, v = linear.gemm_qkv_quant(x8, w8, xs, ws, H, S, bias=b)
    out = ops.attention_fp8_quantized(q, k, v)
    rq, rk, rv = _separate(x8, xs, w8, ws, b, B, S, H)
    ref = ops.attention_fp8_quantized(rq, rk, rv)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


def test_qkv_projection_fp8_from_hidden_states():
    B, S, H, hidden = 2, 384, 2, 256
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(B, S, hidden, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(3 * H * 128, hidden, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    w8, ws = linear.quantize_rows(w)
    q, k, v = linear.qkv_projection_fp8(x, w8, ws, H)
    x8, xs = linear.quantize_rows(x.reshape(B * S, hidden))
    rq, rk, rv = _separate(x8, xs, w8, ws, None, B, S, H)
    torch.cuda.synchronize()
    for f, r in ((q, rq), (k, rk), (v, rv)):
        assert torch.equal(f.data.view(torch.uint8).flatten(), r.data.view(torch.uint8).flatten())
        assert torch.equal(f.scales, r.scales)


def test_fused_qkv_rejects_bad_shapes():
    x8 = torch.zeros(256, 128, dtype=linear.FP8, device="cuda")
    w8 = torch.zeros(3 * 2 * 128, 128, dtype=linear.FP8, device="cuda")
    with pytest.raises(ValueError, match="whole batches"):
        linear.gemm_qkv_quant(x8, w8, 1.0, 1.0, 2, 100)
    with pytest.raises(ValueError, match="w8 must be"):
        linear.gemm_qkv_quant(x8, w8, 1.0, 1.0, 3, 128)
