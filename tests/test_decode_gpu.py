"""Shared-prefix candidate decode on the GPU vs the oracle.

Candidate c's new token i attends to the whole shared prefix and to its own
suffix tokens 0..i; the oracle builds that mask explicitly over dequantised
inputs.  Tolerance as for attention: max-abs <= 2e-2, cosine >= 0.999.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from helpers import fp8_bytes, gen_bf16
from oracle import attention as oa

pytestmark = pytest.mark.gpu


def _run(C, T, P, H, dist="n1", p_mode=0):
    from repercep_runtime_b200 import ops
    from repercep_runtime_b200.attention import SharedPrefixFP8Decode

    D = 128
    q = gen_bf16((C * T, H, D), dist, 1).cuda()
    kp = gen_bf16((P, H, D), dist, 2).cuda()
    vp = gen_bf16((P, H, D), dist, 3).cuda()
    kx = gen_bf16((C * T, H, D), dist, 4).cuda()
    vx = gen_bf16((C * T, H, D), dist, 5).cuda()
    op = SharedPrefixFP8Decode(p_mode=p_mode)
    assert op.available and op.supports(C, T, H, D)
    prefix = op.quantize_prefix(kp, vp)
    qq, kxq, vxq = ops.quantize_fp8(
        (q.unsqueeze(0), kx.unsqueeze(0), vx.unsqueeze(0)), scale_mode=ops.SCALE_PER_BLOCK128, layout="bshd"
    )
    out = ops.prefix_decode_fp8_quantized(qq, prefix.k, prefix.v, kxq, vxq, candidates=C, tokens=T, p_mode=p_mode)
    out_op = op(q, prefix, kx, vx, candidates=C, tokens=T)
    torch.cuda.synchronize()
    assert torch.equal(out, out_op)  # the op quantises the same way
    r = lambda t, n: fp8_bytes(t.data).reshape(H, n, D)  # noqa: E731
    ref = oa.prefix_decode_dequant(
        r(qq, C * T), r(prefix.k, P), r(prefix.v, P), r(kxq, C * T), r(vxq, C * T),
        qq.scales.cpu().numpy(), prefix.k.scales.cpu().numpy(), prefix.v.scales.cpu().numpy(),
        kxq.scales.cpu().numpy(), vxq.scales.cpu().numpy(), C, T, 1 / math.sqrt(D),
    )
    got = out.float().cpu().numpy().transpose(1, 0, 2)  # (H, C*T, D)
    return oa.parity_metrics(got, ref)


@pytest.mark.parametrize(
    "C,T,P,H",
    [
        (64, 8, 512, 4),   # the token-VLA config (64 candidates x 8 tokens, 512 prefix), fewer heads
        (20, 8, 300, 2),   # ragged prefix and ragged candidate rows (160 rows)
        (16, 1, 256, 2),   # single new token per candidate
        (4, 32, 130, 1),   # long per-candidate suffix
    ],
)
def test_prefix_decode_matches_oracle(C, T, P, H):
    m = _run(C, T, P, H)
    assert m["max_abs"] <= 2e-2 and m["cos"] >= 0.999, m


def test_prefix_decode_full_vla_shape_hilo():
    m = _run(64, 8, 512, 32, p_mode=1)
    assert m["max_abs"] <= 2e-2 and m["cos"] >= 0.9999, m


def test_decode_right_after_the_prefix_is_written():
    """The decode is launched as a programmatic dependent of the launch before
    it; with the prefix quantized by that very launch (the suffix and Q
    quantized earlier) it must still read the finished prefix: the result is
    bit-equal to the same decode with a synchronisation in between."""
    from repercep_runtime_b200 import ops
    from repercep_runtime_b200.attention import SharedPrefixFP8Decode

    C, T, P, H, D = 64, 8, 512, 32, 128
    q, kx, vx = (gen_bf16((C * T, H, D), "n1", s).cuda() for s in (11, 12, 13))
    kp, vp = (gen_bf16((P, H, D), "n1", s).cuda() for s in (14, 15))
    op = SharedPrefixFP8Decode()
    qq, kxq, vxq = ops.quantize_fp8(
        (q.unsqueeze(0), kx.unsqueeze(0), vx.unsqueeze(0)), scale_mode=ops.SCALE_PER_BLOCK128, layout="bshd"
    )
    outs = []
    for sync in (True, False):
        prefix = op.quantize_prefix(kp, vp)  # the launch right before the decode
        if sync:
            torch.cuda.synchronize()
        outs.append(ops.prefix_decode_fp8_quantized(qq, prefix.k, prefix.v, kxq, vxq, candidates=C, tokens=T))
        torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
