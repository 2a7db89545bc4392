"""Failure detection without a GPU fault: a bounded pipeline wait that runs out
is reported through the device status word, and the context stays usable.

The kernels never trap or spin forever: every mbarrier wait gives up after a
fixed number of SM cycles, raises a CTA-wide abort flag and records a code.
``rp_selftest_wait_timeout`` runs that same wait on a barrier nothing arrives
on (a ~0.1 s limit here)."""

from __future__ import annotations

import math

import pytest
import torch

from helpers import bits, gen_bf16
from oracle import attention as oa
from oracle import quantize as oq

pytestmark = pytest.mark.gpu


def test_wait_timeout_is_reported_and_the_context_survives():
    from repercep_runtime_b200 import _lib, ops

    lib = _lib.load()
    _lib.device_status(reset=True)
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check("rp_selftest_wait_timeout", lib.rp_selftest_wait_timeout(200_000_000, stream))
    torch.cuda.synchronize()
    assert _lib.device_status() == 0x1FF
    assert _lib.device_status(reset=True) == 0x1FF
    assert _lib.device_status() == 0

    # the same context still runs the hot path correctly
    q, k, v = (gen_bf16((1, 2, 256, 128), "n05", seed=s) for s in (71, 72, 73))
    out = ops.fp8_attention(q.cuda(), k.cuda(), v.cuda()).float().cpu().numpy()
    q8, qs = oq.quantize_with_scales(bits(q), oq.SCALE_PER_BH)
    k8, ks = oq.quantize_with_scales(bits(k), oq.SCALE_PER_BH)
    v8, vs = oq.quantize_with_scales(bits(v), oq.SCALE_PER_BH)
    r = lambda a: a.reshape(2, 256, 128)  # noqa: E731
    ref = oa.attention_dequant(r(q8), r(k8), r(v8), qs, ks, vs, 1 / math.sqrt(128))
    m = oa.parity_metrics(out.reshape(2, 256, 128), ref)
    assert m["cos"] >= 0.999 and m["max_abs"] <= 2e-2, m
    assert _lib.device_status() == 0
