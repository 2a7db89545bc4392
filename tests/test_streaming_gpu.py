"""Host-tensor attention (copies pipelined with compute) equals the device path
bit for bit: the same kernels see the same (b, h) slices."""

from __future__ import annotations

import pytest
import torch

from helpers import gen_bf16
from repercep_runtime_b200 import ops
from repercep_runtime_b200.streaming import ChunkPlan, fp8_attention_host


def _device_ref(q, k, v, scale_mode, causal):
    qq, kq, vq = ops.quantize_fp8((q.cuda(), k.cuda(), v.cuda()), scale_mode=scale_mode)
    return ops.attention_fp8_quantized(qq, kq, vq, causal=causal).cpu()


@pytest.mark.gpu
@pytest.mark.parametrize("scale_mode", [ops.SCALE_PER_BH, ops.SCALE_PER_BLOCK128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("chunk", [1, 3, 8])
def test_host_stream_bit_exact(scale_mode, causal, chunk):
    B, H, S = 2, 4, 333
    q, k, v = (gen_bf16((B, H, S, 128), "n1", seed=s) for s in (21, 22, 23))
    q, k, v = (x.pin_memory() for x in (q, k, v))
    out = fp8_attention_host(q, k, v, causal=causal, scale_mode=scale_mode, plan=ChunkPlan(B * H, chunk))
    assert out.device.type == "cpu" and out.shape == q.shape
    ref = _device_ref(q, k, v, scale_mode, causal)
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))


@pytest.mark.gpu
def test_op_call_on_host_tensors_and_cross_length():
    from repercep_runtime_b200 import _lib
    from repercep_runtime_b200.attention import B200FP8Attention

    q = gen_bf16((1, 6, 200, 128), "n05", seed=31).pin_memory()
    k = gen_bf16((1, 6, 700, 128), "n05", seed=32).pin_memory()
    v = gen_bf16((1, 6, 700, 128), "n05", seed=33).pin_memory()
    op = B200FP8Attention(scale_mode=ops.SCALE_PER_BLOCK128)
    out = op(q, k, v)
    assert out.device.type == "cpu" and out.shape == q.shape
    ref = op(q.cuda(), k.cuda(), v.cuda()).cpu()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
    # pageable (unpinned) host tensors work too
    out2 = op(q.clone(), k.clone(), v.clone())
    assert torch.equal(out2.view(torch.int16), ref.view(torch.int16))
    assert _lib.device_status() == 0
