"""The allocation-free quantizer entry point, rp_quant_fp8_e4m3_noalloc.

Some callers cannot give this library any device memory beyond the tensors
they pass in and out (a plugin whose host hands over only its operands and
whose memory pool forbids raw cudaMalloc).  For them the per-(b,h) quantizer
keeps its partial-amax scratch in a fixed array inside the library.  These
tests call it through the C ABI and require byte-for-byte the same e4m3 output
and the same scales as the workspace-taking entry point, on two calls in a
row, also when a large call is followed by a smaller one that uses a strict
subset of the shared array's slots; that repeated calls leave the device's
free memory unchanged (no allocation anywhere below the call); and a clear
rejection of shapes larger than the array.

This file sorts last so that a run stopping at its first failure has already
run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import gen_bf16

pytestmark = pytest.mark.gpu

MAX_SLOTS = 262144  # capacity of the library's built-in scratch (uint32 slots)


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


def _strides(ts):
    vals = []
    for t in ts:
        vals.extend(t.stride())
    return (ctypes.c_int64 * len(vals))(*vals)


def _outputs(xs):
    B, H, S, D = xs[0].shape
    outs = [torch.empty((B, H, S, D), dtype=torch.float8_e4m3fn, device="cuda") for _ in xs]
    scales = [torch.empty((B * H,), dtype=torch.float32, device="cuda") for _ in xs]
    return outs, scales


def _with_workspace(lib, xs):
    B, H, S, D = xs[0].shape
    outs, scales = _outputs(xs)
    nbytes = ctypes.c_size_t(0)
    assert lib.rp_quant_workspace_bytes(len(xs), B, H, S, D, 0, ctypes.byref(nbytes)) == 0
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.rp_quant_fp8_e4m3(len(xs), _ptrs(xs), _strides(xs), B, H, S, D, 0, _ptrs(outs),
                               _ptrs(scales), ws.data_ptr(), nbytes.value, stream)
    assert rc == 0, lib.rp_last_error()
    return outs, scales


def _without_allocation(lib, xs, outs=None, scales=None):
    B, H, S, D = xs[0].shape
    if outs is None:
        outs, scales = _outputs(xs)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.rp_quant_fp8_e4m3_noalloc(len(xs), _ptrs(xs), _strides(xs), B, H, S, D, _ptrs(outs),
                                       _ptrs(scales), stream)
    assert rc == 0, lib.rp_last_error()
    return outs, scales


def _same_bytes(a: torch.Tensor, b: torch.Tensor) -> bool:
    return bool(torch.equal(a.view(torch.uint8), b.view(torch.uint8)))


def test_noalloc_matches_workspace_entry_point_two_calls_in_a_row():
    from repercep_runtime_b200 import _lib

    lib = _lib.load()
    cases = [((2, 8, 1000, 128), "n1_outlier", 101), ((1, 4, 4096, 128), "n05", 202)]
    for shape, dist, seed in cases:
        xs = [gen_bf16(shape, dist, seed + i).cuda() for i in range(3)]
        ref_out, ref_sc = _with_workspace(lib, xs)
        got_out, got_sc = _without_allocation(lib, xs)
        torch.cuda.synchronize()
        for r, g in zip(ref_out, got_out):
            assert _same_bytes(r, g)
        for r, g in zip(ref_sc, got_sc):
            assert np.array_equal(r.cpu().numpy().view(np.uint32), g.cpu().numpy().view(np.uint32))
    assert _lib.device_status() == 0


def _check_same(lib, xs, got_out, got_sc):
    ref_out, ref_sc = _with_workspace(lib, xs)
    torch.cuda.synchronize()
    for r, g in zip(ref_out, got_out):
        assert _same_bytes(r, g)
    for r, g in zip(ref_sc, got_sc):
        assert np.array_equal(r.cpu().numpy().view(np.uint32), g.cpu().numpy().view(np.uint32))


def test_noalloc_large_call_then_smaller_subset_call():
    """The second call's slots are a strict subset of the first's, so the
    first call's partial maxima are still in the rest of the array; the
    second call must read only what it wrote."""
    from repercep_runtime_b200 import _lib

    lib = _lib.load()
    big = [gen_bf16((2, 16, 6000, 128), "n1_outlier", 301 + i).cuda() * 8 for i in range(3)]
    small = [gen_bf16((1, 2, 700, 128), "n05", 401 + i).cuda() for i in range(2)]
    out_b, sc_b = _without_allocation(lib, big)
    out_s, sc_s = _without_allocation(lib, small)
    torch.cuda.synchronize()
    _check_same(lib, big, out_b, sc_b)
    _check_same(lib, small, out_s, sc_s)
    assert _lib.device_status() == 0


def test_noalloc_calls_leave_device_memory_unchanged():
    from repercep_runtime_b200 import _lib

    lib = _lib.load()
    xs = [gen_bf16((2, 8, 3000, 128), "n05", 501 + i).cuda() for i in range(3)]
    outs, scales = _outputs(xs)
    _without_allocation(lib, xs, outs, scales)  # warm-up: first call's set-up on this device
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(4):
        _without_allocation(lib, xs, outs, scales)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    _check_same(lib, xs, outs, scales)


def test_noalloc_rejects_shapes_beyond_its_scratch():
    from repercep_runtime_b200 import _lib

    lib = _lib.load()
    # 3 tensors x B*H=128 x ceil(89600/128)=700 chunks = 268800 slots > 262144
    B, H, S, D = 2, 64, 89600, 128
    assert 3 * B * H * ((S + 127) // 128) > MAX_SLOTS
    small = [torch.zeros(16, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    fake = (ctypes.c_int64 * 12)(*([H * S * D, S * D, D, 1] * 3))
    rc = lib.rp_quant_fp8_e4m3_noalloc(3, _ptrs(small), fake, B, H, S, D, _ptrs(small),
                                       _ptrs(small), torch.cuda.current_stream().cuda_stream)
    assert rc == -6  # RP_ERR_WORKSPACE
    assert b"scratch" in lib.rp_last_error()
