"""The drop-in seams on CPU: AttentionOp / Backend conformance, selection,
supports() gating, the diffusers bridge routing and its SDPA fallback."""

from __future__ import annotations

import importlib

import pytest
import torch

from repercep_runtime_b200.attention import (
    AttentionKind,
    AttentionOp,
    AttentionShape,
    B200FP8Attention,
    NaiveAttention,
    SharedPrefixFP8Decode,
    select_attention_op,
)
from repercep_runtime_b200.backend import B200Backend, Backend, available_backends, select_backend
from repercep_runtime_b200.backend.b200 import arch_for_capability
from repercep_runtime_b200.hardware import B200, H100, DType, Vendor

SHAPE = AttentionShape(batch=2, heads=32, seq_len_q=57600, seq_len_kv=57600, head_dim=128)


def test_ops_satisfy_the_protocols():
    assert isinstance(B200FP8Attention(), AttentionOp)
    assert isinstance(NaiveAttention(), AttentionOp)
    assert isinstance(B200Backend(), Backend)


def test_names_are_stable():
    assert B200FP8Attention.name == "fp8-b200-flash"
    assert SharedPrefixFP8Decode.name == "fp8-b200-prefix-decode"
    assert B200Backend.name == "cuda-b200"


def test_available_never_raises_and_explains_itself_on_cpu():
    op = B200FP8Attention()
    assert op.available is False
    assert "sm_100" in (op.unavailable_reason or "")
    with pytest.raises(RuntimeError, match="not available"):
        op(torch.zeros(1), torch.zeros(1), torch.zeros(1))


def test_supports_gates_like_the_reference(monkeypatch):
    op = B200FP8Attention()
    monkeypatch.setattr(op, "_import_error", None)
    assert op.supports(SHAPE, DType.BF16)
    assert op.supports(SHAPE, DType.FP16)
    assert not op.supports(SHAPE, DType.FP32)
    for d in (32, 64, 128, 256):  # the reference's head-dim set, fp8_hopper_triton.py:41
        assert op.supports(AttentionShape(2, 32, 4096, 4096, d), DType.BF16)
    assert not op.supports(AttentionShape(2, 32, 4096, 4096, 96), DType.BF16)
    assert not op.supports(AttentionShape(2, 32, 4096, 4096, 128, AttentionKind.NEIGHBORHOOD), DType.BF16)
    assert op.supports(AttentionShape(2, 32, 4096, 4096, 128, AttentionKind.CAUSAL), DType.BF16)
    assert not op.supports(AttentionShape(2, 32, 4096, 1024, 128, AttentionKind.CAUSAL), DType.BF16)
    assert op.supports(AttentionShape(2, 32, 4096, 1024, 128), DType.BF16)  # cross-length, non-causal


def test_env_selects_scale_and_p_modes(monkeypatch):
    monkeypatch.setenv("REPERCEP_B200_SCALE_MODE", "block128")
    monkeypatch.setenv("REPERCEP_B200_P_MODE", "hilo")
    op = B200FP8Attention()
    assert (op.scale_mode, op.p_mode) == (1, 1)
    monkeypatch.setenv("REPERCEP_B200_P_MODE", "bogus")
    with pytest.raises(ValueError, match="REPERCEP_B200_P_MODE"):
        B200FP8Attention()


def test_registry_floor_without_env(monkeypatch):
    monkeypatch.delenv("REPERCEP_FP8_ATTENTION", raising=False)
    import repercep_runtime_b200.attention.registry as reg

    reg = importlib.reload(reg)
    assert reg.select_attention_op(B200, SHAPE, DType.BF16).name == "naive-sdpa"


def test_registry_picks_b200_op_when_enabled_and_supported(monkeypatch):
    monkeypatch.setenv("REPERCEP_FP8_ATTENTION", "1")
    import repercep_runtime_b200.attention.fp8_b200 as f
    import repercep_runtime_b200.attention.registry as reg

    monkeypatch.setattr(f, "b200_device_present", lambda: True)
    reg = importlib.reload(reg)
    try:
        op = reg.select_attention_op(B200, SHAPE, DType.BF16)
        assert op.name == "fp8-b200-flash"
        assert reg.select_attention_op(B200, SHAPE, DType.FP16).name == "fp8-b200-flash"
        # other arch / dtype / head dim fall through to the floor, like the reference's chain
        assert reg.select_attention_op(H100, SHAPE, DType.BF16).name == "naive-sdpa"
        assert reg.select_attention_op(B200, SHAPE, DType.FP32).name == "naive-sdpa"
        odd = AttentionShape(2, 32, 4096, 4096, 96)
        assert reg.select_attention_op(B200, odd, DType.BF16).name == "naive-sdpa"
    finally:
        monkeypatch.delenv("REPERCEP_FP8_ATTENTION")
        importlib.reload(reg)


def test_backend_on_a_cpu_host():
    b = B200Backend()
    assert b.vendor is Vendor.NVIDIA
    assert b.is_available() is False
    assert b.devices() == ()
    assert b.default_dtype() is DType.BF16
    assert "naive-sdpa" in b.capabilities().attention_ops
    assert available_backends() == ()
    with pytest.raises(RuntimeError):
        select_backend()
    with pytest.raises(ValueError, match="unknown backend"):
        select_backend("rocm")
    with pytest.raises(RuntimeError, match="not available"):
        select_backend("cuda-b200")


def test_arch_mapping_closes_the_reference_gap():
    assert arch_for_capability(10, 0) is B200
    assert arch_for_capability(9, 0).family == "unknown"


def test_naive_floor_matches_sdpa():
    q, k, v = (torch.randn(1, 2, 16, 8) for _ in range(3))
    out = NaiveAttention()(q, k, v, causal=True)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert torch.allclose(out, ref)


def test_diffusers_bridge_routes_and_falls_back_on_cpu():
    from repercep_runtime_b200.attention import diffusers_backend as db

    q = torch.randn(1, 4096, 2, 128, dtype=torch.bfloat16)
    assert db._route_should_use_fp8(q, q, q)
    assert not db._route_should_use_fp8(q.float(), q.float(), q.float())
    assert not db._route_should_use_fp8(q[:, :100], q[:, :100], q[:, :100])
    small = torch.randn(1, 64, 2, 32)
    out = db._repercep_fp8_attention(small, small, small)
    ref = torch.nn.functional.scaled_dot_product_attention(
        small.permute(0, 2, 1, 3), small.permute(0, 2, 1, 3), small.permute(0, 2, 1, 3)
    ).permute(0, 2, 1, 3)
    assert out.shape == small.shape and torch.allclose(out, ref)
    with pytest.raises(ValueError, match="return_lse"):
        db._repercep_fp8_attention(small, small, small, return_lse=True)
    assert db.maybe_activate_from_env() is False  # env unset


def test_decode_op_supports():
    op = SharedPrefixFP8Decode()
    assert not op.available
    op._import_error = None
    assert op.supports(64, 8, 32, 128)
    assert not op.supports(64, 3, 32, 128)
    assert not op.supports(64, 8, 32, 64)


def test_ops_reject_cpu_tensors():
    from repercep_runtime_b200 import ops

    x = torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises((ValueError, RuntimeError)):
        ops.quantize_fp8([x])


def test_deferred_finite_guard_counts_without_sync(monkeypatch):
    """The deferred guard adds non-finite calls to a device counter; the
    count is read once, later (here on CPU tensors)."""
    from repercep_runtime_b200.attention import diffusers_backend as db

    monkeypatch.setenv("REPERCEP_B200_FINITE_GUARD", "deferred")
    assert db._guard_mode() == "deferred"
    db.nonfinite_calls(reset=True)
    ok = torch.ones(2, 3)
    bad = torch.ones(2, 3)
    bad[1, 2] = float("nan")
    for t in (ok, bad, ok, bad, bad):
        db.record_nonfinite(t)
    assert db.nonfinite_calls(reset=True) == 3
    assert db.nonfinite_calls() == 0
    monkeypatch.setenv("REPERCEP_B200_FINITE_GUARD", "0")
    assert db._guard_mode() == "off"
    monkeypatch.setenv("REPERCEP_B200_FINITE_GUARD", "1")
    assert db._guard_mode() == "sync"
    monkeypatch.setenv("REPERCEP_B200_FINITE_GUARD", "sync")
    assert db._guard_mode() == "sync"
    monkeypatch.delenv("REPERCEP_B200_FINITE_GUARD")
    assert db._guard_mode() == "deferred"  # the device-side check is the default
