"""diffusers attention-dispatch bridge for B200 — mirrors the reference's
``"repercep_fp8"`` backend (src/repercep/attention/diffusers_backend.py).

The backend function keeps the reference's signature (:160-171) and routing
rules (:44, :52-79, :199-231): bf16 or fp16, q/k/v of one shape, a head dim
in {32, 64, 128, 256}, seq_len >= the crossover, no mask / dropout / GQA /
context-parallel config; everything else goes to a native SDPA fallback.  What changes is the
layout handling: diffusers passes (B, S, H, D) and the B200 kernels read and
write that layout through strides, so the reference's three
``permute(0, 2, 1, 3).contiguous()`` copies in and one out (:264-267, :286)
are gone.  The reference's non-finite guard (``isfinite().all()`` per call,
:271-285, falling back to SDPA for that call) is kept by default because it is
part of the seam's contract, and it costs a host synchronisation per call.
``REPERCEP_B200_FINITE_GUARD=deferred`` keeps the check on the device instead:
every call adds "any non-finite output" to a per-device counter without
synchronising, and ``nonfinite_calls()`` reads it (once per denoise step, say);
``REPERCEP_B200_FINITE_GUARD=0`` drops the check.

Registration touches diffusers' private registry exactly like the reference
(:289-339) and is a no-op when diffusers is not installed.
"""

from __future__ import annotations

import logging
import os
from typing import Any

logger = logging.getLogger(__name__)

# per-device count of calls with a non-finite output (deferred guard)
_NONFINITE: dict[Any, Any] = {}


def _guard_mode() -> str:
    raw = os.environ.get("REPERCEP_B200_FINITE_GUARD", "1").strip().lower()
    if raw in ("0", "off", "false"):
        return "off"
    return "deferred" if raw == "deferred" else "sync"


def record_nonfinite(out: Any) -> None:
    """Add 1 to ``out``'s device counter when ``out`` holds a non-finite
    value, on the device and without synchronising."""
    import torch

    cnt = _NONFINITE.get(out.device)
    if cnt is None:
        cnt = _NONFINITE[out.device] = torch.zeros((), dtype=torch.int64, device=out.device)
    cnt.add_((~torch.isfinite(out).all()).to(torch.int64))


def nonfinite_calls(reset: bool = False) -> int:
    """Calls so far (over all devices) whose output held a non-finite value,
    under the deferred guard.  Synchronises with those devices."""
    total = 0
    for cnt in _NONFINITE.values():
        total += int(cnt.item())
        if reset:
            cnt.zero_()
    return total

REPERCEP_FP8_BACKEND_NAME = "repercep_fp8"


def _min_seq_len() -> int:
    # The reference's crossover on Hopper/MI300 is 4096 tokens (:44).
    return int(os.environ.get("REPERCEP_B200_MIN_SEQ_LEN", "4096"))


def _route_should_use_fp8(query: Any, key: Any, value: Any) -> bool:
    import torch

    if query.dtype not in (torch.bfloat16, torch.float16):
        return False
    if query.shape != key.shape or query.shape != value.shape:
        return False
    if query.dim() != 4 or query.shape[-1] not in (32, 64, 128, 256):
        return False
    return bool(query.shape[-3] >= _min_seq_len())


def _native_fallback(
    query: Any,
    key: Any,
    value: Any,
    *,
    attn_mask: Any,
    dropout_p: float,
    is_causal: bool,
    scale: float | None,
    enable_gqa: bool,
) -> Any:
    """diffusers' native path: SDPA on (B, H, S, D) views, back to (B, S, H, D)."""
    import torch

    if (
        attn_mask is not None
        and attn_mask.ndim == 2
        and attn_mask.shape[0] == query.shape[0]
        and attn_mask.shape[1] == key.shape[1]
    ):
        attn_mask = attn_mask.unsqueeze(1).unsqueeze(1)
    out = torch.nn.functional.scaled_dot_product_attention(
        query.permute(0, 2, 1, 3),
        key.permute(0, 2, 1, 3),
        value.permute(0, 2, 1, 3),
        attn_mask=attn_mask,
        dropout_p=dropout_p,
        is_causal=is_causal,
        scale=scale,
        enable_gqa=enable_gqa,
    )
    return out.permute(0, 2, 1, 3)


def _repercep_fp8_attention(
    query: Any,
    key: Any,
    value: Any,
    attn_mask: Any = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    scale: float | None = None,
    enable_gqa: bool = False,
    return_lse: bool = False,
    _parallel_config: Any = None,
) -> Any:
    """The diffusers backend function: (B, S, H, D) in, (B, S, H, D) out."""
    import torch

    if return_lse:
        raise ValueError("repercep_fp8 backend does not support return_lse=True.")
    fallback = dict(
        attn_mask=attn_mask,
        dropout_p=dropout_p,
        is_causal=is_causal,
        scale=scale,
        enable_gqa=enable_gqa,
    )
    if (
        _parallel_config is not None
        or attn_mask is not None
        or dropout_p != 0.0
        or enable_gqa
        or not _route_should_use_fp8(query, key, value)
    ):
        return _native_fallback(query, key, value, **fallback)

    op = getattr(_repercep_fp8_attention, "_op", None)
    if op is None:
        from repercep_runtime_b200.attention.fp8_b200 import B200FP8Attention

        op = B200FP8Attention()
        _repercep_fp8_attention._op = op  # type: ignore[attr-defined]
    if not op.available:
        return _native_fallback(query, key, value, **fallback)

    from repercep_runtime_b200 import ops

    out = ops.fp8_attention(
        query,
        key,
        value,
        causal=is_causal,
        scale=scale,
        scale_mode=op.scale_mode,
        p_mode=op.p_mode,
        layout="bshd",
    )
    mode = _guard_mode()
    if mode == "deferred":
        record_nonfinite(out)
    elif mode == "sync" and not torch.isfinite(out).all():
        logger.warning(
            "repercep_fp8: non-finite output at shape %s; falling back to native SDPA",
            tuple(query.shape),
        )
        return _native_fallback(query, key, value, **fallback)
    return out


def _ensure_backend_name_registered() -> Any:
    """Add "repercep_fp8" to diffusers' AttentionBackendName lookup maps."""
    from diffusers.models.attention_dispatch import AttentionBackendName

    value, name = REPERCEP_FP8_BACKEND_NAME, "REPERCEP_FP8"
    existing = AttentionBackendName._value2member_map_.get(value)
    if existing is not None:
        return existing
    member = str.__new__(AttentionBackendName, value)
    member._name_ = name
    member._value_ = value
    AttentionBackendName._member_map_[name] = member
    AttentionBackendName._value2member_map_[value] = member
    if name not in AttentionBackendName._member_names_:
        AttentionBackendName._member_names_.append(name)
    return member


def register_repercep_fp8_backend() -> Any:
    """Register the backend function with diffusers (idempotent)."""
    import inspect

    from diffusers.models.attention_dispatch import _AttentionBackendRegistry

    member = _ensure_backend_name_registered()
    if member not in _AttentionBackendRegistry._backends:
        _AttentionBackendRegistry._backends[member] = _repercep_fp8_attention
        _AttentionBackendRegistry._constraints[member] = []
        _AttentionBackendRegistry._supported_arg_names[member] = set(
            inspect.signature(_repercep_fp8_attention).parameters
        )
    return member


def activate_repercep_fp8_backend() -> bool:
    """Make "repercep_fp8" the active diffusers backend; False if already active."""
    from diffusers.models.attention_dispatch import _AttentionBackendRegistry

    member = register_repercep_fp8_backend()
    if _AttentionBackendRegistry._active_backend == member:
        return False
    _AttentionBackendRegistry.set_active_backend(member)
    return True


def maybe_activate_from_env() -> bool:
    """Activate iff REPERCEP_FP8_ATTENTION is truthy (reference :364-388)."""
    if os.environ.get("REPERCEP_FP8_ATTENTION", "").lower() not in ("1", "true", "on", "triton", "b200"):
        return False
    try:
        return activate_repercep_fp8_backend()
    except ImportError:
        logger.info("repercep_fp8: diffusers is not installed; nothing to activate")
        return False


try:  # register on import, like the reference (:394-399)
    register_repercep_fp8_backend()
except Exception as exc:  # diffusers absent or its internals changed
    logger.debug("repercep_fp8: registration deferred (%s: %s)", type(exc).__name__, exc)


__all__ = [
    "REPERCEP_FP8_BACKEND_NAME",
    "activate_repercep_fp8_backend",
    "maybe_activate_from_env",
    "register_repercep_fp8_backend",
]
