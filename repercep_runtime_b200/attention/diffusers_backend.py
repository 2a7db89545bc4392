"""diffusers attention-dispatch bridge for B200 -- the reference's
``"repercep_fp8"`` backend (src/repercep/attention/diffusers_backend.py) with
the B200 kernels behind it.

The backend function keeps the reference's signature (:160-171) and routing
rules (:44, :52-79, :186-231): bf16 or fp16, q/k/v of one shape, a head dim
in {32, 64, 128, 256}, seq_len >= the crossover, no mask / dropout / GQA /
context-parallel config, ``REPERCEP_FP8_ATTENTION`` not ``fa``/``flash``.
What changes is the layout handling: diffusers passes (B, S, H, D) and the
B200 kernels read and write that layout through strides, so the reference's
three ``permute(0, 2, 1, 3).contiguous()`` copies in and one out (:264-267,
:286) are gone.  The reference's non-finite guard (``isfinite().all()`` per
call, :271-285, falling back to SDPA for that call) costs a host
synchronisation per call; by default the check stays on the device instead:
every call adds "any non-finite output" to a per-device counter without
synchronising, and ``nonfinite_calls()`` reads it (once per denoise step, say).
The FP8 path turns finite inputs into finite outputs (the quantizer saturates
at the e4m3 range and the softmax is computed against the running max), so a
non-finite output comes from a non-finite input, where the SDPA fallback is
non-finite too.  ``REPERCEP_B200_FINITE_GUARD=sync`` (or ``1``) restores the
reference's per-call check and fallback; ``REPERCEP_B200_FINITE_GUARD=0`` drops
the check.

Registration: the ``"repercep_fp8"`` entry of diffusers' registry is set to
this module's function even when the reference's module registered first
(importing ``repercep.attention`` does, :394-399); the function it replaces is
kept, and every call this bridge does not serve on the B200 kernel (no sm_100
device, a shape or option the kernel does not take, ``fa``/``flash`` mode) is
handed to it, so the reference's own routing (its flash-attn wrapper, its SDPA
fallback) stays in force for those.  Without a previous function, those calls
go to SDPA as in diffusers' native path.  The reference's Wan installer
(attention/wan_processor.py:45-50) and ``CosmosEngine.load`` (models/cosmos.py:168-170)
look the entry up by name, so they reach this function.  Registration is a
no-op when diffusers is not installed.
"""

from __future__ import annotations

import logging
import os
from typing import Any

logger = logging.getLogger(__name__)

# per-device count of calls with a non-finite output (deferred guard)
_NONFINITE: dict[Any, Any] = {}


def _guard_mode() -> str:
    raw = os.environ.get("REPERCEP_B200_FINITE_GUARD", "deferred").strip().lower()
    if raw in ("0", "off", "false"):
        return "off"
    return "sync" if raw in ("1", "sync", "on", "true") else "deferred"


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

    def hand_off() -> Any:
        prev = handoff_target()
        if prev is not None:
            return prev(query, key, value, **fallback, return_lse=return_lse,
                        _parallel_config=_parallel_config)
        return _native_fallback(query, key, value, **fallback)

    if (
        os.environ.get("REPERCEP_FP8_ATTENTION", "").lower() in ("fa", "flash")
        or _parallel_config is not None
        or attn_mask is not None
        or dropout_p != 0.0
        or enable_gqa
        or not _route_should_use_fp8(query, key, value)
    ):
        return hand_off()

    op = getattr(_repercep_fp8_attention, "_op", None)
    if op is None:
        from repercep_runtime_b200.attention.fp8_b200 import B200FP8Attention

        op = B200FP8Attention()
        _repercep_fp8_attention._op = op  # type: ignore[attr-defined]
    if not op.available or query.device.type != "cuda":
        return hand_off()

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


# The function this module's registration replaced (the reference's, when it
# registered first); calls the B200 kernel does not serve go to it.
_PREVIOUS: dict[str, Any] = {}


def handoff_target() -> Any:
    """Where calls the B200 kernel does not serve go: the function this
    module's registration replaced, else (this module registered first) the
    reference's own backend function when the reference is importable, else
    None (diffusers' native SDPA path, ``_native_fallback``)."""
    fn = _PREVIOUS.get("fn")
    if fn is None:
        try:
            from repercep.attention.diffusers_backend import _repercep_fp8_attention as fn
        except ImportError:
            return None
        _PREVIOUS["fn"] = fn
    return fn


def register_repercep_fp8_backend() -> Any:
    """Make this module's function diffusers' "repercep_fp8" backend
    (idempotent), keeping any function it replaces as the hand-off target."""
    import inspect

    from diffusers.models.attention_dispatch import _AttentionBackendRegistry

    member = _ensure_backend_name_registered()
    prev = _AttentionBackendRegistry._backends.get(member)
    if prev is not _repercep_fp8_attention:
        if prev is not None:
            _PREVIOUS["fn"] = prev
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


# The reference's accepted values (:377) plus "b200".
_ACTIVATE_VALUES = ("1", "true", "on", "triton", "scaled_mm", "fa", "flash", "b200")


def maybe_activate_from_env() -> bool:
    """Activate iff REPERCEP_FP8_ATTENTION is set to one of the reference's
    values (reference :364-388) or ``b200``."""
    if os.environ.get("REPERCEP_FP8_ATTENTION", "").lower() not in _ACTIVATE_VALUES:
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
