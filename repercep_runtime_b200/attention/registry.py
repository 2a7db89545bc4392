"""Attention op selection (reference: src/repercep/attention/registry.py:65-132).

Same rules as the reference: FP8 ops only when the ``REPERCEP_FP8_ATTENTION``
environment variable enables them (read once at import, as the reference
does at :37-39), the first op whose ``supports()`` accepts the problem wins.
On a compute-capability 10.0 arch the B200 op is the first candidate.  When it
declines (or the arch is another one), selection continues with the
reference's own chain if the reference package is importable (its flash and
SDPA ops), else with the SDPA floor ``NaiveAttention``.
"""

from __future__ import annotations

import os
from typing import TYPE_CHECKING

from repercep_runtime_b200.attention.fp8_b200 import B200FP8Attention
from repercep_runtime_b200.attention.naive import NaiveAttention
from repercep_runtime_b200.hardware import is_b200_arch

if TYPE_CHECKING:
    from collections.abc import Callable

    from repercep_runtime_b200.attention.protocol import AttentionOp
    from repercep_runtime_b200.attention.types import AttentionShape
    from repercep_runtime_b200.hardware import DeviceArch, DType

_FP8_ENV = os.environ.get("REPERCEP_FP8_ATTENTION", "").lower()
# The values of the reference's set (:38) that ask for the runtime's own FP8
# kernel on NVIDIA ("1/true/on" auto-pick, "triton" the Repercep-owned kernel),
# plus "b200" to pin this op.  "te"/"transformer_engine" and the AMD-only
# "scaled_mm" ask for other ops and leave this one out, as the reference's
# NVIDIA branch leaves its Triton op out for them (:97).
_FP8_TRUTHY = ("1", "true", "on", "triton", "b200")
_FP8_ENABLED = _FP8_ENV in _FP8_TRUTHY


def fp8_enabled() -> bool:
    """Whether the environment (read at import) enables the B200 FP8 op."""
    return _FP8_ENABLED


def reference_select() -> Callable[..., AttentionOp] | None:
    """The reference's own ``select_attention_op`` (unwrapped), if importable."""
    try:
        from repercep.attention import registry as ref_registry
    except ImportError:
        return None
    fn = ref_registry.select_attention_op
    return getattr(fn, "__wrapped__", fn)


def b200_candidate(arch: DeviceArch, shape: AttentionShape, dtype: DType) -> AttentionOp | None:
    """The B200 op when ``arch`` is compute capability 10.0, FP8 is enabled and
    the op accepts ``(shape, dtype)``; else None."""
    if not (_FP8_ENABLED and is_b200_arch(arch)):
        return None
    op = B200FP8Attention()
    return op if op.supports(shape, dtype) else None


def select_attention_op(arch: DeviceArch, shape: AttentionShape, dtype: DType) -> AttentionOp:
    """Pick the fastest op that supports ``(shape, dtype)`` on ``arch``."""
    op = b200_candidate(arch, shape, dtype)
    if op is not None:
        return op
    ref = reference_select()
    if ref is not None:
        return ref(arch, shape, dtype)
    return NaiveAttention()
