"""Attention op selection (reference: src/repercep/attention/registry.py:65-132).

Same rules: a vendor-branched candidate list, FP8 ops only when the
``REPERCEP_FP8_ATTENTION`` environment variable enables them (read once at
import, as the reference does at :37-39), the first op whose ``supports()``
accepts the problem wins, ``NaiveAttention`` is the floor.  The NVIDIA branch
puts the B200 op first on sm_100 devices; any other arch keeps the floor (the
reference's Hopper/AMD ops are outside this package).
"""

from __future__ import annotations

import os
from typing import TYPE_CHECKING

from repercep_runtime_b200.attention.fp8_b200 import B200FP8Attention
from repercep_runtime_b200.attention.naive import NaiveAttention
from repercep_runtime_b200.hardware import DeviceArch, DType, Vendor

if TYPE_CHECKING:
    from repercep_runtime_b200.attention.protocol import AttentionOp
    from repercep_runtime_b200.attention.types import AttentionShape

_FP8_ENV = os.environ.get("REPERCEP_FP8_ATTENTION", "").lower()
# The reference's truthy set (:38) plus "b200" to pin this op explicitly.
_FP8_TRUTHY = ("1", "true", "on", "triton", "b200")
_FP8_ENABLED = _FP8_ENV in _FP8_TRUTHY


def select_attention_op(arch: DeviceArch, shape: AttentionShape, dtype: DType) -> AttentionOp:
    """Pick the fastest op that supports ``(shape, dtype)`` on ``arch``."""
    candidates: list[AttentionOp] = []
    if arch.vendor is Vendor.NVIDIA and arch.gfx_id.startswith("sm100") and _FP8_ENABLED:
        candidates.append(B200FP8Attention())
    candidates.append(NaiveAttention())
    for op in candidates:
        if op.supports(shape, dtype):
            return op
    return NaiveAttention()
