"""Attention seam of the B200 path (mirrors src/repercep/attention)."""

from __future__ import annotations

from repercep_runtime_b200.attention import diffusers_backend as _diffusers_backend  # noqa: F401
from repercep_runtime_b200.attention.decode import QuantizedPrefix, SharedPrefixFP8Decode
from repercep_runtime_b200.attention.fp8_b200 import B200FP8Attention
from repercep_runtime_b200.attention.naive import NaiveAttention
from repercep_runtime_b200.attention.protocol import AttentionOp
from repercep_runtime_b200.attention.registry import select_attention_op
from repercep_runtime_b200.attention.types import AttentionKind, AttentionShape

__all__ = [
    "AttentionKind",
    "AttentionOp",
    "AttentionShape",
    "B200FP8Attention",
    "NaiveAttention",
    "QuantizedPrefix",
    "SharedPrefixFP8Decode",
    "select_attention_op",
]
