"""Attention problem descriptors, mirrored from the reference
(src/repercep/attention/types.py:9-40); identical names and fields because
callers construct them to ask an op ``supports(shape, dtype)``."""

from __future__ import annotations

import enum
from dataclasses import dataclass


class AttentionKind(enum.StrEnum):
    FULL = "full"
    CAUSAL = "causal"
    NEIGHBORHOOD = "neighborhood"


@dataclass(frozen=True, slots=True)
class AttentionShape:
    """One attention call; layout convention (batch, heads, seq, head_dim)."""

    batch: int
    heads: int
    seq_len_q: int
    seq_len_kv: int
    head_dim: int
    kind: AttentionKind = AttentionKind.FULL

    @property
    def is_self_attention(self) -> bool:
        return self.seq_len_q == self.seq_len_kv
