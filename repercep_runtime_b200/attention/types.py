"""Attention problem descriptors (reference: src/repercep/attention/types.py:9-40).

Callers construct these to ask an op ``supports(shape, dtype)``.  When the
reference package is importable its own ``AttentionKind`` / ``AttentionShape``
are used, so shapes built by the reference's engines and by this package are
the same classes; otherwise local definitions with identical names and fields
stand in (compared with ``==``, which holds across both).
"""

from __future__ import annotations

import enum
from dataclasses import dataclass

try:
    from repercep.attention.types import AttentionKind, AttentionShape
except ImportError:

    class AttentionKind(enum.StrEnum):  # type: ignore[no-redef]
        FULL = "full"
        CAUSAL = "causal"
        NEIGHBORHOOD = "neighborhood"

    @dataclass(frozen=True, slots=True)
    class AttentionShape:  # type: ignore[no-redef]
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


__all__ = ["AttentionKind", "AttentionShape"]
