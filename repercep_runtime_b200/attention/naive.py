"""The SDPA floor op (reference: src/repercep/attention/naive.py:19-43).

Kept because the selection contract ends in it: when the B200 op's
``supports()`` declines a shape, the registry returns this op, exactly as the
reference's registry does (registry.py:127-132)."""

from __future__ import annotations

from typing import TYPE_CHECKING

if TYPE_CHECKING:
    import torch

    from repercep_runtime_b200.attention.types import AttentionShape
    from repercep_runtime_b200.hardware import DType


class NaiveAttention:
    name = "naive-sdpa"
    available = True

    def supports(self, shape: AttentionShape, dtype: DType) -> bool:
        return True

    def __call__(
        self,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        *,
        causal: bool = False,
        scale: float | None = None,
    ) -> torch.Tensor:
        from torch.nn.functional import scaled_dot_product_attention

        return scaled_dot_product_attention(query, key, value, is_causal=causal, scale=scale)
