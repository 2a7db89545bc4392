"""The ``AttentionOp`` Protocol — the drop-in contract, mirrored from the
reference (src/repercep/attention/protocol.py:14-54).  Same members and
call signature: ``name``, ``available``, ``supports(shape, dtype)``,
``__call__(query, key, value, *, causal=False, scale=None)`` on
(batch, heads, seq, head_dim) tensors."""

from __future__ import annotations

from typing import TYPE_CHECKING, Protocol, runtime_checkable

if TYPE_CHECKING:
    import torch

    from repercep_runtime_b200.attention.types import AttentionShape
    from repercep_runtime_b200.hardware import DType


@runtime_checkable
class AttentionOp(Protocol):
    name: str

    @property
    def available(self) -> bool: ...

    def supports(self, shape: AttentionShape, dtype: DType) -> bool: ...

    def __call__(
        self,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        *,
        causal: bool = False,
        scale: float | None = None,
    ) -> torch.Tensor: ...
