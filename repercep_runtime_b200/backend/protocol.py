"""The ``Backend`` Protocol, mirrored from the reference
(src/repercep/backend/protocol.py:15-52): the same members, so a B200 backend
slots into code written against the reference's seam."""

from __future__ import annotations

from typing import TYPE_CHECKING, Protocol, runtime_checkable

if TYPE_CHECKING:
    import torch

    from repercep_runtime_b200.attention.protocol import AttentionOp
    from repercep_runtime_b200.attention.types import AttentionShape
    from repercep_runtime_b200.hardware import BackendCapabilities, DeviceSpec, DType, Vendor


@runtime_checkable
class Backend(Protocol):
    vendor: Vendor
    name: str

    def is_available(self) -> bool: ...

    def devices(self) -> tuple[DeviceSpec, ...]: ...

    def capabilities(self) -> BackendCapabilities: ...

    def torch_device(self, index: int = 0) -> torch.device: ...

    def default_dtype(self) -> DType: ...

    def attention_op(self, shape: AttentionShape, dtype: DType) -> AttentionOp: ...
