"""The B200 CUDA backend.

Closes the gaps the reference's ``CUDABackend`` has on Blackwell
(src/repercep/backend/cuda.py): sm_100 maps to a known arch instead of
``DeviceArch(NVIDIA, "100", "unknown")`` (:108-110), FP8 is advertised
(the reference only does so for sm90/sm89, :164-169), and ``attention_op``
routes through a registry whose NVIDIA branch knows the B200 op.
Placed ahead of the reference's CUDA backend in its backend list
(``repercep_runtime_b200.integration.install`` does so at run time), it
claims only hosts with a compute-capability 10.0 device.  Its value types are
the reference's own classes whenever the reference package is importable.
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from repercep_runtime_b200.attention.registry import select_attention_op
from repercep_runtime_b200.hardware import (
    B200,
    BackendCapabilities,
    DeviceArch,
    DeviceSpec,
    DType,
    Vendor,
    is_b200_arch,
)

if TYPE_CHECKING:
    import torch

    from repercep_runtime_b200.attention.protocol import AttentionOp
    from repercep_runtime_b200.attention.types import AttentionShape


def arch_for_capability(major: int, minor: int) -> DeviceArch:
    if (major, minor) == (10, 0):
        return B200
    return DeviceArch(Vendor.NVIDIA, f"{major}{minor}", "unknown")


class B200Backend:
    vendor: Vendor = Vendor.NVIDIA
    name: str = "cuda-b200"

    def is_available(self) -> bool:
        try:
            import torch
        except ImportError:
            return False
        if torch.version.cuda is None or torch.version.hip or not torch.cuda.is_available():
            return False
        return any(is_b200_arch(d.arch) for d in self.devices())

    def devices(self) -> tuple[DeviceSpec, ...]:
        import torch

        specs: list[DeviceSpec] = []
        if not torch.cuda.is_available():
            return ()
        for i in range(torch.cuda.device_count()):
            props = torch.cuda.get_device_properties(i)
            specs.append(
                DeviceSpec(
                    index=i,
                    arch=arch_for_capability(props.major, props.minor),
                    name=props.name,
                    total_memory_bytes=props.total_memory,
                    multi_processor_count=props.multi_processor_count,
                )
            )
        return tuple(specs)

    def capabilities(self) -> BackendCapabilities:
        from repercep_runtime_b200.attention.fp8_b200 import B200FP8Attention

        ops: list[str] = []
        if B200FP8Attention().available:
            ops.append(B200FP8Attention.name)
        ops.append("naive-sdpa")
        has_b200 = any(is_b200_arch(d.arch) for d in self.devices())
        dtypes = {DType.FP32, DType.FP16, DType.BF16, DType.INT8}
        if has_b200:
            dtypes |= {DType.FP8_E4M3, DType.FP8_E5M2}
        return BackendCapabilities(
            dtypes=frozenset(dtypes),
            supports_flash_attention=False,
            supports_fp8=has_b200,
            supports_torch_compile=True,
            attention_ops=tuple(ops),
        )

    def torch_device(self, index: int = 0) -> torch.device:
        import torch

        return torch.device("cuda", index)

    def default_dtype(self) -> DType:
        return DType.BF16

    def attention_op(self, shape: AttentionShape, dtype: DType) -> AttentionOp:
        devices = self.devices()
        arch = B200 if not devices else devices[0].arch
        return select_attention_op(arch, shape, dtype)
