"""Hardware value types, mirrored from the reference (src/repercep/hardware.py:14-95)
so signatures on the attention path read the same, plus the Blackwell arch.

Field names, enum values and class names are kept identical to the
reference's on purpose: callers pass these objects across the AttentionOp /
Backend seams, so a different spelling would break the drop-in.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass


class Vendor(enum.StrEnum):
    """Compute vendor (reference: hardware.py:14-19)."""

    AMD = "amd"
    NVIDIA = "nvidia"
    INTEL = "intel"


class DType(enum.StrEnum):
    """Numeric types used for kernel selection (reference: hardware.py:22-30)."""

    FP32 = "fp32"
    FP16 = "fp16"
    BF16 = "bf16"
    FP8_E4M3 = "fp8_e4m3"
    FP8_E5M2 = "fp8_e5m2"
    INT8 = "int8"


@dataclass(frozen=True, slots=True)
class DeviceArch:
    """A GPU architecture target (reference: hardware.py:33-47)."""

    vendor: Vendor
    gfx_id: str
    family: str

    def __str__(self) -> str:
        return f"{self.vendor.value}:{self.gfx_id}"


H100 = DeviceArch(Vendor.NVIDIA, "sm90a", "Hopper")
# B200: compute capability 10.0; the kernels are built for the sm_100a target.
B200 = DeviceArch(Vendor.NVIDIA, "sm100a", "Blackwell")


@dataclass(frozen=True, slots=True)
class DeviceSpec:
    """A concrete accelerator (reference: hardware.py:66-78)."""

    index: int
    arch: DeviceArch
    name: str
    total_memory_bytes: int
    multi_processor_count: int

    @property
    def total_memory_gib(self) -> float:
        return self.total_memory_bytes / (1024**3)


@dataclass(frozen=True, slots=True)
class BackendCapabilities:
    """What a backend can do on this host (reference: hardware.py:81-95)."""

    dtypes: frozenset[DType]
    supports_flash_attention: bool
    supports_fp8: bool
    supports_torch_compile: bool
    attention_ops: tuple[str, ...]
