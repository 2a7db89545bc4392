"""Hardware value types of the attention seam (reference: src/repercep/hardware.py:14-95),
plus the Blackwell arch.

Callers construct these objects and pass them across the AttentionOp / Backend
seams, and the reference's own selection code compares them by identity
(``arch.vendor is Vendor.NVIDIA``, src/repercep/attention/registry.py:83).  So
when the reference package (``repercep``) is importable, the reference's own
classes are used here: a ``DeviceArch`` or ``DType`` made by this package is then
the same object the reference's registry expects.  Without it (this package on
its own), local definitions with the same names, fields and enum values stand in.
Code in this package compares these values with ``==`` (never ``is``), which
holds across both sets of classes because the enums are ``StrEnum``.
"""

from __future__ import annotations

import enum
from dataclasses import dataclass

try:
    from repercep.hardware import (  # the reference's own value types
        BackendCapabilities,
        DeviceArch,
        DeviceSpec,
        DType,
        Vendor,
    )

    REFERENCE_TYPES = True
except ImportError:
    REFERENCE_TYPES = False

    class Vendor(enum.StrEnum):  # type: ignore[no-redef]
        """Compute vendor (reference: hardware.py:14-19)."""

        AMD = "amd"
        NVIDIA = "nvidia"
        INTEL = "intel"

    class DType(enum.StrEnum):  # type: ignore[no-redef]
        """Numeric types used for kernel selection (reference: hardware.py:22-30)."""

        FP32 = "fp32"
        FP16 = "fp16"
        BF16 = "bf16"
        FP8_E4M3 = "fp8_e4m3"
        FP8_E5M2 = "fp8_e5m2"
        INT8 = "int8"

    @dataclass(frozen=True, slots=True)
    class DeviceArch:  # type: ignore[no-redef]
        """A GPU architecture target (reference: hardware.py:33-47)."""

        vendor: Vendor
        gfx_id: str
        family: str

        def __str__(self) -> str:
            return f"{self.vendor.value}:{self.gfx_id}"

    @dataclass(frozen=True, slots=True)
    class DeviceSpec:  # type: ignore[no-redef]
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
    class BackendCapabilities:  # type: ignore[no-redef]
        """What a backend can do on this host (reference: hardware.py:81-95)."""

        dtypes: frozenset[DType]
        supports_flash_attention: bool
        supports_fp8: bool
        supports_torch_compile: bool
        attention_ops: tuple[str, ...]


H100 = DeviceArch(Vendor.NVIDIA, "sm90a", "Hopper")
# B200: compute capability 10.0; the kernels are built for the sm_100a target.
B200 = DeviceArch(Vendor.NVIDIA, "sm100a", "Blackwell")

# gfx_id strings that name compute capability 10.0: this package's "sm100a",
# and "100", which the reference's CUDABackend reports for a device it has no
# table entry for (src/repercep/backend/cuda.py:108-110).
B200_GFX_IDS = frozenset({"sm100a", "sm100", "sm_100a", "sm_100", "100"})


def is_b200_arch(arch: object) -> bool:
    """True for an NVIDIA compute-capability 10.0 arch, whichever class made it."""
    vendor = getattr(arch, "vendor", None)
    return vendor == "nvidia" and getattr(arch, "gfx_id", None) in B200_GFX_IDS


__all__ = [
    "B200",
    "B200_GFX_IDS",
    "H100",
    "REFERENCE_TYPES",
    "BackendCapabilities",
    "DType",
    "DeviceArch",
    "DeviceSpec",
    "Vendor",
    "is_b200_arch",
]
