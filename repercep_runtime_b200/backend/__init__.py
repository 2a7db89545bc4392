"""Backend seam of the B200 path (mirrors src/repercep/backend)."""

from __future__ import annotations

from repercep_runtime_b200.backend.b200 import B200Backend
from repercep_runtime_b200.backend.protocol import Backend
from repercep_runtime_b200.backend.registry import available_backends, select_backend

__all__ = ["B200Backend", "Backend", "available_backends", "select_backend"]
