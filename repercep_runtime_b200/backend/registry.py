"""Backend discovery (reference: src/repercep/backend/registry.py:22-57).

Same functions and error behaviour; the list holds the B200 backend.  In the
reference's own list the B200 backend goes in front of ``CUDABackend``
(``repercep_runtime_b200.integration.install`` puts it there at run time).
"""

from __future__ import annotations

from typing import TYPE_CHECKING

from repercep_runtime_b200.backend.b200 import B200Backend

if TYPE_CHECKING:
    from repercep_runtime_b200.backend.protocol import Backend

_ALL_BACKENDS: tuple[Backend, ...] = (B200Backend(),)


def available_backends() -> tuple[Backend, ...]:
    return tuple(b for b in _ALL_BACKENDS if b.is_available())


def select_backend(prefer: str | None = None) -> Backend:
    """First available backend, or the one named ``prefer``.

    Raises ValueError for an unknown name, RuntimeError when unavailable.
    """
    if prefer is not None:
        for backend in _ALL_BACKENDS:
            if backend.name == prefer:
                if not backend.is_available():
                    raise RuntimeError(f"backend {prefer!r} is not available on this host")
                return backend
        known = ", ".join(b.name for b in _ALL_BACKENDS)
        raise ValueError(f"unknown backend {prefer!r}; known backends: {known}")
    for backend in _ALL_BACKENDS:
        if backend.is_available():
            return backend
    raise RuntimeError("no repercep B200 backend is available (no sm_100 GPU visible)")
