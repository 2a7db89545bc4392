"""Bind the B200 path into a running copy of the reference runtime.

The reference (``repercep``) picks its compute path in three places; each one
gets the B200 path here, at run time, with the same effect as the source
patch a maintainer would add to the reference tree:

1. **Backend list** (src/repercep/backend/registry.py:22).  ``B200Backend`` is
   inserted in front of ``CUDABackend``, so ``select_backend()`` returns it on a
   host with a compute-capability 10.0 GPU (it claims no other host).  Its
   ``attention_op`` puts the B200 FP8 op first and otherwise defers to the
   reference's own chain.
2. **Attention op selection** (src/repercep/attention/registry.py:65-132).
   ``select_attention_op`` is wrapped: for a compute-capability 10.0 arch (the
   reference's ``CUDABackend`` reports gfx_id ``"100"`` for it,
   src/repercep/backend/cuda.py:108-110) with FP8 enabled, the B200 op is tried
   first; everything else goes to the reference's function unchanged.  The
   wrapper replaces the name in every loaded ``repercep`` module that imported it.
3. **diffusers dispatch** (src/repercep/attention/diffusers_backend.py:160-388),
   the seam Cosmos (models/cosmos.py:168-170) and Wan (attention/wan_processor.py:38-95)
   go through.  The ``"repercep_fp8"`` entry of diffusers' registry is taken
   over by this package's backend function (strided BSHD, no permute copies),
   which hands calls it cannot serve back to the function it replaced; and the
   reference's own function gets the B200 op as its cached op (``_op``, :238-248)
   when a B200 is present, so a caller holding it directly reaches the B200
   kernel too.

Everything is idempotent; ``install()`` returns what it did.  With no reference
package importable it does nothing and says so.
"""

from __future__ import annotations

import functools
import sys
from typing import Any


def _install_backend() -> str:
    from repercep.backend import registry as breg

    from repercep_runtime_b200.backend.b200 import B200Backend

    current = tuple(breg._ALL_BACKENDS)
    if any(isinstance(b, B200Backend) for b in current):
        return "present"
    names = [getattr(b, "name", "") for b in current]
    at = names.index("cuda") if "cuda" in names else 0
    breg._ALL_BACKENDS = (*current[:at], B200Backend(), *current[at:])
    return f"inserted at {at}"


def _install_select() -> str:
    from repercep.attention import registry as areg

    from repercep_runtime_b200.attention.registry import b200_candidate

    orig = areg.select_attention_op
    if getattr(orig, "_repercep_b200", False):
        return "present"

    @functools.wraps(orig)
    def select_attention_op(arch, shape, dtype):  # type: ignore[no-untyped-def]
        op = b200_candidate(arch, shape, dtype)
        return op if op is not None else orig(arch, shape, dtype)

    select_attention_op._repercep_b200 = True  # type: ignore[attr-defined]
    patched = []
    for name, mod in list(sys.modules.items()):
        if (name == "repercep" or name.startswith("repercep.")) and getattr(
            mod, "select_attention_op", None
        ) is orig:
            mod.select_attention_op = select_attention_op  # type: ignore[attr-defined]
            patched.append(name)
    return "wrapped in " + ", ".join(sorted(patched))


def _install_diffusers() -> str:
    from repercep_runtime_b200.attention import diffusers_backend as ours
    from repercep_runtime_b200.attention.fp8_b200 import B200FP8Attention

    notes = []
    try:
        from repercep.attention import diffusers_backend as ref_bridge

        op = B200FP8Attention()
        if op.available:
            ref_bridge._repercep_fp8_attention._op = op  # type: ignore[attr-defined]
            notes.append("reference bridge op = B200")
    except ImportError:
        pass
    try:
        ours.register_repercep_fp8_backend()
        notes.append("diffusers 'repercep_fp8' -> B200 bridge")
    except ImportError:
        notes.append("diffusers not installed")
    return "; ".join(notes)


def install(*, backend: bool = True, attention: bool = True, diffusers: bool = True) -> dict[str, Any]:
    """Bind the B200 backend, op and diffusers backend into the reference runtime."""
    try:
        import repercep  # noqa: F401
    except ImportError:
        return {"reference": "not importable; nothing to bind"}
    done: dict[str, Any] = {"reference": "bound"}
    if backend:
        done["backend"] = _install_backend()
    if attention:
        done["attention"] = _install_select()
    if diffusers:
        done["diffusers"] = _install_diffusers()
    return done


__all__ = ["install"]
