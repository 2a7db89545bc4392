"""FP8 flash-attention on B200 — the AttentionOp that replaces the reference's
``FP8HopperTritonAttention`` (src/repercep/attention/fp8_hopper_triton.py:52-121).

Same contract: ``name``, ``available`` (never raises; a load failure is kept
as a string), ``supports(shape, dtype)``, and ``__call__`` on
(batch, heads, seq, head_dim) bf16 / fp16 tensors (head_dim 32, 64, 128 or 256)
returning the query's dtype;
calling it while unavailable raises ``RuntimeError`` (reference :114-119).

The call runs two native launches through librepercep_b200.so: one quantize of
Q, K and V together, one tcgen05 attention kernel.  There is no fallback
inside the op — the registry's ``supports()`` chain is where fallback lives.
Host (CPU) bf16 tensors are also accepted: the call then streams (b, h) chunks
through the device with copies overlapped with compute
(``repercep_runtime_b200.streaming``) and returns a host tensor.

Environment switches (read per instance):
  REPERCEP_B200_SCALE_MODE  ``bh`` (default; the reference's per-(b,h) amax) or
                            ``block128`` (one scale per 128-token block)
  REPERCEP_B200_P_MODE      ``e4m3`` (default; P rounded once to e4m3 as the
                            reference does) or ``hilo`` (two-plane P)
"""

from __future__ import annotations

import os
from typing import TYPE_CHECKING

from repercep_runtime_b200.attention.types import AttentionKind, AttentionShape
from repercep_runtime_b200.hardware import DType

if TYPE_CHECKING:
    import torch

_SUPPORTED_HEAD_DIMS = frozenset({32, 64, 128, 256})  # as fp8_hopper_triton.py:41
_SUPPORTED_KINDS = frozenset({AttentionKind.FULL, AttentionKind.CAUSAL})

_SCALE_MODES = {"bh": 0, "per_bh": 0, "block128": 1, "block": 1, "per_block128": 1}
_P_MODES = {"e4m3": 0, "hilo": 1, "e4m3_hilo": 1}


def _env_choice(var: str, table: dict[str, int], default: str) -> int:
    raw = os.environ.get(var, default).strip().lower()
    if raw not in table:
        raise ValueError(f"{var}={raw!r}; expected one of {sorted(table)}")
    return table[raw]


def b200_device_present() -> bool:
    """True when torch sees at least one compute-capability 10.0 device."""
    try:
        import torch

        if not torch.cuda.is_available():
            return False
        return any(
            torch.cuda.get_device_capability(i) == (10, 0) for i in range(torch.cuda.device_count())
        )
    except Exception:
        return False


class B200FP8Attention:
    """FP8 (e4m3) fused attention on sm_100a tcgen05 tensor cores."""

    name = "fp8-b200-flash"

    def __init__(self, scale_mode: int | None = None, p_mode: int | None = None) -> None:
        self.scale_mode = (
            scale_mode
            if scale_mode is not None
            else _env_choice("REPERCEP_B200_SCALE_MODE", _SCALE_MODES, "bh")
        )
        self.p_mode = (
            p_mode if p_mode is not None else _env_choice("REPERCEP_B200_P_MODE", _P_MODES, "e4m3")
        )
        self._import_error: str | None = None
        try:
            from repercep_runtime_b200 import _lib

            _lib.load()
        except Exception as e:  # library missing or unloadable
            self._import_error = f"{type(e).__name__}: {e}"
        if self._import_error is None and not b200_device_present():
            self._import_error = "no sm_100 (B200) CUDA device visible"

    @property
    def available(self) -> bool:
        return self._import_error is None

    @property
    def unavailable_reason(self) -> str | None:
        return self._import_error

    def supports(self, shape: AttentionShape, dtype: DType) -> bool:
        # Compared by value: ``shape`` and ``dtype`` may be the reference's own
        # classes or this package's stand-ins (StrEnum members equal their strings).
        return (
            self.available
            and dtype in (DType.BF16, DType.FP16)
            and shape.head_dim in _SUPPORTED_HEAD_DIMS
            and shape.kind in _SUPPORTED_KINDS
            and shape.seq_len_q >= 1
            and shape.seq_len_kv >= 1
            and shape.batch * shape.heads <= 65535
            # the causal mask is top-left aligned like the reference's, which
            # only means "causal" for self-attention
            and (shape.kind == AttentionKind.FULL or shape.is_self_attention)
        )

    def __call__(
        self,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        *,
        causal: bool = False,
        scale: float | None = None,
    ) -> torch.Tensor:
        if self._import_error is not None:
            raise RuntimeError(
                f"FP8 B200 attention is not available ({self._import_error}). "
                "Fall back to attention_backend='naive-sdpa'."
            )
        if query.device.type == "cpu":
            # Host tensors: copies pipelined with compute, host result returned.
            from repercep_runtime_b200.streaming import fp8_attention_host

            return fp8_attention_host(
                query, key, value, causal=causal, scale=scale, scale_mode=self.scale_mode,
                p_mode=self.p_mode,
            )
        from repercep_runtime_b200 import ops

        return ops.fp8_attention(
            query, key, value, causal=causal, scale=scale, scale_mode=self.scale_mode,
            p_mode=self.p_mode,
        )


__all__ = ["B200FP8Attention", "b200_device_present"]
