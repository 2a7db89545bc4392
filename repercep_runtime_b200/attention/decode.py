"""Shared-prefix candidate decode on B200.

The reference's token-VLA planner decodes N candidate action chunks that
share one prompt+observation prefix (``VLAEngine.plan``,
src/repercep/models/vla.py:229-258); its GPU pipeline expands the prompt N
times and runs HF ``generate`` with SDPA (scripts/run_vla_openvla_gpu.py:
174-186), so the prefix K/V is stored and read N times.  This op computes the
same attention with the prefix K/V held once: every query tile streams each
prefix K/V tile once, then its own candidates' causal suffix.

Semantics for candidate c, head h, new token i (0 <= i < T):
    softmax over [ prefix keys 0..P-1  ||  suffix keys of candidate c, 0..i ]
Layouts: q, suffix K/V (C*T, H, D); prefix K/V (P, H, D); bf16; out (C*T, H, D).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING

from repercep_runtime_b200.attention.fp8_b200 import b200_device_present

if TYPE_CHECKING:
    import torch

    from repercep_runtime_b200.ops import Quantized


@dataclass
class QuantizedPrefix:
    """Prefix K/V quantised once (per-128-token-block scales), reused every step."""

    k: Quantized
    v: Quantized
    length: int


def _as_bshd(x: torch.Tensor) -> torch.Tensor:
    if x.dim() != 3:
        raise ValueError("expected a (tokens, heads, head_dim) tensor")
    return x.unsqueeze(0)


class SharedPrefixFP8Decode:
    """FP8 shared-prefix candidate decode (per-128-token-block scales)."""

    name = "fp8-b200-prefix-decode"

    def __init__(self, p_mode: int = 0) -> None:
        self.p_mode = p_mode
        self._import_error: str | None = None
        try:
            from repercep_runtime_b200 import _lib

            _lib.load()
        except Exception as e:
            self._import_error = f"{type(e).__name__}: {e}"
        if self._import_error is None and not b200_device_present():
            self._import_error = "no sm_100 (B200) CUDA device visible"

    @property
    def available(self) -> bool:
        return self._import_error is None

    def supports(self, candidates: int, tokens: int, heads: int, head_dim: int) -> bool:
        return (
            self.available
            and head_dim == 128
            and tokens >= 1
            and 128 % tokens == 0
            and candidates >= 1
            and heads <= 65535
        )

    def quantize_prefix(self, k_prefix: torch.Tensor, v_prefix: torch.Tensor) -> QuantizedPrefix:
        from repercep_runtime_b200 import ops

        kq, vq = ops.quantize_fp8(
            (_as_bshd(k_prefix), _as_bshd(v_prefix)),
            scale_mode=ops.SCALE_PER_BLOCK128,
            layout="bshd",
        )
        return QuantizedPrefix(kq, vq, int(k_prefix.shape[0]))

    def __call__(
        self,
        query: torch.Tensor,
        prefix: QuantizedPrefix,
        k_suffix: torch.Tensor,
        v_suffix: torch.Tensor,
        *,
        candidates: int,
        tokens: int,
        scale: float | None = None,
        out: torch.Tensor | None = None,
    ) -> torch.Tensor:
        if self._import_error is not None:
            raise RuntimeError(f"FP8 B200 prefix decode is not available ({self._import_error})")
        from repercep_runtime_b200 import ops

        qq, kx, vx = ops.quantize_fp8(
            (_as_bshd(query), _as_bshd(k_suffix), _as_bshd(v_suffix)),
            scale_mode=ops.SCALE_PER_BLOCK128,
            layout="bshd",
        )
        return ops.prefix_decode_fp8_quantized(
            qq,
            prefix.k,
            prefix.v,
            kx,
            vx,
            candidates=candidates,
            tokens=tokens,
            scale=scale,
            p_mode=self.p_mode,
            out=out,
        )


__all__ = ["QuantizedPrefix", "SharedPrefixFP8Decode"]
