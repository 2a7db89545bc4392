"""FP8 attention on host (CPU) tensors, with the copies hidden behind compute.

The reference's ops take device tensors; a caller whose Q, K, V live in host
memory (offloaded activations, a CPU-side pipeline) would copy them over,
run the op and copy the output back, each stage waiting for the previous
one.  Here the (batch x head) slices -- independent under both scale modes,
since every scale belongs to one (b, h) -- are cut into chunks that flow
through a three-slot device ring:

    H2D stream       copy chunk i's Q, K, V into slot i % 3
    compute streams  quantise + attention of chunk i (two streams taking
                     turns, so one chunk's last wave overlaps the next)
    D2H stream       copy chunk i's output back into the host result

Slot reuse is ordered by events (inputs after the compute of the chunk three
back, output after its copy-out).  The result is bit-identical to the device
path: the same kernels see the same (b, h) slices.  The call returns when the
host result is complete.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from repercep_runtime_b200 import ops

SLOTS = 3
TARGET_CHUNKS = 64  # small enough to hide the first copy-in and last copy-out (Cosmos, 64
# slices: 1-slice chunks 75.0 ms per call against 75.8 with 2 and 77.5 with 4)
MIN_CTAS = 148  # one CTA per SM: a chunk should at least fill the GPU once

# One set of streams per device for the life of the process: the caching
# allocator keeps freed blocks per stream, so fresh streams on every call
# would never reuse the previous call's buffers.
_STREAMS: dict[int, tuple[torch.cuda.Stream, torch.cuda.Stream, tuple[torch.cuda.Stream, ...]]] = {}


def _streams(dev: torch.device):  # type: ignore[no-untyped-def]
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _STREAMS:
        _STREAMS[idx] = (
            torch.cuda.Stream(dev),
            torch.cuda.Stream(dev),
            (torch.cuda.Stream(dev), torch.cuda.Stream(dev)),
        )
    return _STREAMS[idx]


@dataclass(frozen=True)
class ChunkPlan:
    """How the B*H slices are cut: ``chunk`` slices per chunk, ``n`` chunks."""

    bh: int
    chunk: int

    @property
    def n(self) -> int:
        return -(-self.bh // self.chunk)

    def bounds(self, i: int) -> tuple[int, int]:
        a = i * self.chunk
        return a, min(self.bh, a + self.chunk)


def plan_chunks(bh: int, seq_q: int, target_chunks: int = TARGET_CHUNKS) -> ChunkPlan:
    """Chunk size for ``bh`` slices of ``seq_q`` query rows: about
    ``target_chunks`` chunks, but never fewer slices than fill every SM once
    (the attention kernel runs ceil(seq_q / 256) CTAs per slice)."""
    if bh < 1 or seq_q < 1:
        raise ValueError("empty attention problem")
    ctas_per_slice = -(-seq_q // 256)
    by_count = -(-bh // target_chunks)
    by_fill = -(-MIN_CTAS // ctas_per_slice)
    return ChunkPlan(bh, max(1, min(bh, max(by_count, by_fill))))


def fp8_attention_host(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    *,
    causal: bool = False,
    scale: float | None = None,
    scale_mode: int = ops.SCALE_PER_BH,
    p_mode: int = ops.P_E4M3,
    device: torch.device | int | None = None,
    out: torch.Tensor | None = None,
    plan: ChunkPlan | None = None,
) -> torch.Tensor:
    """FP8 attention of host bf16 / fp16 (B, H, S, D) tensors; returns a host
    (B, H, Sq, D) tensor of the same dtype (pinned unless ``out`` is given).  Inputs should be
    pinned for the copies to overlap; pageable inputs still work, serially."""
    for name, t in (("query", query), ("key", key), ("value", value)):
        if t.device.type != "cpu":
            raise ValueError(f"{name} must be a host tensor (got {t.device})")
        if t.dtype not in (torch.bfloat16, torch.float16) or t.dim() != 4:
            raise ValueError(f"{name} must be a 4-D bf16 or fp16 tensor (B, H, S, D)")
    dtype = query.dtype
    if key.dtype != dtype or value.dtype != dtype:
        raise ValueError("query, key, value must share a dtype")
    B, H, Sq, D = query.shape
    Skv = key.shape[2]
    if key.shape != value.shape or key.shape[:2] != (B, H) or key.shape[3] != D:
        raise ValueError("query, key, value shapes are inconsistent")
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        dev = torch.device("cuda", device)
    else:
        dev = torch.device(device)
    if out is None:
        out = torch.empty((B, H, Sq, D), dtype=dtype, pin_memory=True)
    elif out.shape != (B, H, Sq, D) or out.dtype != dtype or out.device.type != "cpu":
        raise ValueError("out must be a host (B, H, Sq, D) tensor of the query's dtype")
    bh = B * H
    plan = plan or plan_chunks(bh, Sq)
    q3 = query.reshape(bh, Sq, D)
    k3 = key.reshape(bh, Skv, D)
    v3 = value.reshape(bh, Skv, D)
    o3 = out.view(bh, Sq, D)

    with torch.cuda.device(dev):
        caller = torch.cuda.current_stream(dev)
        h2d, d2h, comp = _streams(dev)
        c = plan.chunk
        slots = [
            (
                torch.empty((c, Sq, D), dtype=dtype, device=dev),
                torch.empty((c, Skv, D), dtype=dtype, device=dev),
                torch.empty((c, Skv, D), dtype=dtype, device=dev),
                torch.empty((c, Sq, D), dtype=dtype, device=dev),
            )
            for _ in range(min(SLOTS, plan.n))
        ]
        ev_in = [torch.cuda.Event() for _ in slots]
        ev_comp = [torch.cuda.Event() for _ in slots]
        ev_out = [torch.cuda.Event() for _ in slots]
        h2d.wait_stream(caller)  # inputs may have been written by earlier stream work
        for i in range(plan.n):
            s = i % len(slots)
            a, b = plan.bounds(i)
            n = b - a
            qd, kd, vd, od = slots[s]
            cs = comp[i % 2]
            with torch.cuda.stream(h2d):
                if i >= len(slots):
                    h2d.wait_event(ev_comp[s])  # slot inputs consumed
                qd[:n].copy_(q3[a:b], non_blocking=True)
                kd[:n].copy_(k3[a:b], non_blocking=True)
                vd[:n].copy_(v3[a:b], non_blocking=True)
                ev_in[s].record(h2d)
            with torch.cuda.stream(cs):
                cs.wait_event(ev_in[s])
                if i >= len(slots):
                    cs.wait_event(ev_out[s])  # slot output copied out
                ops.fp8_attention(
                    qd[:n].unsqueeze(0), kd[:n].unsqueeze(0), vd[:n].unsqueeze(0),
                    causal=causal, scale=scale, scale_mode=scale_mode, p_mode=p_mode,
                    out=od[:n].unsqueeze(0),
                )
                ev_comp[s].record(cs)
            with torch.cuda.stream(d2h):
                d2h.wait_event(ev_comp[s])
                o3[a:b].copy_(od[:n], non_blocking=True)
                ev_out[s].record(d2h)
        d2h.synchronize()
    return out


__all__ = ["ChunkPlan", "fp8_attention_host", "plan_chunks"]
