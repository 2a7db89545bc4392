"""Multi-GPU execution of the FP8 attention path (one process per GPU).

Two schemes (the reference has neither: it runs on one GPU and its diffusers
bridge falls back to SDPA whenever a parallel config is set,
src/repercep/attention/diffusers_backend.py:199-212):

* **batch x head sharding** — (b, h) slices are independent; each rank takes
  a contiguous run of them and no data crosses GPUs (``shard_bh``).
* **context parallelism** (long video sequences) — every rank holds a
  contiguous slice of the sequence for Q, K and V.  It quantises its K/V
  slice to e4m3 with per-128-token-block scales, the ranks all-gather the
  e4m3 K/V (1 byte/element on the wire instead of 2) and the scales over
  NCCL, and each rank runs attention of its own queries against every
  rank's K/V chunk in one kernel launch (``ContextParallelAttention``).
  The gathers write the kernel's (rank, BH, rows, D) layout directly.
  Slices are whole 128-token blocks (the last rank takes the remainder), so
  every block and its scale are exactly those of the single-GPU per-block
  layout and the result is bit-identical to the single-GPU one.  Each rank
  owns complete query rows, so no partial outputs are exchanged.  Remote K/V
  always lands in this GPU's memory before any kernel reads it.
  The reference's own per-(b,h) scale mode spans the whole sequence: each
  rank computes the partial amax of its 128-token chunks, one all-reduce MAX
  of those (B*H x chunks integers) gives every rank the whole sequence's
  amax, and each rank quantizes its slice with the common scales -- again
  bit-identical to one GPU.

The collective is injected (``all_gather``), so the bookkeeping is testable
with gloo ranks on CPU and an oracle in place of the kernel.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

BLOCK = 128


# --------------------------------------------------------------- sharding
def shard_bh(B: int, H: int, rank: int, world: int) -> tuple[int, int]:
    """Half-open range [start, stop) of flattened (b*H + h) slices for ``rank``.

    Slices are split as evenly as possible; ranks differ by at most one.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    total = B * H
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    stop = start + base + (1 if rank < extra else 0)
    return start, stop


@dataclass(frozen=True)
class SeqShard:
    """One rank's slice of a context-parallel sequence."""

    rank: int
    world: int
    seq_len: int
    chunk_rows: int  # rows every rank's buffer holds (multiple of 128)
    start: int  # first global row owned by this rank
    rows: int  # rows actually owned (the last rank may own fewer)

    @property
    def last_rows(self) -> int:
        """Valid rows in the last rank's chunk."""
        return self.seq_len - (self.world - 1) * self.chunk_rows


def seq_shard(seq_len: int, rank: int, world: int) -> SeqShard:
    """Whole-block sequence split for context parallelism.

    Every rank but the last owns ``chunk_rows`` rows (a multiple of 128); the
    last owns the remainder.  Raises if the sequence is too short for
    ``world`` non-empty shards.
    """
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    blocks = -(-seq_len // BLOCK)
    chunk_rows = -(-blocks // world) * BLOCK
    last_rows = seq_len - (world - 1) * chunk_rows
    if last_rows <= 0:
        raise ValueError(f"sequence of {seq_len} tokens is too short for {world} shards")
    start = rank * chunk_rows
    rows = chunk_rows if rank < world - 1 else last_rows
    return SeqShard(rank, world, seq_len, chunk_rows, start, rows)


# ----------------------------------------------------- context parallelism
AllGather = Callable[["object", "object"], None]  # (output, input) -> None


# (b, h) chunks per device call: every chunk's K/V gather is issued up front
# and its attention starts as soon as that gather lands, so all gathers but
# the first run under attention.  Even splits measured on Wan (B2 H40 S75600),
# max over ranks: 8 GPUs 21.95 ms unchunked, 21.25 with 2 chunks, 21.26 with 4;
# 2 GPUs 81.15 / 80.84 / 81.98 (8 chunks).  The default plan (cp_chunk_bounds)
# makes the first chunk about one wave of CTAs, so the one gather nothing
# overlaps is small, and cuts the rest into CP_CHUNKS chunks of whole waves.
CP_CHUNKS = 2


def cp_chunk_bounds(bh: int, q_tiles: int, sms: int = 148, later: int = CP_CHUNKS) -> list[tuple[int, int]]:
    """(b, h) ranges of the overlapped context-parallel call.

    A (b, h) slice of this rank's queries is ceil(q_tiles / 2) two-tile CTAs.
    The first range holds the slices that fill one wave of ``sms`` CTAs (at
    least one), so its gather -- the only one no attention overlaps -- moves
    a small part of K/V; the rest is cut into ``later`` ranges whose sizes are
    multiples of that wave, so no launch ends on a ragged wave."""
    if bh <= 0:
        return []
    pairs = max(1, -(-q_tiles // 2))
    wave = max(1, sms // pairs)
    first = min(wave, bh)
    bounds = [(0, first)]
    rest = bh - first
    if rest > 0:
        step = -(-rest // max(1, later))
        step = -(-step // wave) * wave
        a = first
        while a < bh:
            bounds.append((a, min(bh, a + step)))
            a += step
    return bounds


def nccl_all_reduce_max(group=None):  # type: ignore[no-untyped-def]
    """In-place element-wise max over the ranks of ``group`` (the combine
    step of the per-(b,h) scale under context parallelism)."""
    import torch.distributed as dist

    def reduce(t):  # type: ignore[no-untyped-def]
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)

    return reduce


def nccl_all_gather(group=None, high_priority: bool = True) -> AllGather:  # type: ignore[no-untyped-def]
    """``torch.distributed.all_gather_into_tensor`` bound to ``group``.

    With no group and an NCCL default group, the gathers run in a new NCCL
    group over the same ranks whose streams have high priority, so the block
    scheduler gives the gather kernels SMs ahead of the next attention CTAs
    (call it on every rank, like any group creation).  The returned callable
    takes ``async_op`` and then returns the collective's work handle."""
    import datetime

    import torch.distributed as dist

    if group is None and high_priority and dist.get_backend() == "nccl":
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        group = dist.new_group(backend="nccl", pg_options=opts,
                               timeout=datetime.timedelta(minutes=2))

    def gather(out, inp, async_op: bool = False):  # type: ignore[no-untyped-def]
        return dist.all_gather_into_tensor(out, inp, group=group, async_op=async_op)

    gather.supports_async = True  # type: ignore[attr-defined]
    return gather


class ContextParallelAttention:
    """FP8 attention with the sequence split across ranks.

    ``__call__(q, k, v)`` takes this rank's (B, H, rows, D) bf16 shard (the
    rows of ``seq_shard(seq_len, rank, world)``) and returns the bf16 output
    rows for it.  ``scale_mode``: per-128-token-block scales (default, no
    collective before the gather) or the reference's per-(b,h) scales (one
    all-reduce MAX of partial amaxes through ``all_reduce_max`` first).
    """

    def __init__(
        self,
        seq_len: int,
        rank: int,
        world: int,
        all_gather: AllGather | None = None,
        p_mode: int = 0,
        scale: float | None = None,
        scale_mode: int = 1,
        all_reduce_max=None,  # type: ignore[no-untyped-def]
    ) -> None:
        if scale_mode not in (0, 1):
            raise ValueError(f"unknown scale_mode {scale_mode}")
        self.shard = seq_shard(seq_len, rank, world)
        self.all_gather = all_gather
        self.p_mode = p_mode
        self.scale = scale
        self.scale_mode = scale_mode
        self.all_reduce_max = all_reduce_max
        self._streams: dict = {}  # device index -> chunk streams (attend_quantized)
        if scale_mode == 0 and world > 1 and all_reduce_max is None:
            raise ValueError("per-(b,h) scales over several ranks need all_reduce_max")

    def quantize(self, q, k, v):  # type: ignore[no-untyped-def]
        """This rank's shards to e4m3 in the configured scale mode; per-(b,h)
        scales are those of the whole sequence (partials combined across ranks)."""
        from repercep_runtime_b200 import ops

        if self.scale_mode == 1:
            return ops.quantize_fp8((q, k, v), scale_mode=ops.SCALE_PER_BLOCK128)

        def combine(partials):  # type: ignore[no-untyped-def]
            if self.shard.world > 1:
                self.all_reduce_max(partials)

        # every rank's partial array has the same shape: chunk_rows/128 slots
        return ops.quantize_fp8_bh_phased((q, k, v), combine, npart=self.shard.chunk_rows // BLOCK)

    def gather_kv(self, k8, v8, ks, vs):  # type: ignore[no-untyped-def]
        """All-gather this rank's e4m3 K/V (BH, rows, D) and per-block scales;
        returns (n_chunks, BH, chunk_rows, D) K and V and (n_chunks, BH,
        chunk_rows/128) scales -- the chunked kernel's layout, written by the
        collectives themselves (K, V and the two scale sets as three gathers).
        Only a rank whose shard is short of chunk_rows (the last) pads its
        contribution; nothing is repacked after the gather."""
        k_all, v_all, sc_all, _ = self._gather(k8, v8, ks, vs, async_op=False)
        return k_all, v_all, sc_all[:, 0].contiguous(), sc_all[:, 1].contiguous()

    def _gather(self, k8, v8, ks, vs, async_op: bool):  # type: ignore[no-untyped-def]
        """gather_kv's three collectives; returns (K, V, scales (world, 2, BH,
        nblk), work handles).  With async_op the handles must be waited on
        before the outputs are read (their inputs stay referenced meanwhile)."""
        import torch

        sh = self.shard
        bh, rows, d = k8.shape
        nblk = sh.chunk_rows // BLOCK
        world = sh.world
        if self.all_gather is None:
            raise RuntimeError("no all_gather bound (world > 1 needs a process group)")
        dev = k8.device

        def padded(x):  # type: ignore[no-untyped-def]
            if rows == sh.chunk_rows:
                return x.reshape(bh, rows, d).contiguous()
            buf = torch.zeros((bh, sh.chunk_rows, d), dtype=torch.uint8, device=dev)
            buf[:, :rows].copy_(x.reshape(bh, rows, d))
            return buf

        k_all = torch.empty((world, bh, sh.chunk_rows, d), dtype=torch.uint8, device=dev)
        v_all = torch.empty_like(k_all)
        sc = torch.zeros((2, bh, nblk), dtype=torch.float32, device=dev)
        sc[0, :, : ks.shape[-1]].copy_(ks.reshape(bh, -1))
        sc[1, :, : vs.shape[-1]].copy_(vs.reshape(bh, -1))
        sc_all = torch.empty((world, 2, bh, nblk), dtype=torch.float32, device=dev)
        # outputs as (world * BH, rows, D): the rank-major concatenation every
        # all_gather_into_tensor backend accepts
        jobs = ((k_all.view(world * bh, sh.chunk_rows, d), padded(k8)),
                (v_all.view(world * bh, sh.chunk_rows, d), padded(v8)),
                (sc_all.view(world * 2, bh, nblk), sc))
        works = []
        for o, i in jobs:
            if async_op:
                works.append(self.all_gather(o, i, async_op=True))
            else:
                self.all_gather(o, i)
        return k_all, v_all, sc_all, works

    def _call_host(self, q, k, v):  # type: ignore[no-untyped-def]
        """Host (pinned) shards: (b, h) chunks stream through the device with
        the copies overlapped with quantise + gather + attention, two compute
        streams taking turns.  Every rank cuts the same chunks (the plan
        depends on the shared chunk_rows, not on this rank's rows), so the
        per-chunk collectives line up across ranks."""
        import torch

        from repercep_runtime_b200 import ops
        from repercep_runtime_b200.streaming import SLOTS, fp8_attention_host, plan_chunks, _streams

        sh = self.shard
        B, H, rows, D = q.shape
        if q.dtype != torch.bfloat16:
            raise ValueError("context-parallel attention takes bf16 shards")
        if sh.world == 1:
            return fp8_attention_host(q, k, v, scale=self.scale, scale_mode=self.scale_mode,
                                      p_mode=self.p_mode)
        bh = B * H
        plan = plan_chunks(bh, sh.chunk_rows)
        out = torch.empty((B, H, rows, D), dtype=q.dtype, pin_memory=True)
        q3, k3, v3 = (t.reshape(bh, rows, D) for t in (q, k, v))
        o3 = out.view(bh, rows, D)
        dev = torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(dev):
            caller = torch.cuda.current_stream(dev)
            h2d, d2h, comp = _streams(dev)
            c = plan.chunk
            slots = [
                tuple(torch.empty((c, rows, D), dtype=q.dtype, device=dev) for _ in range(4))
                for _ in range(min(SLOTS, plan.n))
            ]
            ev_in = [torch.cuda.Event() for _ in slots]
            ev_comp = [torch.cuda.Event() for _ in slots]
            ev_out = [torch.cuda.Event() for _ in slots]
            h2d.wait_stream(caller)
            for i in range(plan.n):
                s = i % len(slots)
                a, b = plan.bounds(i)
                n = b - a
                qd, kd, vd, od = slots[s]
                cs = comp[i % 2]
                with torch.cuda.stream(h2d):
                    if i >= len(slots):
                        h2d.wait_event(ev_comp[s])
                    qd[:n].copy_(q3[a:b], non_blocking=True)
                    kd[:n].copy_(k3[a:b], non_blocking=True)
                    vd[:n].copy_(v3[a:b], non_blocking=True)
                    ev_in[s].record(h2d)
                with torch.cuda.stream(cs):
                    cs.wait_event(ev_in[s])
                    if i >= len(slots):
                        cs.wait_event(ev_out[s])
                    self._device_call(qd[:n].unsqueeze(0), kd[:n].unsqueeze(0), vd[:n].unsqueeze(0),
                                      out=od[:n].unsqueeze(0), chunks=1)
                    ev_comp[s].record(cs)
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_comp[s])
                    o3[a:b].copy_(od[:n], non_blocking=True)
                    ev_out[s].record(d2h)
            d2h.synchronize()
        return out

    def __call__(self, q, k, v, out=None):  # type: ignore[no-untyped-def]
        if q.device.type == "cpu":
            if out is not None:
                raise ValueError("host shards return a new host tensor")
            return self._call_host(q, k, v)
        return self._device_call(q, k, v, out=out)

    def _device_call(self, q, k, v, out=None, chunks: int | None = None):  # type: ignore[no-untyped-def]
        import torch

        from repercep_runtime_b200 import ops

        sh = self.shard
        if q.shape[2] != sh.rows or k.shape != q.shape or v.shape != q.shape:
            raise ValueError(f"expected (B, H, {sh.rows}, D) shards for rank {sh.rank}")
        qq, kq, vq = self.quantize(q, k, v)
        if sh.world == 1:
            return ops.attention_fp8_quantized(qq, kq, vq, scale=self.scale, p_mode=self.p_mode, out=out)
        # the chunked kernel reads per-block scales; a per-(b,h) scale repeated
        # over the blocks gives the per-(b,h) arithmetic exactly
        return self.attend_quantized(ops.per_block_view(qq), ops.per_block_view(kq),
                                     ops.per_block_view(vq), out=out, chunks=chunks)

    def attend_quantized(self, qq, kq, vq, out=None, chunks: int | None = None):  # type: ignore[no-untyped-def]
        """Gather K/V and attend, for quantized (per-128-block) shards.

        When the bound all_gather is asynchronous the (b, h) range is cut into
        chunks -- ``cp_chunk_bounds``'s plan by default, or ``chunks`` even
        parts -- every chunk's gathers are issued first, and chunk i's
        attention waits only for chunk i's gathers.  Each chunk's launch goes
        on a stream of its own (after the calling stream's work and its
        gathers), and the calling stream waits for all of them at the end: a
        chunk's CTAs then take the SMs that the previous chunk's last CTAs
        free, instead of waiting for that whole launch to finish."""
        import torch

        from repercep_runtime_b200 import ops

        sh = self.shard
        B, H, rows, D = qq.data.shape
        bh = B * H
        k8 = kq.data.view(torch.uint8).reshape(bh, rows, D)
        v8 = vq.data.view(torch.uint8).reshape(bh, rows, D)
        if chunks is None:
            sms = torch.cuda.get_device_properties(qq.data.device).multi_processor_count
            bounds = self.chunk_plan(bh, sms)
        else:
            n = max(1, min(chunks, bh))
            bounds = [(i * bh // n, (i + 1) * bh // n) for i in range(n)]
        n = len(bounds) if getattr(self.all_gather, "supports_async", False) else 1
        if out is None:
            out = torch.empty((B, H, rows, D), dtype=torch.bfloat16, device=qq.data.device)
        if not out.is_contiguous():
            n = 1  # chunk views of the output need (B, H, rows, D) contiguous
        if n <= 1:
            k_all, v_all, ks_all, vs_all = self.gather_kv(k8, v8, kq.scales, vq.scales)
            return ops.attention_fp8_chunked(qq, k_all.view(ops.FP8), v_all.view(ops.FP8), ks_all,
                                             vs_all, last_rows=sh.last_rows, scale=self.scale,
                                             p_mode=self.p_mode, out=out)
        ks = kq.scales.reshape(bh, -1)
        vs = vq.scales.reshape(bh, -1)
        pending = [self._gather(k8[a:b], v8[a:b], ks[a:b], vs[a:b], async_op=True) for a, b in bounds]
        q4 = qq.data.reshape(1, bh, rows, qq.data.shape[-1])
        qs = qq.scales.reshape(bh, -1)
        o4 = out.view(1, bh, rows, D)
        caller = torch.cuda.current_stream(out.device)
        streams = self._chunk_streams(out.device, len(bounds))
        used = []
        try:
            for s, (a, b), (k_all, v_all, sc_all, works) in zip(streams, bounds, pending):
                s.wait_stream(caller)  # Q, the output and the gather buffers come from the caller's stream
                used.append(s)
                with torch.cuda.stream(s):
                    for w in works:
                        w.wait()  # this chunk's gathers, on this chunk's stream
                    qc = ops.Quantized(q4[:, a:b], qs[a:b], ops.SCALE_PER_BLOCK128, d=qq.d)
                    ops.attention_fp8_chunked(qc, k_all.view(ops.FP8), v_all.view(ops.FP8),
                                              sc_all[:, 0].contiguous(), sc_all[:, 1].contiguous(),
                                              last_rows=sh.last_rows, scale=self.scale, p_mode=self.p_mode,
                                              out=o4[:, a:b])
        finally:
            # also when a launch raised: nothing the chunk streams were given
            # may be reused by the caller's stream before they are done with it
            for s in used:
                caller.wait_stream(s)
        return out

    def chunk_plan(self, bh: int, sms: int = 148) -> list[tuple[int, int]]:
        """The (b, h) ranges of the overlapped call.  Every rank must cut the
        same ranges (each range is one set of collectives), so the plan comes
        from the shared chunk_rows, not from this rank's own row count, which
        is shorter on the last rank."""
        return cp_chunk_bounds(bh, self.shard.chunk_rows // BLOCK, sms)

    def _chunk_streams(self, device, n: int) -> list:  # type: ignore[no-untyped-def]
        """n streams of this device for the chunk launches, created once."""
        import torch

        have = self._streams.setdefault(device.index, [])
        while len(have) < n:
            have.append(torch.cuda.Stream(device=device))
        return have[:n]


__all__ = [
    "CP_CHUNKS",
    "ContextParallelAttention",
    "SeqShard",
    "cp_chunk_bounds",
    "nccl_all_gather",
    "nccl_all_reduce_max",
    "seq_shard",
    "shard_bh",
]
