"""Context-parallel attention on the GPU.

With P ranks emulated on one GPU: each rank's e4m3 K/V chunk and scales are
stacked as the all-gather would deliver them, and the chunked kernel runs each
rank's queries against them.  Because shards are whole 128-token blocks, the
result must equal the single-GPU per-block result bit for bit.  The
reference's per-(b,h) scale mode is checked the same way (partial maxima
combined across the emulated ranks first).  With two or more GPUs, both
checks run over NCCL with one process per GPU.
"""

from __future__ import annotations

import os
import socket
import threading

import pytest
import torch

from helpers import gen_bf16

pytestmark = pytest.mark.gpu


def _single(q, k, v):
    from repercep_runtime_b200 import ops

    return ops.fp8_attention(q, k, v, scale_mode=ops.SCALE_PER_BLOCK128)


@pytest.mark.parametrize("S,world", [(1000, 3), (75600 // 16, 4), (384, 3), (129, 2)])
def test_chunked_kernel_equals_single_gpu(S, world):
    from repercep_runtime_b200 import ops
    from repercep_runtime_b200.parallel import seq_shard

    B, H, D = 1, 4, 128
    q, k, v = (gen_bf16((B, H, S, D), "n05", 60 + i).cuda() for i in range(3))
    ref = _single(q, k, v)
    shards = [seq_shard(S, r, world) for r in range(world)]
    ch = shards[0].chunk_rows
    nblk = ch // 128
    k_all = torch.zeros((world, B * H, ch, D), dtype=torch.uint8, device="cuda")
    v_all = torch.zeros_like(k_all)
    ks_all = torch.zeros((world, B * H, nblk), dtype=torch.float32, device="cuda")
    vs_all = torch.zeros_like(ks_all)
    qs = []
    for r, sh in enumerate(shards):
        sl = slice(sh.start, sh.start + sh.rows)
        qq, kq, vq = ops.quantize_fp8((q[:, :, sl], k[:, :, sl], v[:, :, sl]), scale_mode=ops.SCALE_PER_BLOCK128)
        k_all[r, :, : sh.rows] = kq.data.view(torch.uint8).reshape(B * H, sh.rows, D)
        v_all[r, :, : sh.rows] = vq.data.view(torch.uint8).reshape(B * H, sh.rows, D)
        ks_all[r, :, : kq.scales.shape[1]] = kq.scales
        vs_all[r, :, : vq.scales.shape[1]] = vq.scales
        qs.append(qq)
    for r, sh in enumerate(shards):
        out = ops.attention_fp8_chunked(
            qs[r], k_all.view(ops.FP8), v_all.view(ops.FP8), ks_all, vs_all, last_rows=shards[0].last_rows
        )
        torch.cuda.synchronize()
        assert torch.equal(out, ref[:, :, sh.start : sh.start + sh.rows]), f"rank {r}"


@pytest.mark.parametrize("S,npart_extra", [(1000, 0), (333, 3), (4096, 1)])
def test_phased_per_bh_quantize_equals_one_shot(S, npart_extra):
    """The two phases with nothing combined in between (and spare zero
    slots) give quantize_fp8's per-(b,h) bytes and scales."""
    from repercep_runtime_b200 import ops

    xs = [gen_bf16((2, 3, S, 128), "n1_outlier", 90 + i).cuda() for i in range(3)]
    ref = ops.quantize_fp8(xs, scale_mode=ops.SCALE_PER_BH)
    got = ops.quantize_fp8_bh_phased(xs, lambda part: None, npart=-(-S // 128) + npart_extra)
    torch.cuda.synchronize()
    for r, g in zip(ref, got):
        assert torch.equal(r.data.view(torch.uint8), g.data.view(torch.uint8))
        assert torch.equal(r.scales, g.scales)


@pytest.mark.parametrize("S,world", [(1000, 3), (75600 // 16, 4), (300, 2)])
def test_per_bh_context_parallel_emulated(S, world):
    """The reference's per-(b,h) scales under context parallelism, P ranks
    emulated on one GPU: every rank's partial maxima (chunk_rows/128 slots),
    an element-wise max over the ranks (the all-reduce), each rank's slice
    quantized with the common scales and attended against the stacked K/V.
    Bytes, scales and outputs equal the single-GPU per-(b,h) ones."""
    from repercep_runtime_b200 import ops
    from repercep_runtime_b200.parallel import seq_shard

    B, H, D = 1, 4, 128
    q, k, v = (gen_bf16((B, H, S, D), "n1_outlier", 100 + i).cuda() for i in range(3))
    full = ops.quantize_fp8((q, k, v), scale_mode=ops.SCALE_PER_BH)
    ref = ops.attention_fp8_quantized(*full)
    shards = [seq_shard(S, r, world) for r in range(world)]
    ch = shards[0].chunk_rows
    local = [[t[:, :, sh.start : sh.start + sh.rows] for t in (q, k, v)] for sh in shards]
    parts = [ops.quantize_fp8_bh_partials(loc, npart=ch // 128) for loc in local]
    combined = torch.stack(parts).amax(dim=0)
    quant = [ops.quantize_fp8_bh_apply(loc, combined.clone()) for loc in local]
    for r, sh in enumerate(shards):
        for fq, lq in zip(full, quant[r]):
            assert torch.equal(lq.scales, fq.scales), f"rank {r} scales"
            assert torch.equal(lq.data.view(torch.uint8),
                               fq.data.view(torch.uint8)[:, :, sh.start : sh.start + sh.rows]), f"rank {r}"
    k_all = torch.zeros((world, B * H, ch, D), dtype=torch.uint8, device="cuda")
    v_all = torch.zeros_like(k_all)
    ks_all = torch.zeros((world, B * H, ch // 128), dtype=torch.float32, device="cuda")
    vs_all = torch.zeros_like(ks_all)
    for r, sh in enumerate(shards):
        _, kq, vq = (ops.per_block_view(x) for x in quant[r])
        k_all[r, :, : sh.rows] = kq.data.view(torch.uint8).reshape(B * H, sh.rows, D)
        v_all[r, :, : sh.rows] = vq.data.view(torch.uint8).reshape(B * H, sh.rows, D)
        ks_all[r, :, : kq.scales.shape[1]] = kq.scales
        vs_all[r, :, : vq.scales.shape[1]] = vq.scales
    for r, sh in enumerate(shards):
        out = ops.attention_fp8_chunked(ops.per_block_view(quant[r][0]), k_all.view(ops.FP8),
                                        v_all.view(ops.FP8), ks_all, vs_all, last_rows=shards[0].last_rows)
        torch.cuda.synchronize()
        assert torch.equal(out, ref[:, :, sh.start : sh.start + sh.rows]), f"rank {r}"


class _EventWork:
    """What an asynchronous collective hands back: wait() makes the calling
    stream wait for the transfer (no host wait)."""

    def __init__(self, ev) -> None:  # type: ignore[no-untyped-def]
        self.ev = ev

    def wait(self) -> None:
        torch.cuda.current_stream().wait_event(self.ev)


class _ThreadGather:
    """An asynchronous all_gather_into_tensor for ranks emulated as threads on
    one GPU.  Each rank publishes its input with an event; after a host
    barrier every rank copies all inputs into its output, rank-major, on a
    side stream of its own, and returns a handle whose wait() orders the
    caller's stream after the copies."""

    def __init__(self, world: int) -> None:
        self.world = world
        self.barrier = threading.Barrier(world, timeout=120)
        self.slots: list = [None] * world
        self.side: dict = {}

    def for_rank(self, rank: int):  # type: ignore[no-untyped-def]
        def gather(out, inp, async_op=False):  # type: ignore[no-untyped-def]
            ev = torch.cuda.Event()
            ev.record()
            self.slots[rank] = (inp, ev)
            self.barrier.wait()
            side = self.side.setdefault(rank, torch.cuda.Stream())
            side.wait_stream(torch.cuda.current_stream())
            parts = out.view(self.world, -1)
            with torch.cuda.stream(side):
                for r, (x, e) in enumerate(list(self.slots)):
                    side.wait_event(e)
                    parts[r].copy_(x.reshape(-1))
                    x.record_stream(side)
                done = torch.cuda.Event()
                done.record(side)
            out.record_stream(side)
            self.barrier.wait()  # every rank has read the slots before any rank refills its own
            work = _EventWork(done)
            if async_op:
                return work
            work.wait()
            return None

        gather.supports_async = True  # type: ignore[attr-defined]
        return gather


@pytest.mark.parametrize("S,world,chunks", [(1000, 3, None), (1000, 3, 3), (75600 // 16, 4, 4), (600, 2, None)])
def test_chunk_streams_with_asynchronous_gathers_emulated(S, world, chunks):
    """The overlapped path of ContextParallelAttention (every chunk's gathers
    issued first, each chunk's attention on a stream of its own that waits only
    for its gathers, the caller's stream joining them all), with the ranks as
    threads on one GPU and an asynchronous all-gather between them.  Two calls
    per rank (the chunk streams are reused); every rank's rows equal the
    single-GPU per-block result bit for bit.  (600, 2): the two ranks' shards
    have different query-tile counts, and both must still cut the same chunks."""
    from repercep_runtime_b200.parallel import ContextParallelAttention

    B, H, D = 1, 80 if S == 600 else 4, 128
    q, k, v = (gen_bf16((B, H, S, D), "n05", 90 + i).cuda() for i in range(3))
    ref = _single(q, k, v)
    torch.cuda.synchronize()
    tg = _ThreadGather(world)
    outs: list = [None] * world
    errors: list = []

    def run(rank: int) -> None:
        try:
            torch.cuda.set_device(0)
            with torch.cuda.stream(torch.cuda.Stream()):
                cp = ContextParallelAttention(S, rank, world, all_gather=tg.for_rank(rank))
                sh = cp.shard
                sl = slice(sh.start, sh.start + sh.rows)
                shards = [t[:, :, sl].contiguous() for t in (q, k, v)]
                for _ in range(2):
                    o = cp._device_call(*shards, chunks=chunks)
                torch.cuda.current_stream().synchronize()
                outs[rank] = (sl, o)
        except BaseException as e:  # noqa: BLE001 - reported below
            errors.append(e)
            tg.barrier.abort()

    threads = [threading.Thread(target=run, args=(r,)) for r in range(world)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not any(th.is_alive() for th in threads), "emulated ranks did not finish"
    assert not errors, errors
    for rank, (sl, o) in enumerate(outs):
        assert torch.equal(o, ref[:, :, sl]), f"rank {rank}"


def test_context_parallel_world_one_is_the_plain_call():
    from repercep_runtime_b200.parallel import ContextParallelAttention

    q, k, v = (gen_bf16((1, 2, 300, 128), "n05", 70 + i).cuda() for i in range(3))
    out = ContextParallelAttention(300, 0, 1)(q, k, v)
    assert torch.equal(out, _single(q, k, v))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank: int, world: int, port: int, S: int) -> None:
    import torch.distributed as dist

    from repercep_runtime_b200.parallel import ContextParallelAttention, nccl_all_gather

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        q, k, v = (gen_bf16((1, 12, S, 128), "n05", 80 + i).cuda() for i in range(3))
        cp = ContextParallelAttention(S, rank, world, all_gather=nccl_all_gather())
        sh = cp.shard
        sl = slice(sh.start, sh.start + sh.rows)
        out = cp(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(), v[:, :, sl].contiguous())
        ref = _single(q, k, v)[:, :, sl]
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"rank {rank}"
        # host shards: chunks streamed through the device, same bits
        host = [t[:, :, sl].contiguous().cpu().pin_memory() for t in (q, k, v)]
        out_h = cp(*host)
        assert out_h.device.type == "cpu" and torch.equal(out_h, ref.cpu()), f"rank {rank} (host)"
        # the reference's per-(b,h) scales: partial maxima all-reduced first
        from repercep_runtime_b200 import ops
        from repercep_runtime_b200.parallel import nccl_all_reduce_max

        cpb = ContextParallelAttention(S, rank, world, all_gather=nccl_all_gather(), scale_mode=0,
                                       all_reduce_max=nccl_all_reduce_max())
        out_b = cpb(q[:, :, sl].contiguous(), k[:, :, sl].contiguous(), v[:, :, sl].contiguous())
        ref_b = ops.fp8_attention(q, k, v, scale_mode=ops.SCALE_PER_BH)[:, :, sl]
        torch.cuda.synchronize()
        assert torch.equal(out_b, ref_b), f"rank {rank} (per-(b,h))"
        out_bh = cpb(*host)
        assert torch.equal(out_bh, ref_b.cpu()), f"rank {rank} (per-(b,h), host)"
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_context_parallel_over_nccl():
    import torch.multiprocessing as mp

    # 32768 tokens: 16384-row shards, 64 CTAs per slice -> the host path cuts 4 chunks of 3 slices
    mp.spawn(_nccl_worker, args=(2, _free_port(), 32768), nprocs=2, join=True)
