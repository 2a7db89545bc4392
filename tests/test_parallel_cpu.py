"""Multi-GPU host logic on CPU: batch x head sharding, the whole-block
sequence split, and the context-parallel K/V gather run as two gloo ranks with
the oracle standing in for the kernel."""

from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from repercep_runtime_b200.parallel import ContextParallelAttention, seq_shard, shard_bh


@pytest.mark.parametrize("B,H,world", [(2, 32, 1), (2, 32, 8), (2, 40, 8), (1, 3, 2), (2, 5, 4)])
def test_shard_bh_partitions_every_slice_once(B, H, world):
    seen = []
    for r in range(world):
        a, b = shard_bh(B, H, r, world)
        seen.extend(range(a, b))
        assert (b - a) in (B * H // world, B * H // world + 1)
    assert seen == list(range(B * H))


@pytest.mark.parametrize("S,world", [(75600, 2), (75600, 4), (75600, 8), (57600, 8), (300, 2), (128, 1)])
def test_seq_shard_is_whole_blocks_and_covers_the_sequence(S, world):
    rows = []
    for r in range(world):
        sh = seq_shard(S, r, world)
        assert sh.chunk_rows % 128 == 0
        assert sh.start % 128 == 0
        rows.extend(range(sh.start, sh.start + sh.rows))
    assert rows == list(range(S))
    assert seq_shard(S, world - 1, world).rows == seq_shard(S, 0, world).last_rows


def test_seq_shard_rejects_too_short():
    with pytest.raises(ValueError, match="too short"):
        seq_shard(200, 3, 4)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cp_worker(rank: int, world: int, port: int, S: int) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from helpers import bits, gen_bf16
        from oracle import attention as oa
        from oracle import quantize as oq

        B, H, D = 1, 2, 64
        full = [gen_bf16((B, H, S, D), "n1", 40 + i) for i in range(3)]
        cp = ContextParallelAttention(
            S, rank, world, all_gather=lambda o, i: dist.all_gather_into_tensor(o, i)
        )
        sh = cp.shard
        local = [t[:, :, sh.start : sh.start + sh.rows] for t in full]
        # this rank's K/V quantised per block (the oracle in place of the CUDA quantizer)
        k8, ks = oq.quantize_with_scales(bits(local[1]), oq.SCALE_PER_BLOCK128)
        v8, vs = oq.quantize_with_scales(bits(local[2]), oq.SCALE_PER_BLOCK128)
        k_all, v_all, ks_all, vs_all = cp.gather_kv(
            torch.from_numpy(k8.reshape(B * H, sh.rows, D)),
            torch.from_numpy(v8.reshape(B * H, sh.rows, D)),
            torch.from_numpy(ks),
            torch.from_numpy(vs),
        )
        assert k_all.shape == (world, B * H, sh.chunk_rows, D)
        # the gathered chunks, trimmed to their valid rows, are the global per-block layout
        kg = np.concatenate(
            [k_all[c, :, : (sh.chunk_rows if c < world - 1 else sh.last_rows)].numpy() for c in range(world)], 1
        )
        vg = np.concatenate(
            [v_all[c, :, : (sh.chunk_rows if c < world - 1 else sh.last_rows)].numpy() for c in range(world)], 1
        )
        nb = lambda c: sh.chunk_rows // 128 if c < world - 1 else -(-sh.last_rows // 128)  # noqa: E731
        ksg = np.concatenate([ks_all[c, :, : nb(c)].numpy() for c in range(world)], 1)
        vsg = np.concatenate([vs_all[c, :, : nb(c)].numpy() for c in range(world)], 1)
        kf, ksf = oq.quantize_with_scales(bits(full[1]), oq.SCALE_PER_BLOCK128)
        vf, vsf = oq.quantize_with_scales(bits(full[2]), oq.SCALE_PER_BLOCK128)
        assert (kg == kf.reshape(B * H, S, D)).all() and (vg == vf.reshape(B * H, S, D)).all()
        assert (ksg == ksf).all() and (vsg == vsf).all()
        # attention of this rank's rows over the gathered K/V == the same rows of the full problem
        q8, qs = oq.quantize_with_scales(bits(full[0]), oq.SCALE_PER_BLOCK128)
        rows = np.arange(sh.start, sh.start + sh.rows)
        got = oa.attention_dequant(q8.reshape(B * H, S, D), kg, vg, qs, ksg, vsg, 1 / math.sqrt(D), rows=rows)
        ref = oa.attention_dequant(q8.reshape(B * H, S, D), kf.reshape(B * H, S, D), vf.reshape(B * H, S, D),
                                   qs, ksf, vsf, 1 / math.sqrt(D), rows=rows)
        assert np.array_equal(got, ref)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("S,world", [(300, 2), (512, 2)])
def test_context_parallel_gather_with_gloo_ranks(S, world):
    mp.spawn(_cp_worker, args=(world, _free_port(), S), nprocs=world, join=True)


def _async_chunk_worker(rank: int, world: int, port: int, S: int) -> None:
    """The overlapped path's gathers: per (b, h) chunk, asynchronous, through
    ``nccl_all_gather`` bound to a gloo group -- the same bytes as one
    synchronous gather of everything."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from repercep_runtime_b200.parallel import nccl_all_gather

        BH, D = 5, 64
        gather = nccl_all_gather()  # gloo default group: no high-priority subgroup, async supported
        assert getattr(gather, "supports_async", False)
        cp = ContextParallelAttention(S, rank, world, all_gather=gather)
        sh = cp.shard
        g = torch.Generator().manual_seed(rank)
        k8 = torch.randint(0, 256, (BH, sh.rows, D), generator=g, dtype=torch.uint8)
        v8 = torch.randint(0, 256, (BH, sh.rows, D), generator=g, dtype=torch.uint8)
        nblk = -(-sh.rows // 128)
        ks = torch.rand((BH, nblk), generator=g)
        vs = torch.rand((BH, nblk), generator=g)
        k_all, v_all, ks_all, vs_all = cp.gather_kv(k8, v8, ks, vs)
        for bounds in ([(0, 2), (2, 5)], [(0, 1), (1, 3), (3, 5)]):
            pending = [cp._gather(k8[a:b], v8[a:b], ks[a:b], vs[a:b], async_op=True) for a, b in bounds]
            for (a, b), (kc, vc, sc, works) in zip(bounds, pending):
                assert len(works) == 3
                for w in works:
                    w.wait()
                assert torch.equal(kc, k_all[:, a:b]) and torch.equal(vc, v_all[:, a:b])
                assert torch.equal(sc[:, 0], ks_all[:, a:b]) and torch.equal(sc[:, 1], vs_all[:, a:b])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("S,world", [(300, 2), (700, 3)])
def test_chunked_async_gathers_match_one_gather(S, world):
    mp.spawn(_async_chunk_worker, args=(world, _free_port(), S), nprocs=world, join=True)


def _bh_scale_worker(rank: int, world: int, port: int, S: int) -> None:
    """Per-(b,h) scales under context parallelism on gloo ranks, the oracle in
    place of the two quantizer phases: each rank's chunk maxima in
    chunk_rows/128 slots, combined by ``nccl_all_reduce_max`` (bound to the
    gloo group), give the whole sequence's scales and bytes."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from helpers import bits, gen_bf16
        from oracle import quantize as oq
        from repercep_runtime_b200.parallel import nccl_all_reduce_max

        B, H, D = 2, 3, 64
        full = gen_bf16((B, H, S, D), "n1_outlier", 7)
        sh = seq_shard(S, rank, world)
        xb = bits(full[:, :, sh.start : sh.start + sh.rows])
        npart = sh.chunk_rows // 128
        part = np.zeros((B * H, npart), dtype=np.int32)
        for c in range(-(-sh.rows // 128)):
            blk = xb[:, :, c * 128 : (c + 1) * 128].reshape(B * H, -1)
            part[:, c] = oq.absmax_bits(blk, axis=1)
        t = torch.from_numpy(part)
        nccl_all_reduce_max()(t)
        sc = oq.scale_from_amax_bits(t.numpy().max(axis=1).astype(np.uint16))
        ref_sc = oq.per_bh_scale(bits(full))
        assert np.array_equal(sc.view(np.uint32), ref_sc.view(np.uint32))
        full8, _ = oq.quantize_with_scales(bits(full), oq.SCALE_PER_BH)
        local8 = oq.quantize(xb, sc)
        assert np.array_equal(local8, full8[:, :, sh.start : sh.start + sh.rows])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("S,world", [(300, 2), (1000, 3)])
def test_per_bh_scales_combined_across_gloo_ranks(S, world):
    mp.spawn(_bh_scale_worker, args=(world, _free_port(), S), nprocs=world, join=True)


def test_per_bh_context_parallel_needs_a_reduce():
    with pytest.raises(ValueError, match="all_reduce_max"):
        ContextParallelAttention(1000, 0, 2, scale_mode=0)


@pytest.mark.parametrize("bh,rows,first,sizes", [
    (80, 9450, 4, [4, 40, 36]),     # Wan over 8 ranks: 37 two-tile CTAs per slice, 4 slices a wave
    (80, 18900, 2, [2, 40, 38]),    # 4 ranks: 74 per slice
    (80, 37800, 1, [1, 40, 39]),    # 2 ranks: 148 per slice, one slice a wave
    (3, 300, 3, [3]),               # everything fits in the first wave
    (1, 75600, 1, [1]),
])
def test_cp_chunk_plan(bh, rows, first, sizes):
    from repercep_runtime_b200.parallel import cp_chunk_bounds

    b = cp_chunk_bounds(bh, -(-rows // 128))
    assert [y - x for x, y in b] == sizes
    assert b[0] == (0, first)
    assert b[0][0] == 0 and b[-1][1] == bh and all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))


@pytest.mark.parametrize("S,world", [(600, 2), (75600, 8), (75600, 7), (1000, 3), (129, 2), (57600, 6)])
def test_every_rank_cuts_the_same_chunks(S, world):
    """Each chunk of the overlapped call is one set of collectives, so every
    rank must plan the same (b, h) ranges -- also the last rank, whose shard
    is shorter (S = 600 on 2 ranks: 384 and 216 rows, 3 and 2 query tiles)."""
    from repercep_runtime_b200.parallel import ContextParallelAttention

    for bh in (1, 12, 80, 400):
        plans = {tuple(ContextParallelAttention(S, r, world).chunk_plan(bh)) for r in range(world)}
        assert len(plans) == 1, (bh, plans)
        (plan,) = plans
        assert plan[0][0] == 0 and plan[-1][1] == bh
