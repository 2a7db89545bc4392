"""Context-parallel attention on the GPU.

With P ranks emulated on one GPU: each rank's e4m3 K/V chunk and scales are
stacked as the all-gather would deliver them, and the chunked kernel runs each
rank's queries against them.  Because shards are whole 128-token blocks, the
result must equal the single-GPU per-block result bit for bit.  With two or
more GPUs, the same check runs over NCCL with one process per GPU.
"""

from __future__ import annotations

import os
import socket

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
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_context_parallel_over_nccl():
    import torch.multiprocessing as mp

    # 32768 tokens: 16384-row shards, 64 CTAs per slice -> the host path cuts 4 chunks of 3 slices
    mp.spawn(_nccl_worker, args=(2, _free_port(), 32768), nprocs=2, join=True)
