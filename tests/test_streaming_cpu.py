"""Chunk planning of the host-tensor attention path (no GPU needed)."""

from __future__ import annotations

import pytest

from repercep_runtime_b200.streaming import MIN_CTAS, ChunkPlan, plan_chunks


@pytest.mark.parametrize("bh,seq", [(64, 57600), (64, 8192), (80, 75600), (3, 200), (1, 1), (1000, 128), (7, 300000)])
def test_plan_covers_every_slice_once(bh, seq):
    plan = plan_chunks(bh, seq)
    seen = []
    for i in range(plan.n):
        a, b = plan.bounds(i)
        assert 0 <= a < b <= bh
        seen.extend(range(a, b))
    assert seen == list(range(bh))


def test_plan_fills_the_gpu_and_bounds_the_chunk_count():
    # Cosmos: 225 CTAs per slice -> one slice already fills the GPU; ~64 chunks
    assert plan_chunks(64, 57600) == ChunkPlan(64, 1)
    # cfg2: 32 CTAs per slice -> at least 5 slices per chunk
    p = plan_chunks(64, 8192)
    assert p.chunk * 32 >= MIN_CTAS and p.n == 13
    # tiny problems stay one chunk
    assert plan_chunks(3, 200).n == 1


def test_plan_rejects_empty():
    with pytest.raises(ValueError):
        plan_chunks(0, 128)
