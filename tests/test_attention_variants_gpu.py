"""The attention kernel's alternative schedules, each through the GPU
attention (and context-parallel, or decode) parity suite in a fresh process
(the library reads these switches once per process).  Default: the lane-split
row layout (two lanes per query row, 8 softmax warps per query tile), every
exp on MUFU, each tile's next QK issued right after its PV.

* REPERCEP_B200_ROW_SPLIT=1 -- one thread per query row (the earlier
  default, with 2 of every 8 exps on the FMA pipe and tile 1's exp phase
  staggered after tile 0's), alone and with each of its switches:
  STAGGER=0 (no stagger), STAGGER=3 (ping-pong), MMA_AHEAD=1, TAIL_SPLIT=1
  (a last wave at most half full run as one-tile CTAs), EXP_POLY=0 / 4;
* REPERCEP_B200_ROW_SPLIT=2 -- two warps per row, maxima swapped through
  shared memory;
* REPERCEP_B200_EXP_POLY=2 / REPERCEP_B200_MMA_AHEAD=0 -- the lane split
  with 2 of 8 exps on the FMA pipe / with every tile's QK before every PV;
* REPERCEP_B200_STEP_TABLE=0 -- per-step scale constants formed in the step
  loop (the path sequences longer than the shared-memory table take);
* REPERCEP_B200_RESCALE_TAU=0 -- O rescaled on every growth of a row max,
  as the reference kernel does;
* REPERCEP_B200_DECODE_KSPLIT=0 -- the shared-prefix decode on one softmax
  warpgroup taking every K/V step (instead of two taking alternate steps);
* REPERCEP_B200_DECODE_PDL=0 -- the decode launched after its quantize launch
  completes instead of as its programmatic dependent.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
ATTN = ["tests/test_attention_gpu.py", "tests/test_context_parallel_gpu.py"]
DECODE = ["tests/test_decode_gpu.py"]

VARIANTS = [
    ("REPERCEP_B200_ROW_SPLIT=1", ATTN + DECODE),
    ("REPERCEP_B200_ROW_SPLIT=1 REPERCEP_B200_STAGGER=0", ATTN),
    ("REPERCEP_B200_ROW_SPLIT=1 REPERCEP_B200_STAGGER=3", ATTN),
    ("REPERCEP_B200_ROW_SPLIT=1 REPERCEP_B200_MMA_AHEAD=1", ATTN),
    ("REPERCEP_B200_ROW_SPLIT=1 REPERCEP_B200_TAIL_SPLIT=1", ATTN),
    ("REPERCEP_B200_ROW_SPLIT=1 REPERCEP_B200_EXP_POLY=0", ATTN),
    ("REPERCEP_B200_ROW_SPLIT=1 REPERCEP_B200_EXP_POLY=4", ATTN),
    ("REPERCEP_B200_ROW_SPLIT=2", ATTN),
    ("REPERCEP_B200_EXP_POLY=2", ATTN),
    ("REPERCEP_B200_MMA_AHEAD=0", ATTN),
    ("REPERCEP_B200_STEP_TABLE=0", ATTN + DECODE),
    ("REPERCEP_B200_RESCALE_TAU=0", ATTN + DECODE),
    ("REPERCEP_B200_DECODE_KSPLIT=0", DECODE),
    ("REPERCEP_B200_DECODE_PDL=0", DECODE),
]


@pytest.mark.gpu
@pytest.mark.parametrize("switches,suite", VARIANTS, ids=[v[0] for v in VARIANTS])
def test_attention_suite_under_schedule_switch(switches, suite):
    env = dict(os.environ)
    for item in switches.split():
        key, value = item.split("=")
        env[key] = value
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", *suite],
        cwd=REPO,
        env=env,
        capture_output=True,
        text=True,
        timeout=900,
    )
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-2000:]
