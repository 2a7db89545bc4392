"""The attention kernel's alternative schedules, each through the whole GPU
attention / decode / context-parallel parity suite in a fresh process (the
library reads these switches once per process):

* REPERCEP_B200_STEP_TABLE=0 -- per-step scale constants formed in the step
  loop (the path sequences longer than the shared-memory table take);
* REPERCEP_B200_STAGGER=0 -- the two query tiles' exp phases not staggered;
* REPERCEP_B200_RESCALE_TAU=0 -- O rescaled on every growth of a row max,
  as the reference kernel does;
* REPERCEP_B200_ROW_SPLIT=2 -- two threads per query row (row max and sum
  exchanged through shared memory);
* REPERCEP_B200_EXP_POLY=0 / 4 -- every exp on MUFU / half on the FMA pipe;
* REPERCEP_B200_DECODE_KSPLIT=0 -- the shared-prefix decode on one softmax
  warpgroup taking every K/V step (instead of two taking alternate steps);
* REPERCEP_B200_DECODE_PDL=0 -- the decode launched after its quantize launch
  completes instead of as its programmatic dependent;
* REPERCEP_B200_MMA_AHEAD=1 -- per step, each tile's PV followed by its
  next-but-one QK (instead of every tile's QK, then every tile's PV);
* REPERCEP_B200_STAGGER=3 -- ping-pong: tile 0's exp phase also waits for
  tile 1's of the previous step;
* REPERCEP_B200_TAIL_SPLIT=1 -- a last wave of two-tile CTAs at most half
  full runs as one-tile CTAs instead.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
SUITE = ["tests/test_attention_gpu.py", "tests/test_decode_gpu.py", "tests/test_context_parallel_gpu.py"]


@pytest.mark.gpu
@pytest.mark.parametrize(
    "switch",
    [
        "REPERCEP_B200_STEP_TABLE=0",
        "REPERCEP_B200_STAGGER=0",
        "REPERCEP_B200_RESCALE_TAU=0",
        "REPERCEP_B200_ROW_SPLIT=2",
        "REPERCEP_B200_EXP_POLY=0",
        "REPERCEP_B200_EXP_POLY=4",
        "REPERCEP_B200_DECODE_KSPLIT=0",
        "REPERCEP_B200_DECODE_PDL=0",
        "REPERCEP_B200_MMA_AHEAD=1",
        "REPERCEP_B200_STAGGER=3",
        "REPERCEP_B200_TAIL_SPLIT=1",
    ],
)
def test_attention_suite_under_schedule_switch(switch):
    key, value = switch.split("=")
    env = dict(os.environ, **{key: value})
    proc = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", *SUITE],
        cwd=REPO,
        env=env,
        capture_output=True,
        text=True,
        timeout=900,
    )
    assert proc.returncode == 0, proc.stdout[-4000:] + proc.stderr[-2000:]
