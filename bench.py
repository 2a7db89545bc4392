#!/usr/bin/env python
"""Benchmark of the B200 FP8 attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cosmos]
                    [--impl b200|reference] [--scaling weak|strong]

One *step* is one pass of the hot path over one batch: quantize Q, K, V
(bf16 -> e4m3 + scales) and run the FP8 attention kernel (bf16 out) — the
work of the reference's ``fp8_flash_attention`` call.  Default workload:
the Cosmos-shaped attention (B=2, H=32, S=57600, D=128, N(0,0.5), per-128-
token-block scales).  Metric: algorithmic TFLOP/s (4*B*H*S^2*D per call),
whole-job aggregate over N GPUs, device-timed with CUDA events, max over
ranks.  Multi-GPU: batch x head slices shard across ranks with no
collective on the data path (weak scaling by default: every rank runs a full
Cosmos-shaped call on its own slices).

``--impl reference`` times the reference's own CPU attention (its AMX BF16
flash kernel, built from its source into oracle/_ref; the numpy oracle when
that cannot run) on a bounded sample of the same workload on the host cores.
Rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

METRIC = "FP8 attn TFLOP/s per GPU & % of FP8 tensor peak at 1/2/4/8 B200; ms/call"
UNIT = "TFLOP/s"
FP8_NOMINAL_TFLOPS = 4500.0  # B200 dense e4m3, per GPU (nominal)

WORKLOADS = {
    "cosmos": dict(B=2, H=32, S=57600, D=128, dist="n05", scale_mode=1,
                   desc="Cosmos-7B DiT self-attn, 16x45x80 patches, N(0,0.5), per-128-block scales"),
    "cfg2": dict(B=2, H=32, S=8192, D=128, dist="n1_outlier", scale_mode=0,
                 desc="B=2 H=32 S=8192, N(0,1) with 1% x20 outliers, per-(b,h) scales"),
    "wan": dict(B=2, H=40, S=75600, D=128, dist="n05", scale_mode=1,
                desc="Wan-2.2 DiT self-attn, 21x45x80 patches, N(0,0.5), per-128-block scales"),
}


def flops_per_call(w: dict) -> float:
    return 4.0 * w["B"] * w["H"] * w["S"] * w["S"] * w["D"]


# ------------------------------------------------------------------ helpers
def gen_inputs(w: dict, seed: int, device: str):
    """Seeded synthetic bf16 Q, K, V on `device` (Q=seed, K=seed+1, V=seed+2)."""
    import torch

    shape = (w["B"], w["H"], w["S"], w["D"])
    out = []
    for i in range(3):
        g = torch.Generator(device=device).manual_seed(seed + i)
        x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        if w["dist"] == "n05":
            x.mul_(0.5)
        elif w["dist"] == "n1_outlier":
            mask = torch.rand(shape, generator=g, device=device) < 0.01
            x = torch.where(mask, x * 20.0, x)
        out.append(x.to(torch.bfloat16))
        del x
    return out


def load_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            pass
    return {}


def profile_traffic(workload: str) -> float | None:
    """DRAM bytes per attention launch, from the committed ncu summary."""
    p = REPO / "profiles" / f"fa8_fwd_{workload}.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the timed region runs."""

    FIELDS = (
        "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
        "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
        "clocks_event_reasons.sw_power_cap"
    )
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.proc = None
        self.ident = None
        try:
            import torch

            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            self.ident = uuid if uuid.startswith("GPU-") else f"GPU-{uuid}"
        except Exception:
            self.ident = None

    def start(self) -> None:
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if self.ident:
            cmd.insert(1, f"--id={self.ident}")
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], [], set()
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for name, val in zip(self.REASONS, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {
            "sm_mhz": statistics.median(sm),
            "sm_max_mhz": max(mx),
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ------------------------------------------------------------- CPU baseline
def cpu_reference_sample(w: dict, target_s: float = 8.0) -> dict:
    """Time the reference's CPU attention on a bounded sample of workload `w`.

    The reference's CPU path is bf16 (it has no FP8; src/repercep/backend/cpu.py:264).
    Kind "reference": its AMX flash kernel (kernels/cpu/amx_attn/flash_attn_amx.cpp,
    built into oracle/_ref) on whole (b,h) slices at the full sequence length.
    Kind "port": the numpy oracle on a few query rows of one slice.
    """
    import torch

    from oracle.build_ref import load_reference_kernel

    S, D = w["S"], w["D"]
    g = torch.Generator().manual_seed(7)
    cores = torch.get_num_threads()
    mod = None
    try:
        mod = load_reference_kernel()
    except Exception:
        mod = None
    if mod is not None and S % 32 == 0 and D in (64, 128):
        q, k, v = (torch.randn((1, 1, S, D), generator=g).mul_(0.5).to(torch.bfloat16) for _ in range(3))
        sm = 1.0 / math.sqrt(D)
        mod.flash_attn_bf16(q[:, :, :128].contiguous(), k[:, :, :128].contiguous(), v[:, :, :128].contiguous(), sm, False)
        t0 = time.perf_counter()
        mod.flash_attn_bf16(q, k, v, sm, False)
        one = time.perf_counter() - t0
        reps = max(1, min(8, int(target_s / max(one, 1e-3))))
        t0 = time.perf_counter()
        for _ in range(reps):
            mod.flash_attn_bf16(q, k, v, sm, False)
        dt = (time.perf_counter() - t0) / reps
        flops = 4.0 * S * S * D
        return {
            "value": flops / dt / 1e12,
            "unit": UNIT,
            "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or cores)),
            "kind": "reference",
            "sample": f"reference AMX bf16 flash kernel, 1 (b,h) slice at full S={S}, D={D}, {reps} calls "
                      f"({dt * 1e3:.0f} ms each); scaled from 1 of {w['B'] * w['H']} slices",
            "seconds_per_sample": dt,
        }
    # numpy oracle port (single process; BLAS threads)
    import numpy as np

    from oracle.attention import softmax_attention

    rows = 256
    rng = np.random.default_rng(7)
    qn = (rng.standard_normal((rows, D)) * 0.5).astype(np.float32)
    kn = (rng.standard_normal((S, D)) * 0.5).astype(np.float32)
    vn = (rng.standard_normal((S, D)) * 0.5).astype(np.float32)
    t0 = time.perf_counter()
    softmax_attention(qn, kn, vn, 1 / math.sqrt(D))
    dt = time.perf_counter() - t0
    return {
        "value": 4.0 * rows * S * D / dt / 1e12,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": f"numpy oracle attention, {rows} query rows x S={S} keys of 1 (b,h) slice",
        "seconds_per_sample": dt,
    }


def run_reference_arm(args, w: dict, rank: int, world: int) -> None:
    if rank != 0:
        return
    base = cpu_reference_sample(w, target_s=2.0)
    times = []
    for i in range(args.warmup + args.steps):
        r = cpu_reference_sample(w, target_s=0.0)
        if i >= args.warmup:
            times.append(r["value"])
    value = statistics.mean(times) if times else base["value"]
    flops = flops_per_call(w)
    ms_call = flops / (value * 1e12) * 1e3
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_call,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "impl": "reference",
        "config": config_for(args, w, world),
        "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")} | {"value": value},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
        "note": "each step times one bounded sample (one (b,h) slice at full S) on the host cores; "
                "ms_per_step is the extrapolated time of one full call",
    }
    print(json.dumps(line), flush=True)


def config_for(args, w: dict, world: int) -> dict:
    bh = w["B"] * w["H"]
    return {
        "workload": args.workload,
        "desc": w["desc"],
        "batch": w["B"],
        "heads": w["H"],
        "seq_len": w["S"],
        "head_dim": w["D"],
        "scale_mode": "per_block128" if w["scale_mode"] == 1 else "per_bh",
        "p_mode": "hilo" if args.p_mode == 1 else "e4m3",
        "flops_per_call": flops_per_call(w),
        "global_bh": bh * world if args.scaling == "weak" else bh,
        "per_rank_bh": bh if args.scaling == "weak" else bh // world,
        "parallelism": f"bh-shard x{world}",
        "l2": "inputs (3 x %.2f GB bf16) exceed the 126 MB L2; no flush needed"
        % (w["B"] * w["H"] * w["S"] * w["D"] * 2 / 1e9),
    }


# ---------------------------------------------------------------- B200 arm
def run_b200_arm(args, w: dict, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from repercep_runtime_b200 import _lib, ops
    from repercep_runtime_b200.attention import B200FP8Attention

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    wl = dict(w)
    if args.scaling == "strong" and world > 1:
        # shard the B*H slices of one call: ranks take whole heads of both batches
        if w["H"] % world:
            raise SystemExit(f"H={w['H']} does not split over {world} ranks")
        wl["H"] = w["H"] // world
    q, k, v = gen_inputs(wl, seed=1000 * rank + 1, device=str(dev))
    flops = flops_per_call(wl)
    stream = torch.cuda.current_stream(dev)

    def step(ev_pair=None):
        qq, kq, vq = ops.quantize_fp8((q, k, v), scale_mode=wl["scale_mode"])
        if ev_pair is not None:
            ev_pair[0].record(stream)
        out = ops.attention_fp8_quantized(qq, kq, vq, p_mode=args.p_mode)
        if ev_pair is not None:
            ev_pair[1].record(stream)
        return out

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    _lib.device_status(reset=True)

    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.3)  # let the sampler start before the timed region
    t0.record(stream)
    for i in range(args.steps):
        step(kev[i])
    t1.record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    ms_total = t0.elapsed_time(t1)
    attn_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    status = _lib.device_status()

    t = torch.tensor([ms_total, attn_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, attn_ms_max = float(t[0]), float(t[1])
    ms_step = ms_total / args.steps
    value = flops * world * args.steps / (ms_total / 1e3) / 1e12

    # e2e through the public AttentionOp with host buffers (pinned), copies timed
    e2e = None
    if not args.no_e2e:
        op = B200FP8Attention(scale_mode=wl["scale_mode"], p_mode=args.p_mode)
        hq, hk, hv = (x.cpu().pin_memory() for x in (q, k, v))
        dq, dk, dv = (torch.empty_like(x) for x in (q, k, v))
        hout = torch.empty(q.shape, dtype=torch.bfloat16, pin_memory=True)

        def e2e_step():
            dq.copy_(hq, non_blocking=True)
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            o = op(dq, dk, dv)
            hout.copy_(o, non_blocking=True)

        e2e_step()
        torch.cuda.synchronize(dev)
        n_e2e = max(1, min(args.steps, 5))
        if world > 1:
            dist.barrier()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        te = torch.tensor([a.elapsed_time(b)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te[0]) / n_e2e
        nbytes = q.numel() * 2
        e2e = {
            "value": flops * world / (e2e_ms / 1e3) / 1e12,
            "unit": UNIT,
            "h2d_bytes_per_step": 3 * nbytes,
            "d2h_bytes_per_step": nbytes,
            "ms_per_step": e2e_ms,
            "api": "B200FP8Attention.__call__ (AttentionOp) with pinned host Q/K/V in, host O out",
        }
        del hq, hk, hv, dq, dk, dv, hout

    if rank != 0:
        return
    peaks = load_peaks()
    if "bf16_tflops_sustained" in peaks:
        peak = 2.0 * float(peaks["bf16_tflops_sustained"])
        peak_src = "of measured: 2 x MEASURED_PEAKS bf16_tflops_sustained (B200 dense e4m3 rate = 2x bf16)"
    else:
        peak = 2.0 * 1400.0
        peak_src = "of fallback: 2 x 1.4 PFLOP/s sustained bf16"
    attn_tflops = flops / (attn_ms / 1e3) / 1e12
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        r = cpu_reference_sample(w)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample")}
    traffic = profile_traffic(args.workload)
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": args.scaling,
        "vs_baseline": None,
        "dtype": "fp8_e4m3",
        "data": "synthetic",
        "config": config_for(args, w, world),
        "tflops_per_gpu": value / world,
        "pct_fp8_peak_nominal": 100.0 * value / world / FP8_NOMINAL_TFLOPS,
        "pct_fp8_peak_measured": 100.0 * value / world / peak,
        "ms_per_call": ms_step,
        "attn_kernel_ms": attn_ms,
        "attn_kernel_ms_max_rank": attn_ms_max,
        "roofline": {
            "bound": "tensor",
            "achieved": attn_tflops,
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": attn_tflops / peak,
            "traffic": traffic,
            "peak_source": peak_src,
            "kernel": "fa8_fwd_kernel<2,%d>" % args.p_mode,
        },
        "cpu_baseline": cpu,
        "e2e": e2e,
        "clocks": clocks,
        "gpu_launches": args.steps * (2 if wl["scale_mode"] == 0 else 1) + args.steps,
        "device_status": status,
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cosmos")
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--scaling", choices=("weak", "strong"), default="weak")
    ap.add_argument("--p-mode", type=int, choices=(0, 1), default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = WORKLOADS[args.workload]

    if args.impl == "reference":
        run_reference_arm(args, w, rank, world)
        return

    import datetime

    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group(
            "nccl",
            timeout=datetime.timedelta(seconds=120),
            device_id=torch.device("cuda", local_rank),
        )
    try:
        run_b200_arm(args, w, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
