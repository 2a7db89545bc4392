#!/usr/bin/env python
"""Benchmark of the B200 FP8 attention hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cosmos]
                    [--impl b200|reference] [--scaling strong|weak]

One *step* is one pass of the hot path over one batch: quantize Q, K, V
(bf16 -> e4m3 + scales) and run the FP8 attention kernel (bf16 out) -- the
work of the reference's ``fp8_flash_attention`` call.  Default workload: the
Cosmos-shaped attention (B=2, H=32, S=57600, D=128, N(0,0.5), per-128-token
block scales).  Metric: algorithmic TFLOP/s (4*B*H*Sq*Skv*D per call), whole
job aggregate over N GPUs, device-timed with CUDA events, max over ranks.

Multi-GPU (one process per GPU under torchrun):
  cosmos / cfg2  batch x head slices shard across ranks with no collective;
                 strong scaling by default (the ranks split one call's
                 slices, so ``value`` is one call's rate); --scaling weak
                 gives every rank a full call's worth of slices.  At N > 1
                 the line also carries a ``wan_cp`` record: the Wan-shaped
                 call over the same N ranks with context parallelism (NCCL
                 all-gather of e4m3 K/V), beside rank 0's single-GPU time for
                 the whole call and a bit-exactness check of sampled slices.
  wan            context parallelism: the sequence splits across ranks, e4m3
                 K/V is all-gathered over NCCL (strong scaling).
  decode         shared-prefix candidate decode, independent replicas.

At N = 1 the line carries side records measured outside the timed region:
the quantize kernel's bandwidth, the shared-prefix decode (CUDA-graph
replays), torch's bf16 SDPA and the reference's own FP8 Triton kernel on the
same inputs, and the FP8 linears.

``--impl reference`` times the reference's own CPU attention on a bounded
sample of the same workload on all the host cores: its default CPU op
(``AMXSDPAAttention``, torch SDPA on CPU) and its AMX BF16 flash kernel
(built from its source into oracle/_ref; the numpy oracle when neither can
run), the faster of the two as ``value``; under torchrun only rank 0 runs it.
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
    "cosmos": dict(kind="attn", B=2, H=32, S=57600, D=128, dist="n05", scale_mode=1,
                   desc="Cosmos-7B DiT self-attn, 16x45x80 patches, N(0,0.5), per-128-block scales"),
    "cfg2": dict(kind="attn", B=2, H=32, S=8192, D=128, dist="n1_outlier", scale_mode=0,
                 desc="B=2 H=32 S=8192, N(0,1) with 1% x20 outliers, per-(b,h) scales"),
    "wan": dict(kind="attn", B=2, H=40, S=75600, D=128, dist="n05", scale_mode=1,
                desc="Wan-2.2 DiT self-attn, 21x45x80 patches, N(0,0.5), per-128-block scales; "
                     "context parallel over N GPUs"),
    "decode": dict(kind="decode", C=64, T=8, H=32, P=512, D=128, dist="n1",
                   desc="token-VLA shared-prefix decode: 64 candidates x 8 new tokens, 512-token "
                        "prefix (quantised once, e4m3-resident), causal per-candidate suffix"),
    "plumbing": dict(kind="cpu", B=1, H=8, S=1024, D=64, dist="n1", scale_mode=0,
                     desc="CPU plumbing case: B=1 H=8 S=1024 D=64, N(0,1) (reference CPU path only)"),
}


def flops_per_call(w: dict) -> float:
    if w["kind"] == "decode":
        rows = w["C"] * w["T"]
        pairs = rows * w["P"] + w["C"] * w["T"] * (w["T"] + 1) // 2
        return 4.0 * w["H"] * pairs * w["D"]
    return 4.0 * w["B"] * w["H"] * w["S"] * w["S"] * w["D"]


# ------------------------------------------------------------------ helpers
def gen_tensor(shape, dist: str, seed: int, device: str):
    """Seeded synthetic bf16 tensor on `device`."""
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
    if dist == "n05":
        x.mul_(0.5)
    elif dist == "n1_outlier":
        mask = torch.rand(shape, generator=g, device=device) < 0.01
        x = torch.where(mask, x * 20.0, x)
    return x.to(torch.bfloat16)


def load_peaks() -> dict:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            pass
    return {}


def profile_traffic(workload: str) -> float | None:
    """DRAM bytes per launch of the dominant kernel, from the committed ncu summary."""
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
        return self.parse(out)

    @classmethod
    def parse(cls, out: str) -> dict | None:
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
            for name, val in zip(cls.REASONS, parts[3:7]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- CPU baseline
REF_PKG = REPO / "baseline" / "_ref"  # the reference's package, installed by oracle/build_ref.py


def host_cores() -> int:
    """Host threads this process may run on (its CPU affinity)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def use_all_host_cores() -> int:
    """Let torch and OpenMP use every host core this process may run on,
    whatever a launcher exported (torch.distributed.run sets
    OMP_NUM_THREADS=1).  Call before the reference's OpenMP kernel is loaded:
    its OpenMP runtime reads OMP_NUM_THREADS when it starts."""
    n = host_cores()
    os.environ["OMP_NUM_THREADS"] = str(n)
    import torch

    torch.set_num_threads(n)
    return torch.get_num_threads()


def reference_cpu_op():  # type: ignore[no-untyped-def]
    """The reference's default CPU attention op, ``AMXSDPAAttention``
    (src/repercep/attention/amx_sdpa.py:76-94, which CPUBackend.attention_op
    picks, src/repercep/backend/cpu.py:281-284), imported unmodified from the
    installed reference package; None when it is not installed."""
    if not (REF_PKG / "repercep" / "__init__.py").exists():
        return None
    if str(REF_PKG) not in sys.path:
        sys.path.append(str(REF_PKG))
    try:
        from repercep.attention.amx_sdpa import AMXSDPAAttention

        op = AMXSDPAAttention()
        return op if op.available else None
    except Exception:
        return None


def _time_calls(fn, target_s: float) -> tuple[float, int]:  # type: ignore[no-untyped-def]
    """Seconds per call of fn (one warm call, then enough for ~target_s)."""
    fn()
    t0 = time.perf_counter()
    fn()
    one = time.perf_counter() - t0
    reps = max(1, min(20, int(target_s / max(one, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(reps):
        fn()
    return (time.perf_counter() - t0) / reps, reps


def cpu_reference_sample(w: dict, target_s: float = 8.0, only: str | None = None) -> dict:
    """Time the reference's CPU attention on a bounded sample of workload `w`.

    The reference's CPU path is bf16 (it has no FP8; src/repercep/backend/cpu.py:264).
    Kind "reference": its two CPU ops on one (b,h) slice at the full sequence
    length (the whole problem for the plumbing case), on all host cores:
    the default op AMXSDPAAttention (torch SDPA on CPU) and the AMX flash
    kernel (kernels/cpu/amx_attn/flash_attn_amx.cpp, built into oracle/_ref);
    ``value`` is the faster one.  Kind "port": the numpy oracle on a few query
    rows of one slice, when neither reference op can run.  Decode: the
    prefix+suffix attention of one head.  ``only`` times just the named op.
    """
    import torch

    from oracle.build_ref import load_reference_kernel

    cores = use_all_host_cores()
    g = torch.Generator().manual_seed(7)
    if w["kind"] == "decode":
        S, D, label = w["P"] + w["C"] * w["T"], w["D"], "one head of the decode (prefix+suffix keys)"
        B, H = 1, 1
    else:
        D, S = w["D"], w["S"]
        B, H = (w["B"], w["H"]) if w["kind"] == "cpu" else (1, 1)
        label = "the whole call" if B * H > 1 else f"1 (b,h) slice of {w['B'] * w['H']}"
    sm = 1.0 / math.sqrt(D)
    ops: dict = {}
    sdpa = reference_cpu_op() if only in (None, "amx-sdpa") else None
    if sdpa is not None:
        q, k, v = (torch.randn((B, H, S, D), generator=g).to(torch.bfloat16) for _ in range(3))
        dt, reps = _time_calls(lambda: sdpa(q, k, v, scale=sm), target_s / 2)
        ops["amx-sdpa"] = {"value": 4.0 * B * H * S * S * D / dt / 1e12, "S": S,
                           "desc": f"reference AMXSDPAAttention (its default CPU op): {reps} calls of "
                                   f"{dt * 1e3:.1f} ms"}
    mod = None
    try:
        mod = load_reference_kernel() if only in (None, "amx-bf16-flash") else None
    except Exception:
        mod = None
    # The AMX kernel takes sequence lengths in whole 32-row tiles: a ragged S
    # (Wan's 75600) is timed at the multiple of 32 below it; the metric is a rate.
    S_amx = S - S % 32
    if mod is not None and S_amx >= 32 and D in (64, 128):
        q, k, v = (torch.randn((B, H, S_amx, D), generator=g).to(torch.bfloat16) for _ in range(3))
        dt, reps = _time_calls(lambda: mod.flash_attn_bf16(q, k, v, sm, False), target_s / 2)
        ops["amx-bf16-flash"] = {
            "value": 4.0 * B * H * S_amx * S_amx * D / dt / 1e12, "S": S_amx,
            "desc": f"reference AMX bf16 flash kernel (kernels/cpu/amx_attn): {reps} calls of "
                    f"{dt * 1e3:.1f} ms" + (" at S rounded down to its 32-row tiles" if S_amx != S else "")}
    if ops:
        best = max(ops, key=lambda n: ops[n]["value"])
        return {
            "value": ops[best]["value"],
            "unit": UNIT,
            "cores": cores,
            "kind": "reference",
            "sample": f"{label} at S={S}, D={D}, bf16, {cores} threads; faster of the reference's CPU ops: "
                      + "; ".join(f"{n} {o['value']:.3f} TFLOP/s ({o['desc']})" for n, o in ops.items()),
            "ops": {n: o["value"] for n, o in ops.items()},
            "best_op": best,
        }
    import numpy as np

    from oracle.attention import softmax_attention

    rows = min(256, S)
    rng = np.random.default_rng(7)
    qn = rng.standard_normal((rows, D)).astype(np.float32)
    kn = rng.standard_normal((S, D)).astype(np.float32)
    vn = rng.standard_normal((S, D)).astype(np.float32)
    t0 = time.perf_counter()
    softmax_attention(qn, kn, vn, 1 / math.sqrt(D))
    dt = time.perf_counter() - t0
    return {
        "value": 4.0 * rows * S * D / dt / 1e12,
        "unit": UNIT,
        "cores": cores,
        "kind": "port",
        "sample": f"numpy oracle attention, {rows} query rows x {S} keys of one slice",
    }


def config_for(args, w: dict, world: int) -> dict:
    cfg = {"workload": args.workload, "desc": w["desc"], "flops_per_call": flops_per_call(w)}
    if w["kind"] == "decode":
        cfg.update(candidates=w["C"], new_tokens=w["T"], heads=w["H"], prefix=w["P"], head_dim=w["D"],
                   parallelism=f"replicas x{world}")
        return cfg
    bh = w["B"] * w["H"]
    cfg.update(batch=w["B"], heads=w["H"], seq_len=w["S"], head_dim=w["D"],
               scale_mode="per_block128" if w["scale_mode"] == 1 else "per_bh",
               p_mode="hilo" if args.p_mode == 1 else "e4m3")
    if w["kind"] == "attn":
        mode = parallel_mode(args, w, world)
        if mode == "cp":
            cfg.update(parallelism=f"context-parallel x{world} (NCCL all-gather of e4m3 K/V)")
        else:
            cfg.update(parallelism=f"bh-shard x{world}",
                       global_bh=bh * world if args.scaling == "weak" else bh,
                       per_rank_bh=bh if args.scaling == "weak" else -(-bh // world))
        cfg["l2"] = "inputs (3 x %.2f GB bf16) exceed the 126 MB L2; no flush needed" % (
            w["B"] * w["H"] * w["S"] * w["D"] * 2 / 1e9)
    return cfg


def parallel_mode(args, w: dict, world: int) -> str:
    if w["kind"] != "attn" or world == 1:
        return "single"
    return "cp" if args.workload == "wan" else "shard"


def run_reference_arm(args, w: dict, rank: int, world: int) -> None:
    if rank != 0:
        return
    use_all_host_cores()
    base = cpu_reference_sample(w, target_s=2.0)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_reference_sample(w, target_s=0.0, only=base.get("best_op"))
        if i >= args.warmup:
            vals.append(r["value"])
    value = statistics.mean(vals) if vals else base["value"]
    ms_call = flops_per_call(w) / (value * 1e12) * 1e3
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_call, "higher_is_better": True,
        "scaling": args.scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "impl": "reference", "config": config_for(args, w, world),
        "cpu_baseline": {k: base[k] for k in ("unit", "cores", "kind", "sample")} | {"value": value}
                        | ({"ops": base["ops"], "best_op": base["best_op"]} if "ops" in base else {}),
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
        "note": "each step times one bounded sample on the host cores; ms_per_step is the "
                "extrapolated time of one full call",
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- B200 arm
class Runner:
    """Builds the per-rank inputs and one step of the hot path for a workload."""

    def __init__(self, args, w: dict, rank: int, world: int, dev) -> None:  # type: ignore[no-untyped-def]
        import torch

        from repercep_runtime_b200 import ops

        self.args, self.w, self.rank, self.world, self.dev = args, w, rank, world, dev
        self.stream = torch.cuda.current_stream(dev)
        self.mode = parallel_mode(args, w, world)
        self.launches_per_step = 2
        d = str(dev)
        if w["kind"] == "decode":
            from repercep_runtime_b200.attention import SharedPrefixFP8Decode

            C, T, H, P, D = w["C"], w["T"], w["H"], w["P"], w["D"]
            self.op = SharedPrefixFP8Decode(p_mode=args.p_mode)
            self.q = gen_tensor((C * T, H, D), w["dist"], 100 * rank + 1, d)
            self.kx = gen_tensor((C * T, H, D), w["dist"], 100 * rank + 2, d)
            self.vx = gen_tensor((C * T, H, D), w["dist"], 100 * rank + 3, d)
            kp = gen_tensor((P, H, D), w["dist"], 100 * rank + 4, d)
            vp = gen_tensor((P, H, D), w["dist"], 100 * rank + 5, d)
            self.prefix = self.op.quantize_prefix(kp, vp)
            self.rank_flops = flops_per_call(w)
            self.job_flops = self.rank_flops * world
            self.inputs = [self.q, self.kx, self.vx]
            return
        B, H, S, D = w["B"], w["H"], w["S"], w["D"]
        self.scale_mode = w["scale_mode"]
        if self.mode == "cp":
            from repercep_runtime_b200.parallel import ContextParallelAttention, nccl_all_gather

            self.cp = ContextParallelAttention(S, rank, world, all_gather=nccl_all_gather(),
                                               p_mode=args.p_mode)
            shape = (B, H, self.cp.shard.rows, D)
            self.scale_mode = ops.SCALE_PER_BLOCK128
            self.job_flops = flops_per_call(w)
            self.rank_flops = 4.0 * B * H * self.cp.shard.rows * S * D
        elif self.mode == "shard" and args.scaling == "strong":
            from repercep_runtime_b200.parallel import shard_bh

            a, b = shard_bh(B, H, rank, world)
            shape = (1, b - a, S, D)
            self.job_flops = flops_per_call(w)
            self.rank_flops = 4.0 * (b - a) * S * S * D
        else:
            shape = (B, H, S, D)
            self.rank_flops = flops_per_call(w)
            self.job_flops = self.rank_flops * world
        self.launches_per_step = 1 + (2 if self.scale_mode == ops.SCALE_PER_BH else 1)
        self.inputs = [gen_tensor(shape, w["dist"], 1000 * rank + i, d) for i in range(3)]

    def step(self, ev=None):  # type: ignore[no-untyped-def]
        """One pass of the hot path; `ev` brackets the dominant kernel."""
        import torch

        from repercep_runtime_b200 import ops

        if self.w["kind"] == "decode":
            qq, kx, vx = ops.quantize_fp8(
                (self.q.unsqueeze(0), self.kx.unsqueeze(0), self.vx.unsqueeze(0)),
                scale_mode=ops.SCALE_PER_BLOCK128, layout="bshd")
            if ev:
                ev[0].record(self.stream)
            out = ops.prefix_decode_fp8_quantized(qq, self.prefix.k, self.prefix.v, kx, vx,
                                                  candidates=self.w["C"], tokens=self.w["T"],
                                                  p_mode=self.args.p_mode)
            if ev:
                ev[1].record(self.stream)
            return out
        q, k, v = self.inputs
        qq, kq, vq = ops.quantize_fp8((q, k, v), scale_mode=self.scale_mode)
        if self.mode == "cp":
            # K/V gathers in (b, h) chunks, each chunk's attention starting when
            # its gather lands: the bracket holds the attention launches and the
            # gathers they did not hide
            if ev:
                ev[0].record(self.stream)
            out = self.cp.attend_quantized(qq, kq, vq)
        else:
            if ev:
                ev[0].record(self.stream)
            out = ops.attention_fp8_quantized(qq, kq, vq, p_mode=self.args.p_mode)
        if ev:
            ev[1].record(self.stream)
        return out

    def quantized_suffix(self):  # type: ignore[no-untyped-def]
        from repercep_runtime_b200 import ops

        return ops.quantize_fp8((self.q.unsqueeze(0), self.kx.unsqueeze(0), self.vx.unsqueeze(0)),
                                scale_mode=ops.SCALE_PER_BLOCK128, layout="bshd")

    def decode_kernel(self, qq, kx, vx):  # type: ignore[no-untyped-def]
        from repercep_runtime_b200 import ops

        return ops.prefix_decode_fp8_quantized(qq, self.prefix.k, self.prefix.v, kx, vx,
                                               candidates=self.w["C"], tokens=self.w["T"],
                                               p_mode=self.args.p_mode)

    def host_api(self) -> bool:
        """True when the public op takes this workload's host tensors directly."""
        return self.w["kind"] != "decode"

    def public_call_host(self, host_inputs):  # type: ignore[no-untyped-def]
        """The user-facing call on host tensors (copies pipelined inside)."""
        from repercep_runtime_b200.attention import B200FP8Attention

        if self.mode == "cp":
            return self.cp(*host_inputs)
        if not hasattr(self, "_op"):
            self._op = B200FP8Attention(scale_mode=self.scale_mode, p_mode=self.args.p_mode)
        return self._op(*host_inputs)

    def public_call(self, host_inputs, dev_inputs):  # type: ignore[no-untyped-def]
        """The user-facing call on device copies of host inputs."""
        if self.w["kind"] == "decode":
            q, kx, vx = dev_inputs
            return self.op(q, self.prefix, kx, vx, candidates=self.w["C"], tokens=self.w["T"])
        if self.mode == "cp":
            return self.cp(*dev_inputs)
        from repercep_runtime_b200.attention import B200FP8Attention

        if not hasattr(self, "_op"):
            self._op = B200FP8Attention(scale_mode=self.scale_mode, p_mode=self.args.p_mode)
        return self._op(*dev_inputs)


def _event_ms(fn, stream, n: int) -> float:  # type: ignore[no-untyped-def]
    """Mean device time of `fn` over n calls (after one untimed call)."""
    import torch

    fn()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(n):
        fn()
    b.record(stream)
    b.synchronize()
    return a.elapsed_time(b) / n


# The Cosmos-7B DiT block's linears (hidden 4096, MLP 16384) over one chunk of
# 16384 tokens: (tokens M, in_features K, out_features N).
LINEAR_SHAPES = {
    "qkv": (16384, 4096, 12288),
    "ffn_up": (16384, 4096, 16384),
    "ffn_down": (16384, 16384, 4096),
}


def linear_measurements(dev, stream, peaks: dict) -> dict:  # type: ignore[no-untyped-def]
    """FP8 DiT linears (``rp_fp8_gemm_ex``): the GEMM alone and the whole
    ``fp8_linear`` (per-token activation quantize + GEMM), per-token x
    per-channel scales, against cuBLASLt's row-scaled FP8 GEMM
    (``torch._scaled_mm``) and torch's bf16 matmul on the same operands.
    Algorithmic FLOPs 2*M*N*K; the kernel is timed alone, so the peak is the
    burst e4m3 rate (2 x the measured bf16 burst)."""
    import torch

    from repercep_runtime_b200 import linear

    if "bf16_tflops" in peaks:
        peak, src = 2.0 * float(peaks["bf16_tflops"]), "of measured: 2 x MEASURED_PEAKS bf16_tflops (burst)"
    else:
        peak, src = 2.0 * 1590.0, "of fallback: 2 x 1.59 PFLOP/s burst bf16"
    rows: dict = {}
    for name, (M, K, N) in LINEAR_SHAPES.items():
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.randn(M, K, device=dev, generator=g, dtype=torch.bfloat16)
        w = (torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        x8, xs = linear.quantize_rows(x)
        w8, ws = linear.quantize_rows(w)
        fl = 2.0 * M * N * K
        row: dict = {"M": M, "K": K, "N": N}
        ms = _event_ms(lambda: linear.gemm_ex(x8, w8, xs, ws), stream, 10)
        row["gemm_ms"] = ms
        row["gemm_tflops"] = fl / ms / 1e9
        row["frac"] = row["gemm_tflops"] / peak
        ms = _event_ms(lambda: linear.fp8_linear(x, w8, ws), stream, 10)
        row["fp8_linear_tflops"] = fl / ms / 1e9
        wt, sa, sb = w8.t(), xs[:, None].contiguous(), ws[None, :].contiguous()
        try:
            ms = _event_ms(lambda: torch._scaled_mm(x8, wt, scale_a=sa, scale_b=sb,
                                                    out_dtype=torch.bfloat16), stream, 10)
            row["cublaslt_fp8_rowwise_tflops"] = fl / ms / 1e9
        except Exception as e:  # pragma: no cover - depends on the torch build
            row["cublaslt_fp8_rowwise_tflops"] = f"unavailable: {type(e).__name__}"
        ms = _event_ms(lambda: x @ w.t(), stream, 10)
        row["torch_bf16_tflops"] = fl / ms / 1e9
        rows[name] = row
        del x, w, x8, w8, xs, ws, wt, sa, sb
    # The QKV projection feeding attention: the per-128-token-block quantizer
    # fused into the GEMM epilogue (rp_fp8_gemm_qkv_quant) against the GEMM
    # with a bf16 output followed by the quantize launch it replaces.
    from repercep_runtime_b200 import ops

    M, K, N = LINEAR_SHAPES["qkv"]
    H = N // (3 * 128)
    g = torch.Generator(device=dev).manual_seed(1)
    x8, xs = linear.quantize_rows(torch.randn(M, K, device=dev, generator=g, dtype=torch.bfloat16))
    w8, ws = linear.quantize_rows((torch.randn(N, K, device=dev, generator=g) * 0.02).to(torch.bfloat16))
    fl = 2.0 * M * N * K

    def separate():  # type: ignore[no-untyped-def]
        c5 = linear.gemm_ex(x8, w8, xs, ws).view(1, M, 3, H, 128)
        return ops.quantize_fp8([c5[:, :, i] for i in range(3)], scale_mode=ops.SCALE_PER_BLOCK128,
                                layout="bshd")

    ms_f = _event_ms(lambda: linear.gemm_qkv_quant(x8, w8, xs, ws, H, M), stream, 10)
    ms_s = _event_ms(separate, stream, 10)
    rows["qkv_quant"] = {
        "M": M, "K": K, "N": N, "heads": H,
        "fused_ms": ms_f, "separate_ms": ms_s, "fused_tflops": fl / ms_f / 1e9,
        "separate_tflops": fl / ms_s / 1e9,
        "bf16_bytes_avoided": 2 * 2 * M * N,
        "desc": "QKV GEMM -> e4m3 Q/K/V + per-128-token-block scales: fused epilogue vs GEMM (bf16 out) "
                "then the quantize launch; outputs bit-identical (tests/test_qkv_quant_gpu.py)",
    }
    del x8, w8, xs, ws
    torch.cuda.synchronize(dev)
    return {"kernel": "fp8_gemm_kernel (2-SM pairs, 256x256 tiles)", "bound": "tensor", "unit": "TFLOP/s",
            "peak": peak, "peak_source": src, "shapes": rows}


def reference_triton_child(workload: str) -> None:
    """Child-process body of reference_triton_row: the reference's own FP8
    Triton kernel (kernels/triton_kernels/fp8_flash_attn_hopper.py:432-586,
    imported unmodified from the installed reference package, static fallback
    tile because autotuning is disabled) on the workload's rank-0 inputs,
    beside this package's kernel in the reference's per-(b,h) scale mode on
    the same inputs.  Prints one JSON line."""
    import torch

    from triton_kernels.fp8_flash_attn_hopper import fp8_flash_attention  # type: ignore[import-not-found]

    from repercep_runtime_b200 import ops

    w = WORKLOADS[workload]
    q, k, v = (gen_tensor((w["B"], w["H"], w["S"], w["D"]), w["dist"], i, "cuda:0") for i in range(3))
    stream = torch.cuda.current_stream()
    res: dict = {"config": "static fallback tile (REPERCEP_FP8_DISABLE_AUTOTUNE=1)"}
    t0 = time.perf_counter()
    out_ref = fp8_flash_attention(q, k, v)
    torch.cuda.synchronize()
    res["first_call_s"] = time.perf_counter() - t0
    ms = _event_ms(lambda: fp8_flash_attention(q, k, v), stream, 3)
    res["ms"] = ms
    res["tflops"] = flops_per_call(w) / (ms / 1e3) / 1e12
    ours = ops.fp8_attention(q, k, v, scale_mode=ops.SCALE_PER_BH)
    a, b = out_ref.float().flatten(), ours.float().flatten()
    res["vs_b200_per_bh"] = {
        "max_abs": float((a - b).abs().max()),
        "cos": float(torch.nn.functional.cosine_similarity(a, b, dim=0)),
        "finite": bool(torch.isfinite(a).all()),
    }
    print(json.dumps(res), flush=True)


def reference_triton_row(workload: str) -> dict:
    """Run reference_triton_child in a fresh process (a compile or launch
    failure of the reference's kernel on sm_100 is recorded, never raised)."""
    if not (REF_PKG / "triton_kernels" / "fp8_flash_attn_hopper.py").exists():
        return {"unavailable": "the reference package is not installed into baseline/_ref "
                               "(oracle/build_ref.py needs the reference source tree)"}
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REF_PKG), str(REPO), env.get("PYTHONPATH", "")])
    env["REPERCEP_FP8_DISABLE_AUTOTUNE"] = "1"
    code = f"import bench; bench.reference_triton_child({workload!r})"
    try:
        proc = subprocess.run([sys.executable, "-c", code], env=env, cwd=str(REPO), capture_output=True,
                              text=True, timeout=600)
    except subprocess.TimeoutExpired:
        return {"failed": "did not finish within 600 s"}
    if proc.returncode != 0:
        tail = (proc.stderr or proc.stdout).strip().splitlines()[-3:]
        return {"failed": f"exit {proc.returncode}: " + " | ".join(tail)[:400]}
    try:
        return json.loads(proc.stdout.strip().splitlines()[-1])
    except (ValueError, IndexError):
        return {"failed": "no result line: " + proc.stdout[-300:]}


def side_measurements(runner: Runner, dev, stream, peaks: dict) -> dict:  # type: ignore[no-untyped-def]
    """Outside the timed region, one GPU only: the quantize kernel's bandwidth
    and torch's bf16 SDPA on the same inputs (the GPU comparison rows)."""
    import torch
    import torch.nn.functional as F

    from repercep_runtime_b200 import ops

    if runner.w["kind"] == "decode" or runner.mode == "cp":
        return {}
    out: dict = {}
    q, k, v = runner.inputs
    elts = q.numel() + k.numel() + v.numel()
    ms = _event_ms(lambda: ops.quantize_fp8((q, k, v), scale_mode=runner.scale_mode), stream, 5)
    algo = 3 * elts  # bf16 read once (2 B) + e4m3 written once (1 B)
    moved = (5 if runner.scale_mode == ops.SCALE_PER_BH else 3) * elts  # per-(b,h): amax pass reads x again
    quant = {"ms": ms, "algorithmic_bytes": algo, "achieved_gbs": algo / ms / 1e6,
             "moved_bytes": moved, "moved_gbs": moved / ms / 1e6, "unit": "GB/s"}
    if "hbm_gbs" in peaks:
        quant["peak_gbs"] = float(peaks["hbm_gbs"])
        quant["frac_moved"] = quant["moved_gbs"] / quant["peak_gbs"]
        quant["peak_source"] = "of measured"
    out["quantize"] = quant
    rows = {}
    n = 3 if runner.rank_flops > 1e13 else 10
    try:
        from torch.nn.attention import SDPBackend, sdpa_kernel

        backends = [("sdpa_bf16_flash", SDPBackend.FLASH_ATTENTION),
                    ("sdpa_bf16_cudnn", SDPBackend.CUDNN_ATTENTION)]
    except Exception:  # pragma: no cover
        backends = []
    for name, be in backends:
        try:
            with sdpa_kernel(be):
                ms = _event_ms(lambda: F.scaled_dot_product_attention(q, k, v), stream, n)
            rows[name] = {"ms": ms, "tflops": runner.rank_flops / (ms / 1e3) / 1e12}
        except Exception as e:  # backend not available for this shape / build
            rows[name] = {"unavailable": f"{type(e).__name__}: {str(e)[:120]}"}
    if os.environ.get("REPERCEP_BENCH_REF_TRITON", "1") != "0":
        rows["reference_fp8_triton"] = reference_triton_row(runner.args.workload)
    out["gpu_comparison"] = rows
    torch.cuda.synchronize(dev)
    try:
        out["fp8_linear"] = linear_measurements(dev, stream, peaks)
    except Exception as e:  # a failure here must not hide the headline line
        out["fp8_linear"] = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
    return out


def dominant_roofline(w: dict, runner: Runner, kernel_ms: float, peaks: dict) -> dict:
    if w["kind"] == "decode":
        C, T, H, P, D = w["C"], w["T"], w["H"], w["P"], w["D"]
        rows = C * T
        # e4m3 Q + prefix K/V + suffix K/V read once, bf16 output written once
        algo = H * D * (rows + 2 * P + 2 * rows) + rows * H * D * 2
        peak = float(peaks.get("hbm_gbs", 6650.0))
        return {"bound": "hbm", "achieved": algo / (kernel_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                "frac": algo / (kernel_ms / 1e3) / 1e9 / peak, "traffic": profile_traffic("decode"),
                "algorithmic_bytes": algo,
                "kernel": ("fa8_fwd_kernel<2,0,0,3,1,1,1> (prefix decode, K/V steps split between two softmax "
                           "warpgroups, two lanes per row)" if runner.args.p_mode == 0
                           else "fa8_fwd_kernel<1,1> (prefix decode)"),
                "peak_source": "of measured" if "hbm_gbs" in peaks else "of fallback"}
    if "bf16_tflops_sustained" in peaks:
        peak = 2.0 * float(peaks["bf16_tflops_sustained"])
        src = "of measured: 2 x MEASURED_PEAKS bf16_tflops_sustained (B200 dense e4m3 rate = 2x bf16)"
    else:
        peak, src = 2.0 * 1400.0, "of fallback: 2 x 1.4 PFLOP/s sustained bf16"
    ach = runner.rank_flops / (kernel_ms / 1e3) / 1e12
    return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
            "traffic": profile_traffic(runner.args.workload), "peak_source": src,
            "kernel": "fa8_fwd_kernel<2,%d>" % runner.args.p_mode}


DECODE_SETTLE_S = 1.0  # idle seconds between the timed region and the decode record


def decode_record(args, dev, stream, peaks: dict) -> dict:  # type: ignore[no-untyped-def]
    """The shared-prefix decode (token-VLA config) on this GPU, outside the
    timed region: one decode step (quantize the new queries and suffix K/V,
    then the decode kernel) and the kernel alone, captured as CUDA graphs and
    replayed, timed with CUDA events.

    ``step_us`` / ``kernel_us``: per call, ten calls captured in one graph (a
    decode loop captured whole, so one graph launch is shared by ten calls);
    ``*_graph1``: one call per graph, back to back (each call also pays a
    graph launch, ~1.7 us on B200); ``*_isolated``: the one-call graph, each
    replay bracketed by its own events."""
    import torch

    w = WORKLOADS["decode"]
    r = Runner(args, w, 0, 1, dev)
    for _ in range(3):
        r.step()
    qq, kx, vx = r.quantized_suffix()
    calls = {"step": r.step, "kernel": lambda: r.decode_kernel(qq, kx, vx)}
    per_graph, n_calls = 10, 200
    out = {}
    graphs = []
    for name, fn in calls.items():
        for per, key in ((per_graph, f"{name}_us"), (1, f"{name}_us_graph1")):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(per):
                    fn()
            graphs.append(g)
            for _ in range(5):
                g.replay()
            n = n_calls // per
            # back to back: n replays between two events (a decode loop's rate)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(n):
                g.replay()
            b.record(stream)
            torch.cuda.synchronize(dev)
            out[key] = 1e3 * a.elapsed_time(b) / (n * per)
            if per == 1:
                # isolated: each replay bracketed by its own events (includes their overhead)
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                       for _ in range(50)]
                for c, d in evs:
                    c.record(stream)
                    g.replay()
                    d.record(stream)
                torch.cuda.synchronize(dev)
                out[f"{name}_us_isolated"] = 1e3 * statistics.median(c.elapsed_time(d) for c, d in evs)
    roof = dominant_roofline(w, r, out["kernel_us"] / 1e3, peaks)
    del graphs
    return {"workload": "decode", "desc": w["desc"], **out,
            "tflops": flops_per_call(w) / (out["kernel_us"] / 1e6) / 1e12,
            "achieved_gbs": roof["achieved"], "peak_gbs": roof["peak"], "frac": roof["frac"],
            "algorithmic_bytes": roof["algorithmic_bytes"], "kernel": roof["kernel"],
            "timing": f"*_us: {n_calls} calls as {n_calls // per_graph} replays of a CUDA graph holding "
                      f"{per_graph} calls, back to back between two CUDA events; *_us_graph1: {n_calls} "
                      f"replays of a one-call graph; *_isolated: median of 50 one-call replays each "
                      f"bracketed by its own events"}


def wan_cp_record(args, rank: int, world: int, dev, stream) -> dict | None:  # type: ignore[no-untyped-def]
    """The Wan-shaped call (B2 H40 S75600) over this job's ranks with context
    parallelism, beside rank 0's single-GPU time for the whole call on the
    same box, and a bit-exactness check of sampled (b,h) slices against it.

    Every rank builds the same global inputs from one seed and attends its
    shard of the sequence (ContextParallelAttention: per-block quantize, NCCL
    all-gather of e4m3 K/V and scales into this GPU's memory, chunked
    attention overlapped with the gathers).  Times are CUDA events, max over
    ranks."""
    import torch
    import torch.distributed as dist

    from repercep_runtime_b200 import ops
    from repercep_runtime_b200.parallel import CP_CHUNKS, ContextParallelAttention, nccl_all_gather

    w = WORKLOADS["wan"]
    B, H, S, D = w["B"], w["H"], w["S"], w["D"]
    d = str(dev)
    full = [gen_tensor((B, H, S, D), w["dist"], 900 + i, d) for i in range(3)]
    cp = ContextParallelAttention(S, rank, world, all_gather=nccl_all_gather(), p_mode=args.p_mode)
    sh = cp.shard
    q, k, v = (x[:, :, sh.start:sh.start + sh.rows].contiguous() for x in full)

    def timed(fn, n: int) -> float:  # type: ignore[no-untyped-def]
        fn()
        torch.cuda.synchronize(dev)
        dist.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        t = torch.tensor([a.elapsed_time(b) / n], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t[0])

    out_cp = cp(q, k, v)
    cp_ms = timed(lambda: cp(q, k, v, out=out_cp), 5)
    quant_ms = timed(lambda: ops.quantize_fp8((q, k, v), scale_mode=ops.SCALE_PER_BLOCK128), 5)
    qq, kq, vq = ops.quantize_fp8((q, k, v), scale_mode=ops.SCALE_PER_BLOCK128)
    bh = B * H
    k_all, v_all, ks_all, vs_all = cp.gather_kv(kq.data.view(torch.uint8).reshape(bh, sh.rows, D),
                                                 vq.data.view(torch.uint8).reshape(bh, sh.rows, D),
                                                 kq.scales, vq.scales)
    attn_out = torch.empty_like(out_cp)
    attn_ms = timed(lambda: ops.attention_fp8_chunked(
        qq, k_all.view(ops.FP8), v_all.view(ops.FP8), ks_all, vs_all, last_rows=sh.last_rows,
        p_mode=args.p_mode, out=attn_out), 5)
    del k_all, v_all, attn_out

    # rank 0: the whole call on one GPU (the other ranks wait at the barrier)
    single_ms, out1 = None, None
    if rank == 0:
        def one():  # type: ignore[no-untyped-def]
            a8, b8, c8 = ops.quantize_fp8(full, scale_mode=ops.SCALE_PER_BLOCK128)
            return ops.attention_fp8_quantized(a8, b8, c8, p_mode=args.p_mode)

        out1 = one()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(3):
            one()
        b.record(stream)
        torch.cuda.synchronize(dev)
        single_ms = a.elapsed_time(b) / 3
    dist.barrier()

    # bit-exactness: sampled (b,h) slices of every rank's rows, gathered to all ranks
    samples = sorted({0, bh // 2, bh - 1})
    mine = torch.zeros((len(samples), sh.chunk_rows, D), dtype=out_cp.dtype, device=dev)
    o3 = out_cp.reshape(bh, sh.rows, D)
    for i, s_ in enumerate(samples):
        mine[i, :sh.rows].copy_(o3[s_])
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine)
    record = None
    if rank == 0:
        got = torch.cat(parts, dim=1)[:, :S]
        ref = out1.reshape(bh, S, D)[samples]
        exact = bool(torch.equal(got.view(torch.int16), ref.view(torch.int16)))
        fl = flops_per_call(w)
        record = {
            "workload": "wan", "desc": w["desc"], "n_gpus": world,
            "parallelism": f"context-parallel x{world} (NCCL all-gather of e4m3 K/V + scales in (b,h) "
                           f"chunks: a first chunk of one CTA wave, then {CP_CHUNKS} whole-wave chunks, each "
                           f"chunk's attention overlapping the later chunks' gathers)",
            "ms_per_call": cp_ms, "tflops": fl / (cp_ms / 1e3) / 1e12,
            "tflops_per_gpu": fl / (cp_ms / 1e3) / 1e12 / world,
            "quantize_ms": quant_ms, "attention_ms": attn_ms,
            "exposed_gather_ms": cp_ms - quant_ms - attn_ms,
            "single_gpu_ms_rank0": single_ms, "single_gpu_tflops_rank0": fl / (single_ms / 1e3) / 1e12,
            "bit_exact_vs_single_gpu": exact, "sampled_bh_slices": samples,
            "timing": "CUDA events over 5 calls after a warm call, max over ranks; single GPU: rank 0 "
                      "alone, 3 calls",
        }
    del full, q, k, v, out_cp, qq, kq, vq, out1, mine, parts
    torch.cuda.empty_cache()
    return record


def run_b200_arm(args, w: dict, rank: int, world: int, local_rank: int) -> None:
    import torch
    import torch.distributed as dist

    from repercep_runtime_b200 import _lib

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    runner = Runner(args, w, rank, world, dev)
    stream = runner.stream

    def barrier():  # type: ignore[no-untyped-def]
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        runner.step()
    torch.cuda.synchronize(dev)
    _lib.device_status(reset=True)

    # Launch-bound workloads (decode: microseconds of GPU work per step) are
    # captured once as CUDA graphs and replayed, so host submission latency
    # is not timed as GPU time; the kernels and their arguments are the same.
    graphs = None
    if runner.w["kind"] == "decode" and not args.no_graph:
        g_step, g_kernel = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_step):
            runner.step()
        qq, kx, vx = runner.quantized_suffix()
        with torch.cuda.graph(g_kernel):
            runner.decode_kernel(qq, kx, vx)
        for _ in range(args.warmup):
            g_step.replay()
            g_kernel.replay()
        torch.cuda.synchronize(dev)
        graphs = (g_step, g_kernel)

    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local_rank)
    barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.3)  # the sampler's first reading lands inside the timed region
    t0.record(stream)
    for i in range(args.steps):
        if graphs is None:
            runner.step(kev[i])
        else:
            graphs[0].replay()
    t1.record(stream)
    if graphs is not None:  # the dominant kernel alone, same graph mechanism
        for i in range(args.steps):
            kev[i][0].record(stream)
            graphs[1].replay()
            kev[i][1].record(stream)
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier()
    ms_total = t0.elapsed_time(t1)
    kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in kev)
    status = _lib.device_status()
    t = torch.tensor([ms_total, kernel_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total, kernel_ms_max = float(t[0]), float(t[1])
    ms_step = ms_total / args.steps
    value = runner.job_flops * args.steps / (ms_total / 1e3) / 1e12

    decode = None
    if world == 1 and not args.no_side and w["kind"] != "decode":
        # The decode is latency-bound and sensitive to the SM clock: right after seconds
        # of power-capped work (the side rows' GEMMs) it ran ~50 % slower on B200 until
        # the clocks recovered, so it runs before them, after a short idle, with its own
        # clock samples.
        time.sleep(DECODE_SETTLE_S)
        dec_clock = ClockSampler(local_rank)
        dec_clock.start()
        time.sleep(0.3)  # the sampler's first reading lands inside the measurement
        try:
            decode = decode_record(args, dev, stream, load_peaks())
        except Exception as e:  # a failure here must not hide the headline line
            decode = {"error": f"{type(e).__name__}: {str(e)[:200]}"}
        decode["clocks"] = dec_clock.stop()
        decode["settle_s"] = DECODE_SETTLE_S
    side = side_measurements(runner, dev, stream, load_peaks()) if world == 1 and not args.no_side else {}
    if decode is not None:
        side["decode"] = decode

    e2e = None
    if not args.no_e2e:
        host = [x.cpu().pin_memory() for x in runner.inputs]
        if runner.host_api():
            # The op on host tensors: it pipelines the copies with compute.
            hout = runner.public_call_host(host)

            def e2e_step():  # type: ignore[no-untyped-def]
                runner.public_call_host(host)

            api = ("public op (B200FP8Attention / ContextParallelAttention).__call__ on pinned host "
                   "tensors (copies of (b,h) chunks pipelined with compute), host result")
        else:
            devc = [torch.empty_like(x) for x in runner.inputs]
            out0 = runner.public_call(host, devc)
            hout = torch.empty(out0.shape, dtype=out0.dtype, pin_memory=True)

            def e2e_step():  # type: ignore[no-untyped-def]
                for dd, hh in zip(devc, host):
                    dd.copy_(hh, non_blocking=True)
                hout.copy_(runner.public_call(host, devc), non_blocking=True)

            api = ("public op SharedPrefixFP8Decode.__call__ on pinned host inputs, output "
                   "copied back")

        e2e_step()
        torch.cuda.synchronize(dev)
        n_e2e = max(1, min(args.steps, 5))
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n_e2e):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        te = torch.tensor([a.elapsed_time(b)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e_ms = float(te[0]) / n_e2e
        e2e = {
            "value": runner.job_flops / (e2e_ms / 1e3) / 1e12,
            "unit": UNIT,
            "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in host),
            "d2h_bytes_per_step": hout.numel() * hout.element_size(),
            "ms_per_step": e2e_ms,
            "api": api,
        }

    wan_cp = None
    if world > 1 and w["kind"] == "attn" and runner.mode != "cp" and not args.no_wan_cp:
        del runner.inputs  # this rank's Cosmos slices are no longer needed
        torch.cuda.empty_cache()
        wan_cp = wan_cp_record(args, rank, world, dev, stream)

    if rank != 0:
        return
    peaks = load_peaks()
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        r = cpu_reference_sample(w)
        cpu = {k: r[k] for k in ("value", "unit", "cores", "kind", "sample", "ops", "best_op") if k in r}
    per_gpu = value / world
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak" if w["kind"] == "decode" else ("strong" if runner.mode == "cp" else args.scaling),
        "vs_baseline": None, "dtype": "fp8_e4m3", "data": "synthetic",
        "config": config_for(args, w, world),
        "tflops_per_gpu": per_gpu,
        "pct_fp8_peak_nominal": 100.0 * per_gpu / FP8_NOMINAL_TFLOPS,
        "pct_fp8_peak_measured": 100.0 * per_gpu / (2.0 * float(peaks.get("bf16_tflops_sustained", 1400.0))),
        "ms_per_call": ms_step,
        "kernel_ms": kernel_ms,
        "kernel_ms_max_rank": kernel_ms_max,
        "roofline": dominant_roofline(w, runner, kernel_ms, peaks),
        "cpu_baseline": cpu,
        "e2e": e2e,
        **side,
        "clocks": clocks,
        "gpu_launches": args.steps * runner.launches_per_step,
        "cuda_graph": graphs is not None,
        "device_status": status,
    }
    if wan_cp is not None:
        line["wan_cp"] = wan_cp
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cosmos")
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--scaling", choices=("weak", "strong"), default="strong")
    ap.add_argument("--p-mode", type=int, choices=(0, 1), default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-side", action="store_true",
                    help="skip the side measurements (quantize bandwidth, SDPA and FP8 linear rows)")
    ap.add_argument("--no-graph", action="store_true", help="decode: launch eagerly instead of replaying a CUDA graph")
    ap.add_argument("--no-wan-cp", action="store_true", help="N > 1: skip the wan_cp record")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the workload's batch (profiling a smaller case of the same kernel)")
    ap.add_argument("--heads", type=int, default=None, help="override the workload's head count")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    w = dict(WORKLOADS[args.workload])
    for key, val in (("B", args.batch), ("H", args.heads)):
        if val is not None:
            if key not in w or val <= 0:
                ap.error(f"--{'batch' if key == 'B' else 'heads'} does not apply to {args.workload}")
            w[key] = val
            w["desc"] += f" [{key} overridden to {val}]"

    if args.impl == "reference":
        run_reference_arm(args, w, rank, world)
        return
    if w["kind"] == "cpu":
        ap.error(f"workload {args.workload!r} is the reference's CPU case; use --impl reference")

    import datetime

    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_b200_arm(args, w, rank, world, local_rank)
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
