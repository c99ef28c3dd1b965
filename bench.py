#!/usr/bin/env python
"""Benchmark of the fused TensorProduct forward + VJP on B200 (the BASELINE metric).

One step = TensorProduct(128, 6, parity='full') forward and full VJP (dx, dy, dw)
with a ones cotangent over N = 65,536 rows per GPU (config 2 of the benchmark
recipe; seeded init, iid N(0, 1) inputs).  With N > 1 GPUs (torchrun, one process
per GPU) every rank runs its own 65,536-row shard and dw is all-reduced over NCCL
(weak scaling); `value` is rows of all ranks / max-over-ranks step time.

Prints one JSON line with the metric, the roofline of the dominant kernel, an
end-to-end figure through the public API with host buffers, clocks sampled during
the timed region, and (rank 0, N = 1) the CPU oracle timed on the host cores.
`--impl reference` times the reference algorithm's CPU restatement (the oracle
port) on the host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "fwd+VJP rows/s, TensorProduct C128 m6 full N=65536; % HBM peak; 1–8 GPU"
A100_PUBLISHED_ROWS_PER_S = 65536 / 30.087e-3  # complete_matrix.csv:383
CHANNELS, M_MAX, PARITY = 128, 6, "full"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


# ------------------------------------------------------------------ CPU baseline

def _cpu_worker(task):
    """Oracle fwd + VJP (float32) on `rows` seeded rows; returns seconds."""
    rows, seed = task
    import numpy as np
    from oracle import o2_oracle as O
    oracle = O.TpOracle(CHANNELS, M_MAX, PARITY)
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, oracle.width), dtype=np.float32)
    y = rng.standard_normal((rows, oracle.width), dtype=np.float32)
    w = (rng.standard_normal(oracle.weight_numel) * 0.02).astype(np.float32)
    g = np.ones_like(x)
    start = time.perf_counter()
    oracle.vjp(x, y, w, g)
    return time.perf_counter() - start


def cpu_rows_per_second(rows_per_worker: int, steps: int, warmup: int) -> dict:
    """Times the CPU oracle on all host cores (one spawned process per core)."""
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    values = []
    with ctx.Pool(cores, initializer=_pin_single_thread) as pool:
        for step in range(warmup + steps):
            tasks = [(rows_per_worker, 1000 * step + i) for i in range(cores)]
            elapsed = max(pool.map(_cpu_worker, tasks))
            if step >= warmup:
                values.append(rows_per_worker * cores / elapsed)
    return {"value": statistics.median(values), "unit": "rows/s", "cores": cores,
            "kind": "port",
            "sample": f"{rows_per_worker} rows x {cores} processes per step (float32 numpy "
                      f"oracle, TensorProduct({CHANNELS},{M_MAX},{PARITY!r}) fwd+VJP, ones "
                      f"cotangent), median of {steps} steps"}


def _pin_single_thread():
    os.environ["OMP_NUM_THREADS"] = "1"


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu_index), "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ GPU arm

def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def run_gpu(args) -> dict | None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=device)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False

    from ictc_o2_hp_b200 import TensorProduct, ops

    rows = args.rows
    torch.manual_seed(0)
    tp = TensorProduct(CHANNELS, M_MAX, parity=PARITY).to(device)
    W = tp.representation_dimension
    gen = torch.Generator(device=device)
    gen.manual_seed(1000 + rank)
    x = torch.randn(rows, W, device=device, generator=gen).requires_grad_(True)
    y = torch.randn(rows, W, device=device, generator=gen).requires_grad_(True)
    g = torch.ones(rows, W, device=device)

    def step():
        out = tp(x, y)
        dx, dy, dw = torch.autograd.grad(out, (x, y, tp.weight), g)
        if world > 1:
            dist.all_reduce(dw)
        return out, dx, dy, dw

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        time.sleep(0.3)
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    launches_per_step = 4  # forward; backward prescale, main, slot reduction

    # Per-kernel timing for the roofline, on the launching (current) stream.
    def time_op(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps

    with torch.no_grad():
        xd, yd = x.detach(), y.detach()
        fwd_ms = time_op(lambda: ops.tp_forward(xd, yd, tp.weight.detach(), CHANNELS, M_MAX,
                                                PARITY, "component"), args.steps)
        bwd_ms = time_op(lambda: ops.tp_backward(xd, yd, tp.weight.detach(), g, CHANNELS, M_MAX,
                                                 PARITY, "component"), args.steps)
    fwd_ms, bwd_ms = max_over_ranks(fwd_ms), max_over_ranks(bwd_ms)

    # End to end through the public API with host buffers: H2D of x, y and the
    # cotangent, forward + VJP, D2H of out, dx, dy and dw, every step.
    e2e = None
    if not args.no_e2e:
        pin = dict(dtype=torch.float32, pin_memory=True)
        xh, yh, gh = (torch.empty(rows, W, **pin) for _ in range(3))
        xh.copy_(x.detach()), yh.copy_(y.detach()), gh.fill_(1.0)
        outh, dxh, dyh = (torch.empty(rows, W, **pin) for _ in range(3))
        dwh = torch.empty(tp.weight.numel(), **pin)
        xd2 = torch.empty(rows, W, device=device, requires_grad=False)
        yd2, gd2 = torch.empty_like(xd2), torch.empty_like(xd2)

        def e2e_step():
            xd2.copy_(xh, non_blocking=True)
            yd2.copy_(yh, non_blocking=True)
            gd2.copy_(gh, non_blocking=True)
            xa, ya = xd2.requires_grad_(True), yd2.requires_grad_(True)
            out = tp(xa, ya)
            dx, dy, dw = torch.autograd.grad(out, (xa, ya, tp.weight), gd2)
            if world > 1:
                dist.all_reduce(dw)
            outh.copy_(out, non_blocking=True)
            dxh.copy_(dx, non_blocking=True)
            dyh.copy_(dy, non_blocking=True)
            dwh.copy_(dw, non_blocking=True)
            xd2.requires_grad_(False), yd2.requires_grad_(False)

        e2e_steps = max(3, min(args.steps, 10))
        for _ in range(2):
            e2e_step()
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(e2e_steps):
            e2e_step()
        b.record()
        torch.cuda.synchronize()
        barrier()
        e2e_ms = max_over_ranks(a.elapsed_time(b) / e2e_steps)
        e2e = {"value": rows * world / (e2e_ms * 1e-3), "unit": "rows/s",
               "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": 3 * rows * W * 4,
               "d2h_bytes_per_step": 3 * rows * W * 4 + tp.weight.numel() * 4,
               "steps": e2e_steps}

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None

    peak, peak_kind = peaks()
    hbm = float(peak["hbm_gbs"])
    bwd_bytes = 20 * W * rows  # x, y, g read; dx, dy written (algorithmic)
    fwd_bytes = 12 * W * rows  # x, y read; out written
    dominant = ("tp_backward", bwd_bytes, bwd_ms) if bwd_ms >= fwd_ms else \
        ("tp_forward", fwd_bytes, fwd_ms)
    achieved = dominant[1] / (dominant[2] * 1e-3) / 1e9
    step_bytes = 32 * W * rows
    result = {
        "metric": METRIC,
        "value": rows * world / (ms * 1e-3),
        "unit": "rows/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": rows * world / (ms * 1e-3) / A100_PUBLISHED_ROWS_PER_S,
        "dtype": "f32",
        "data": "synthetic (seeded iid N(0,1) inputs, seeded module init, ones cotangent)",
        "config": {
            "workload": f"TensorProduct({CHANNELS}, {M_MAX}, parity='{PARITY}') forward + VJP "
                        f"(dx, dy, dw), {rows} rows per GPU",
            "rows_per_gpu": rows, "width": W, "weight_numel": tp.weight.numel(),
            "l2": "inputs larger than L2 (each operand is rows x width x 4 B = "
                  f"{rows * W * 4 / 1e6:.0f} MB)",
            "parallelism": f"row shards on {world} GPU(s), one NCCL all_reduce of dw",
        },
        "step_hbm_fraction": step_bytes / (ms * 1e-3) / 1e9 / hbm,
        "kernel_ms": {"tp_forward": fwd_ms, "tp_backward": bwd_ms},
        "roofline": {
            "kernel": dominant[0],
            "bound": "hbm",
            "achieved": achieved,
            "peak": hbm,
            "unit": "GB/s",
            "frac": achieved / hbm,
            "peak_source": f"{peak_kind} hbm_gbs",
            "algorithmic_bytes_per_launch": dominant[1],
            "traffic": None,
        },
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if e2e is not None:
        result["e2e"] = e2e
    return result


# ------------------------------------------------------------------ reference arm

def run_reference(args) -> dict | None:
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    base = cpu_rows_per_second(args.cpu_rows, args.steps, max(1, min(args.warmup, 1)))
    value = base["value"]
    return {
        "metric": METRIC, "impl": "reference", "value": value, "unit": "rows/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": args.cpu_rows * base["cores"] / value * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded iid N(0,1) inputs, ones cotangent)",
        "config": {"workload": f"TensorProduct({CHANNELS}, {M_MAX}, parity='{PARITY}') forward "
                               f"+ VJP on the CPU (reference algorithm, numpy port), bounded "
                               f"sample of {args.cpu_rows} rows per core per step"},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--rows", type=int, default=65536)
    parser.add_argument("--cpu-rows", type=int, default=1024,
                        help="rows per host core per CPU-baseline step")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")

    if args.impl == "reference":
        result = run_reference(args)
        if result is not None:
            print(json.dumps(result), flush=True)
        return 0

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        # The process pool starts before the first CUDA call (spawned workers).
        cpu = cpu_rows_per_second(args.cpu_rows, 3, 1)
    result = run_gpu(args)
    if result is not None:
        if cpu is not None:
            result["cpu_baseline"] = cpu
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
