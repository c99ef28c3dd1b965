#!/usr/bin/env python
"""Benchmark of the B200 tensor-product kernels on the BASELINE configurations.

Default workload (the BASELINE metric): TensorProduct(128, 6, parity='full')
forward and full VJP (dx, dy, dw) with a ones cotangent over N = 65,536 rows per
GPU (config 2; seeded init, iid N(0, 1) inputs).  With N > 1 GPUs (torchrun, one
process per GPU) every rank runs its own 65,536-row shard and dw is all-reduced
over NCCL (weak scaling); `value` = rows of all ranks / max-over-ranks step time.

Other workloads (``--workload``): ``uvu`` = UvuTensorProduct(128, 32, 3) shared
weights over 131,072 rows per GPU (config 4); ``radial`` = the config-5 message-
passing layer, 1,048,576 edges in total sharded over the ranks (strong scaling),
Bessel(8) x cosine-cutoff radial basis -> MLP 8->64->64 (SiLU) -> fused affine +
V=1 uvu (C=64, m_max=3, full, angular harmonics up to 3), forward and VJP through
the whole radial network, one all-reduce of every parameter gradient.

Prints one JSON line: the metric, the roofline of the dominant kernel, an
end-to-end figure through the public API with host buffers (H2D of the inputs and
D2H of the results every step), clocks sampled during the timed region, and (rank
0, N = 1) the CPU oracle timed on the host cores.  ``--impl reference`` times the
reference algorithm's CPU restatement (the oracle port) on the host cores instead.
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

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}
# FP32 FMA peak of a B200: 148 SMs x 128 FMA lanes x 2 FLOP x 1.965 GHz (max SM clock).
# The uvu and radial kernels are strict FP32 (no tensor cores), so this is their roof.
FP32_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12

METRICS = {
    "tp": "fwd+VJP rows/s, TensorProduct C128 m6 full N=65536; % HBM peak; 1–8 GPU",
    "uvu": "fwd+VJP rows/s, UvuTensorProduct C128 V32 m3 full shared weights N=131072",
    "uvu_rowwise": "fwd+VJP rows/s, UvuTensorProduct C128 V32 m3 full per-row weights, "
                   "16384 rows per GPU",
    "radial": "fwd+VJP edges/s, RadialUvuTensorProduct C64 m3 radial MLP 8-64-64, E=1048576",
    "radial_mp": "fwd+VJP edges/s, message-passing layer: gather by source, "
                 "RadialUvuTensorProduct C64 m3, fixed-order sum to destinations, E=1048576 "
                 "over 65536 nodes",
    "radial_m6": "fwd+VJP edges/s, RadialUvuTensorProduct C{channels} m6 full / angular "
                 "canonical, radial MLP 16-64-64, E=131072",
    "radial_m6_force": "force-loss training edges/s (second derivatives), "
                       "RadialUvuTensorProduct C{channels} m6, radial MLP 16-64-64, E=131072",
}
# A100 published fwd+VJP for config 2 (benchmarks/eqx/results/complete_matrix.csv:383)
A100_TP_ROWS_PER_S = 65536 / 30.087e-3
# A100 published full VJP of the radial chain m6, N = 131,072 edges, by channel count
# (docs/RADIAL_PERFORMANCE.md:9, :59, :15)
A100_RADIAL_M6_MS = {64: 114.167, 128: 208.039, 256: 410.604}


# ------------------------------------------------------------------ CPU baseline

def _cpu_worker(task):
    """Oracle fwd + VJP (float32) on `rows` seeded rows of a workload; returns s."""
    workload, rows, seed, channels = task
    import numpy as np
    from oracle import o2_oracle as O
    rng = np.random.default_rng(seed)
    if workload == "tp":
        oracle = O.TpOracle(128, 6, "full")
        x = rng.standard_normal((rows, oracle.width), dtype=np.float32)
        y = rng.standard_normal((rows, oracle.width), dtype=np.float32)
        w = (rng.standard_normal(oracle.weight_numel) * 0.02).astype(np.float32)
        g = np.ones_like(x)
        start = time.perf_counter()
        oracle.vjp(x, y, w, g)
    elif workload in ("uvu", "uvu_rowwise"):
        shared = workload == "uvu"
        oracle = O.UvuOracle(128, 32, 3)
        x = rng.standard_normal((rows, oracle.width1), dtype=np.float32)
        y = rng.standard_normal((rows, oracle.width2), dtype=np.float32)
        wshape = (oracle.weight_numel,) if shared else (rows, oracle.weight_numel)
        w = (rng.standard_normal(wshape) / np.sqrt(32)).astype(np.float32)
        g = np.ones_like(x)
        start = time.perf_counter()
        oracle.vjp(x, y, w, g, shared=shared)
    else:
        m6 = workload.startswith("radial_m6")
        uvu = O.UvuOracle(channels if m6 else 64, 1, 6 if m6 else 3, "full", "canonical")
        radial = O.RadialOracle(uvu)
        x = rng.standard_normal((rows, uvu.width1), dtype=np.float32)
        y = rng.standard_normal((rows, uvu.width2), dtype=np.float32)
        h = rng.standard_normal((rows, 64), dtype=np.float32)
        a = (rng.standard_normal((uvu.weight_numel, 64)) / 8).astype(np.float32)
        g = np.ones_like(x)
        start = time.perf_counter()
        radial.vjp(x, y, h, a, g)
    return time.perf_counter() - start


def _pin_single_thread():
    os.environ["OMP_NUM_THREADS"] = "1"


def cpu_units_per_second(workload: str, rows_per_worker: int, steps: int, warmup: int,
                         channels: int = 64) -> dict:
    """Times the CPU oracle on all host cores (one spawned process per core)."""
    import multiprocessing as mp
    cores = os.cpu_count() or 1
    ctx = mp.get_context("spawn")
    values = []
    with ctx.Pool(cores, initializer=_pin_single_thread) as pool:
        for step in range(warmup + steps):
            tasks = [(workload, rows_per_worker, 1000 * step + i, channels) for i in range(cores)]
            elapsed = max(pool.map(_cpu_worker, tasks))
            if step >= warmup:
                values.append(rows_per_worker * cores / elapsed)
    unit = "edges/s" if workload.startswith("radial") else "rows/s"
    return {"value": statistics.median(values), "unit": unit, "cores": cores, "kind": "port",
            "sample": f"{rows_per_worker} rows x {cores} processes per step (float32 numpy "
                      f"oracle of the reference algorithm, {workload} fwd+VJP), median of "
                      f"{steps} steps"}


# The force-loss workload has no CPU leg: the numpy oracle has no second derivatives.
CPU_ROWS = {"tp": 1024, "uvu": 16, "uvu_rowwise": 4, "radial": 256, "radial_m6": 64}

# Rows (edges) per step of the reference package's own CPU path: about a second of
# work per step on 16 host threads.
REF_CPU_ROWS = {"tp": 4096, "uvu": 512, "uvu_rowwise": 32, "radial": 1024, "radial_m6": 256}
REF_DIR = ROOT / "baseline" / "_ref"


def reference_cpu_available() -> bool:
    return (REF_DIR / "ictc_o2_hp").is_dir()


def reference_cpu_units_per_second(workload: str, rows: int, steps: int, warmup: int,
                                   channels: int = 64) -> dict:
    """Times the reference package's own CPU PyTorch path (installed under baseline/_ref;
    CPU tensors take its PyTorch algebra, fast_o2.py / uvu_o2.py / radial_uvu.py) on all
    host threads: forward + VJP of a seeded sample of `rows` rows per step, float32,
    median over `steps` steps after `warmup`.  Runs before any CUDA work of the process."""
    import torch
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import ictc_o2_hp as ref
    prev = torch.get_num_threads()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    try:
        gen = torch.Generator().manual_seed(0)
        torch.manual_seed(0)
        if workload == "tp":
            tp = ref.TensorProduct(128, 6, parity="full")
            W = tp.representation_dimension
            x, y = (torch.randn(rows, W, generator=gen) for _ in range(2))
            g = torch.ones(rows, W)
            leaves, call = [tp.weight], (lambda xx, yy: tp(xx, yy))
        elif workload in ("uvu", "uvu_rowwise"):
            shared = workload == "uvu"
            tp = ref.UvuTensorProduct(128, 32, 3, shared_weights=shared,
                                      internal_weights=shared)
            x = torch.randn(rows, tp.input1_dimension, generator=gen)
            y = torch.randn(rows, tp.input2_dimension, generator=gen)
            g = torch.ones(rows, tp.input1_dimension)
            if shared:
                leaves, call = [tp.weight], (lambda xx, yy: tp(xx, yy))
            else:
                w = (torch.randn(rows, tp.weight_numel, generator=gen) / 32 ** 0.5)
                w.requires_grad_(True)
                leaves, call = [w], (lambda xx, yy: tp(xx, yy, w))
        else:
            m6 = workload.startswith("radial_m6")
            tp = ref.UvuTensorProduct(channels if m6 else 64, 1, 6 if m6 else 3, parity="full",
                                      parity_in2="canonical", shared_weights=False)
            model = ref.RadialUvuTensorProduct(
                tp, torch.nn.Linear(64, tp.weight_numel, bias=False))
            x = torch.randn(rows, tp.input1_dimension, generator=gen)
            y = torch.randn(rows, tp.input2_dimension, generator=gen)
            h = torch.randn(rows, 64, generator=gen).requires_grad_(True)
            g = torch.ones(rows, tp.input1_dimension)
            leaves = [h] + list(model.parameters())
            call = lambda xx, yy: model(xx, yy, h)  # noqa: E731
        x.requires_grad_(True)
        y.requires_grad_(True)
        values = []
        for step in range(warmup + steps):
            start = time.perf_counter()
            torch.autograd.grad(call(x, y), [x, y] + leaves, g)
            elapsed = time.perf_counter() - start
            if step >= warmup:
                values.append(rows / elapsed)
    finally:
        torch.set_num_threads(prev)
    unit = "edges/s" if workload.startswith("radial") else "rows/s"
    return {"value": statistics.median(values), "unit": unit, "cores": cores,
            "kind": "reference",
            "sample": f"{rows} rows per step through the reference package's own CPU path "
                      f"(float32 PyTorch, {cores} threads, {workload} fwd+VJP), median of "
                      f"{steps} steps"}


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines = []

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
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [line for line in out.splitlines() if line.strip()]
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
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


def peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


# ------------------------------------------------------------------ workloads

class Workload:
    """Common parts of the bench workloads."""

    def e2e_outputs(self, results):
        """Results read back to the host in the end-to-end figure (all of them)."""
        return _leaves(results)

    def collective_numel(self) -> int:
        """float32 elements of the one all-reduce a step makes with N > 1 ranks."""
        return 0


class TpWorkload(Workload):
    """Config 2: TensorProduct(128, 6, 'full') fwd + VJP, 65,536 rows per GPU."""

    name, scaling, unit = "tp", "weak", "rows/s"

    def __init__(self, args, device, rank, world):
        import torch
        from ictc_o2_hp_b200 import TensorProduct, ops
        self.ops, self.torch, self.world = ops, torch, world
        self.rows = args.rows or 65536
        torch.manual_seed(0)
        self.tp = TensorProduct(128, 6, parity="full").to(device)
        self.W = self.tp.representation_dimension
        gen = torch.Generator(device=device)
        gen.manual_seed(1000 + rank)
        self.x = torch.randn(self.rows, self.W, device=device, generator=gen)
        self.y = torch.randn(self.rows, self.W, device=device, generator=gen)
        self.g = torch.ones(self.rows, self.W, device=device)
        self.units = self.rows
        self.launches = 4  # forward; backward prescale, main, slot reduction

    def step(self, x=None, y=None, g=None):
        torch = self.torch
        x = (self.x if x is None else x).detach().requires_grad_(True)
        y = (self.y if y is None else y).detach().requires_grad_(True)
        out = self.tp(x, y)
        dx, dy, dw = torch.autograd.grad(out, (x, y, self.tp.weight),
                                         self.g if g is None else g)
        if self.world > 1:
            torch.distributed.all_reduce(dw)
        return out, dx, dy, dw

    def kernels(self, time_op):
        ops, w = self.ops, self.tp.weight.detach()
        fwd = time_op(lambda: ops.tp_forward(self.x, self.y, w, 128, 6, "full", "component"))
        bwd = time_op(lambda: ops.tp_backward(self.x, self.y, w, self.g, 128, 6, "full",
                                              "component"))
        return {"tp_forward": (fwd, 12 * self.W * self.rows),
                "tp_backward": (bwd, 20 * self.W * self.rows)}, "hbm"

    def host_inputs(self):
        return (self.x, self.y, self.g)

    def e2e_runner(self):
        """Host-buffer path: ictc_o2_hp_b200.host.TensorProductHostRunner streams the
        rows in chunks with the two copy directions overlapped."""
        from ictc_o2_hp_b200.host import TensorProductHostRunner
        runner = TensorProductHostRunner(self.tp)
        torch = self.torch

        def run(x, y, g, out, dx, dy, dw_host):
            dw = runner.run(x, y, g, out, dx, dy)
            if self.world > 1:
                torch.distributed.all_reduce(dw)
            dw_host.copy_(dw, non_blocking=True)

        return run, (self.x, self.y, self.g), (self.x, self.x, self.x, self.tp.weight)

    def config(self):
        return {"workload": f"TensorProduct(128, 6, parity='full') forward + VJP (dx, dy, dw), "
                            f"{self.rows} rows per GPU, ones cotangent",
                "rows_per_gpu": self.rows, "width": self.W,
                "weight_numel": self.tp.weight.numel(),
                "l2": f"inputs larger than L2 (each operand {self.rows * self.W * 4 / 1e6:.0f} MB)",
                "parallelism": f"row shards on {self.world} GPU(s), one NCCL all_reduce of dw"}

    def step_bytes(self):
        return 32 * self.W * self.rows

    def collective_numel(self):
        return self.tp.weight.numel()


class UvuWorkload(Workload):
    """Config 4 (shared weights): UvuTensorProduct(128, 32, 3) fwd + VJP."""

    name, scaling, unit = "uvu", "weak", "rows/s"

    def __init__(self, args, device, rank, world):
        import torch
        from ictc_o2_hp_b200 import UvuTensorProduct, ops
        self.ops, self.torch, self.world = ops, torch, world
        self.rows = args.rows or 131072
        torch.manual_seed(0)
        self.tp = UvuTensorProduct(128, 32, 3).to(device)
        with torch.no_grad():
            self.tp.weight.copy_(torch.randn(self.tp.weight_numel, device=device) / 32 ** 0.5)
        gen = torch.Generator(device=device)
        gen.manual_seed(2000 + rank)
        self.x = torch.randn(self.rows, self.tp.input1_dimension, device=device, generator=gen)
        self.y = torch.randn(self.rows, self.tp.input2_dimension, device=device, generator=gen)
        self.g = torch.ones(self.rows, self.tp.input1_dimension, device=device)
        self.units = self.rows
        self.launches = 6
        e2 = self.tp.entries_in2
        self.fma_per_row = sum(128 * 32 * e2[j].dim for (_, j, _) in self.tp.paths)

    def step(self, x=None, y=None, g=None):
        torch = self.torch
        x = (self.x if x is None else x).detach().requires_grad_(True)
        y = (self.y if y is None else y).detach().requires_grad_(True)
        out = self.tp(x, y)
        dx, dy, dw = torch.autograd.grad(out, (x, y, self.tp.weight),
                                         self.g if g is None else g)
        if self.world > 1:
            torch.distributed.all_reduce(dw)
        return out, dx, dy, dw

    def kernels(self, time_op):
        ops, tp = self.ops, self.tp
        w = tp.weight.detach()
        fwd = time_op(lambda: ops.uvu_forward(self.x, self.y, w, tp._table, tp._config, True))
        bwd = time_op(lambda: ops.uvu_backward(self.x, self.y, w, self.g, tp._table, tp._config,
                                               True, 7))
        flops = 2 * self.fma_per_row * self.rows
        return {"uvu_forward": (fwd, flops), "uvu_backward": (bwd, 3 * flops)}, "fp32"

    def host_inputs(self):
        return (self.x, self.y, self.g)

    def config(self):
        return {"workload": f"UvuTensorProduct(128, 32, 3, parity='full') shared weights, "
                            f"forward + VJP (dx, dy, dw), {self.rows} rows per GPU",
                "rows_per_gpu": self.rows, "weight_numel": self.tp.weight_numel,
                "l2": "inputs larger than L2",
                "parallelism": f"row shards on {self.world} GPU(s), one NCCL all_reduce of dw"}

    def step_bytes(self):
        return (3 * self.tp.input1_dimension + self.tp.input2_dimension) * 4 * self.rows * 2

    def collective_numel(self):
        return self.tp.weight_numel


class UvuRowWorkload(UvuWorkload):
    """Config 4 (per-row weights): UvuTensorProduct(128, 32, 3), an (N, weight_numel)
    weight tensor ~ N(0,1)/sqrt(32); 16,384 rows per GPU (the full N = 131,072 needs
    318 GB of weights: it runs 8-way sharded, 16,384 rows per GPU)."""

    name, scaling, unit = "uvu_rowwise", "weak", "rows/s"

    def __init__(self, args, device, rank, world):
        import torch
        from ictc_o2_hp_b200 import UvuTensorProduct, ops
        self.ops, self.torch, self.world = ops, torch, world
        self.rows = args.rows or 16384
        self.tp = UvuTensorProduct(128, 32, 3, shared_weights=False).to(device)
        gen = torch.Generator(device=device)
        gen.manual_seed(4000 + rank)
        self.x = torch.randn(self.rows, self.tp.input1_dimension, device=device, generator=gen)
        self.y = torch.randn(self.rows, self.tp.input2_dimension, device=device, generator=gen)
        self.w = torch.randn(self.rows, self.tp.weight_numel, device=device,
                             generator=gen) / 32 ** 0.5
        self.g = torch.ones(self.rows, self.tp.input1_dimension, device=device)
        self.units = self.rows
        self.launches = 2

    def step(self, x=None, y=None, g=None):
        torch = self.torch
        x = (self.x if x is None else x).detach().requires_grad_(True)
        y = (self.y if y is None else y).detach().requires_grad_(True)
        w = self.w.detach().requires_grad_(True)
        out = self.tp(x, y, w)
        dx, dy, dw = torch.autograd.grad(out, (x, y, w), self.g if g is None else g)
        return out, dx, dy, dw

    def kernels(self, time_op):
        ops, tp = self.ops, self.tp
        fwd = time_op(lambda: ops.uvu_forward(self.x, self.y, self.w, tp._table, tp._config,
                                              False))
        bwd = time_op(lambda: ops.uvu_backward(self.x, self.y, self.w, self.g, tp._table,
                                               tp._config, False, 7))
        wbytes = 4 * self.tp.weight_numel * self.rows
        act = 4 * (self.tp.input1_dimension + self.tp.input2_dimension) * self.rows
        # forward: read w, x, y, write out; VJP: read w, x, y, g, write dw, dx, dy
        return {"uvu_forward": (fwd, wbytes + act + 4 * self.tp.input1_dimension * self.rows),
                "uvu_backward": (bwd, 2 * wbytes + 2 * act + 4 * self.tp.input1_dimension
                                 * self.rows)}, "hbm"

    def host_inputs(self):
        return (self.x, self.y, self.g)

    def e2e_outputs(self, results):
        # out, dx and dy; dw (2.4 MB per row, like the weights) stays on the device
        return results[:3]

    def collective_numel(self):
        return 0

    def config(self):
        return {"workload": f"UvuTensorProduct(128, 32, 3, parity='full') per-row weights, "
                            f"forward + VJP (dx, dy, dw), {self.rows} rows per GPU",
                "rows_per_gpu": self.rows, "weight_numel": self.tp.weight_numel,
                "l2": "inputs larger than L2 (weights 2.4 MB per row)",
                "parallelism": f"row shards on {self.world} GPU(s), no collective (per-row "
                               "weights)"}

    def step_bytes(self):
        return 3 * 4 * self.tp.weight_numel * self.rows


class RadialWorkload(Workload):
    """Config 5: 1,048,576 edges over 65,536 nodes, sharded over the ranks."""

    name, scaling, unit = "radial", "strong", "edges/s"
    EDGES, NODES, RC = 1048576, 65536, 5.0

    def __init__(self, args, device, rank, world):
        import torch
        from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct, ops
        from ictc_o2_hp_b200.parallel import shard_bounds
        self.ops, self.torch, self.world = ops, torch, world
        total = args.rows or self.EDGES
        start, stop = shard_bounds(total, world, rank)
        self.total, self.edges = total, stop - start
        torch.manual_seed(0)
        tp = UvuTensorProduct(64, 1, 3, parity="full", parity_in2="canonical",
                              shared_weights=False)
        self.trunk = torch.nn.Sequential(torch.nn.Linear(8, 64), torch.nn.SiLU(),
                                         torch.nn.Linear(64, 64), torch.nn.SiLU()).to(device)
        self.model = RadialUvuTensorProduct(
            tp, torch.nn.Linear(64, tp.weight_numel, bias=False)).to(device)
        gen = torch.Generator(device=device)
        gen.manual_seed(3000)
        nodes = torch.randn(self.NODES, tp.input1_dimension, device=device, generator=gen)
        src = torch.randint(0, self.NODES, (total,), device=device, generator=gen)
        off = torch.randint(1, self.NODES, (total,), device=device, generator=gen)
        dst = (src + off) % self.NODES  # uniform over the other nodes: no self-loops
        r = torch.rand(total, device=device, generator=gen) * 4.5 + 0.5
        theta = torch.rand(total, device=device, generator=gen) * 2 * math.pi
        sl = slice(start, stop)
        # gather of node features by source: outside the reference chain
        self.x = nodes[src[sl]].contiguous()
        self.nodes, self.src_shard, self.dst_shard = nodes, src[sl], dst[sl]
        self.dst = dst[sl]
        self.r = r[sl].contiguous()
        th = theta[sl]
        self.angular = torch.stack([torch.ones_like(th)] + [
            f(m * th) for m in range(1, 4) for f in (torch.cos, torch.sin)], dim=-1).contiguous()
        self.g = torch.ones(self.edges, tp.input1_dimension, device=device)
        self.units = self.edges
        self.launches = 6
        self.params = list(self.trunk.parameters()) + list(self.model.parameters())

    def basis(self, r):
        torch = self.torch
        n = torch.arange(1, 9, device=r.device, dtype=r.dtype)
        bessel = math.sqrt(2 / self.RC) * torch.sin(n * math.pi * r[:, None] / self.RC) / r[:, None]
        cutoff = 0.5 * (torch.cos(math.pi * r / self.RC) + 1)
        return bessel * cutoff[:, None]

    def step(self, x=None, y=None, g=None):
        torch = self.torch
        x = (self.x if x is None else x).detach().requires_grad_(True)
        ang = (self.angular if y is None else y).detach().requires_grad_(True)
        hidden = self.trunk(self.basis(self.r))
        out = self.model(x, ang, hidden)
        grads = torch.autograd.grad(out, [x, ang] + self.params, self.g if g is None else g)
        if self.world > 1:
            flat = torch.cat([t.reshape(-1) for t in grads[2:]])
            torch.distributed.all_reduce(flat)
        return out, grads

    def kernels(self, time_op):
        ops, m = self.ops, self.model
        torch = self.torch
        with torch.no_grad():
            hidden = self.trunk(self.basis(self.r)).contiguous()
        alpha = m.radial_out.weight.detach()
        empty = alpha.new_empty(0)
        rc = m._rconfig()
        fwd = time_op(lambda: ops.radial_forward(self.x, self.angular, hidden, alpha, empty,
                                                 m.tp._table, rc, False))
        bwd = time_op(lambda: ops.radial_backward(self.x, self.angular, hidden, alpha, empty,
                                                  self.g, m.tp._table, rc, False, 15))
        wn = m.tp.weight_numel
        flops = 2 * wn * 64 * self.edges  # affine regeneration per edge
        return {"radial_forward": (fwd, flops), "radial_backward": (bwd, 3 * flops)}, "fp32"

    def host_inputs(self):
        return (self.x, self.angular, self.g)

    def config(self):
        return {"workload": "RadialUvuTensorProduct message-passing layer: 1048576 edges over "
                            "65536 nodes, Bessel(8) x cosine cutoff 5.0, MLP 8-64-64 SiLU, fused "
                            "affine (bias=False) + V=1 uvu C64 m3 full / angular canonical m3, "
                            "forward + VJP through the radial network",
                "edges_total": self.total, "edges_per_gpu": self.edges,
                "l2": "inputs larger than L2 (per-edge features 3.7 GB)",
                "parallelism": f"edge shards on {self.world} GPU(s), one NCCL all_reduce of all "
                               "parameter gradients"}

    def step_bytes(self):
        return (3 * 896 + 2 * 7 + 64 * 2) * 4 * self.edges

    def collective_numel(self):
        return sum(p.numel() for p in self.params)


class RadialMpWorkload(RadialWorkload):
    """Config 5 as a message-passing layer: node features read by source inside the
    radial kernels (graph.radial_messages: the gather is folded into the edge tile),
    the radial product, messages summed into the destination nodes
    (ictc_o2_segment_sum, fixed order); the VJP covers the node features (per-edge
    gradients summed by source), the angular inputs and every parameter.  Edges
    are sharded; each rank reads the full node set and its node gradients join the
    one all-reduce."""

    name = "radial_mp"

    def __init__(self, args, device, rank, world):
        super().__init__(args, device, rank, world)
        from ictc_o2_hp_b200.graph import EdgeIndex, radial_messages, scatter_sum
        from ictc_o2_hp_b200 import parallel
        self.radial_messages, self.scatter_sum = radial_messages, scatter_sum
        self.parallel = parallel
        # edges stored in source order (CSR by source, as graph libraries keep them):
        # the same edges, relabelled, so consecutive edges share their node row
        perm = self.torch.sort(self.src_shard, stable=True).indices
        self.src_shard, self.dst_shard = self.src_shard[perm], self.dst_shard[perm]
        self.r, self.angular = self.r[perm].contiguous(), self.angular[perm].contiguous()
        self.edge_index = EdgeIndex(self.src_shard, self.dst_shard, self.NODES)
        # --node-partition (N > 1): rank r owns node block r; node features are
        # all-gathered, node outputs and node gradients reduce-scattered to the owners
        self.node_partition = bool(getattr(args, "node_partition", False)) and world > 1
        self.counts = parallel.node_counts(self.NODES, world)
        n0, n1 = parallel.shard_bounds(self.NODES, world, rank)
        if self.node_partition:
            self.nodes = self.nodes[n0:n1].contiguous()
        self.g_nodes = self.torch.ones_like(self.nodes)
        self.launches = 8  # radial kernels + message sum and the node-gradient sum

    def step(self, x=None, y=None, g=None):
        torch = self.torch
        nodes = (self.nodes if x is None else x).detach().requires_grad_(True)
        ang = (self.angular if y is None else y).detach().requires_grad_(True)
        hidden = self.trunk(self.basis(self.r))
        table = (self.parallel.all_gather_rows(nodes, self.counts) if self.node_partition
                 else nodes)
        # the gather by source is folded into the radial kernels (no [E, 896] copy)
        messages = self.radial_messages(self.model, table, self.edge_index, ang, hidden)
        out = self.scatter_sum(messages, self.edge_index)
        if self.node_partition:
            out = self.parallel.reduce_scatter_rows(out, self.counts)
        grads = torch.autograd.grad(out, [nodes, ang] + self.params,
                                    self.g_nodes if g is None else g)
        if self.world > 1:
            # node gradients are already reduced onto their owners when partitioned
            shared = ([] if self.node_partition else [grads[0]]) + list(grads[2:])
            flat = torch.cat([t.reshape(-1) for t in shared])
            torch.distributed.all_reduce(flat)
        return out, grads

    def host_inputs(self):
        return (self.nodes, self.angular, self.g_nodes)

    def collective_numel(self):
        nodes = 0 if self.node_partition else self.nodes.numel()
        return nodes + sum(p.numel() for p in self.params)

    def config(self):
        c = super().config()
        c["workload"] = ("message-passing layer (config 5 shapes): edges stored in source "
                         "order, node features [65536, 896] "
                         "read by source inside the radial kernels (no gathered copy), Bessel(8) "
                         "x cosine cutoff, MLP 8-64-64 SiLU, fused affine + V=1 uvu C64 m3, "
                         "messages summed into destination nodes in a fixed order; VJP to node "
                         "features, angular and all parameters")
        if self.node_partition:
            c["parallelism"] = (f"edge shards and node blocks on {self.world} GPU(s): node "
                                "features all-gathered, node outputs and node gradients "
                                "reduce-scattered to their owners (NCCL), one all_reduce of "
                                "the parameter gradients")
        else:
            c["parallelism"] = (f"edge shards on {self.world} GPU(s), full node set per rank, "
                                "one NCCL all_reduce of node-feature and parameter gradients")
        return c


class RadialM6Workload(Workload):
    """The reference's published radial chain (docs/RADIAL_PERFORMANCE.md:6-12): radial
    features [N, 16] -> Linear(16,64) -> SiLU -> Linear(64,64) -> SiLU -> fused
    Linear(64, P*C, bias=False) + V=1 uvu, C64, m_max 6, first input / output full,
    angular canonical; N = 131,072 edges; the full VJP covers the three inputs and every
    network parameter."""

    name, scaling, unit = "radial_m6", "strong", "edges/s"
    EDGES = 131072

    @staticmethod
    def published(args):
        ms = A100_RADIAL_M6_MS.get(args.channels)
        return None if ms is None or (args.rows or 131072) != 131072 else 131072 / (ms * 1e-3)

    def __init__(self, args, device, rank, world):
        import torch
        from ictc_o2_hp_b200 import RadialUvuTensorProduct, UvuTensorProduct, ops
        from ictc_o2_hp_b200.parallel import shard_bounds
        self.ops, self.torch, self.world = ops, torch, world
        total = args.rows or self.EDGES
        start, stop = shard_bounds(total, world, rank)
        self.total, self.edges = total, stop - start
        torch.manual_seed(0)
        self.channels = args.channels
        tp = UvuTensorProduct(self.channels, 1, 6, parity="full", parity_in2="canonical",
                              shared_weights=False)
        self.trunk = torch.nn.Sequential(torch.nn.Linear(16, 64), torch.nn.SiLU(),
                                         torch.nn.Linear(64, 64), torch.nn.SiLU()).to(device)
        self.model = RadialUvuTensorProduct(
            tp, torch.nn.Linear(64, tp.weight_numel, bias=False)).to(device)
        gen = torch.Generator(device=device)
        gen.manual_seed(4000)
        x = torch.randn(total, tp.input1_dimension, device=device, generator=gen)
        feat = torch.randn(total, 16, device=device, generator=gen)
        theta = torch.rand(total, device=device, generator=gen) * 2 * math.pi
        sl = slice(start, stop)
        self.x = x[sl].contiguous()
        self.feat = feat[sl].contiguous()
        th = theta[sl]
        self.angular = torch.stack([torch.ones_like(th)] + [
            f(m * th) for m in range(1, 7) for f in (torch.cos, torch.sin)], dim=-1).contiguous()
        self.g = torch.ones(self.edges, tp.input1_dimension, device=device)
        self.units = self.edges
        self.launches = 6
        self.params = list(self.trunk.parameters()) + list(self.model.parameters())

    def step(self, x=None, y=None, f=None, g=None):
        torch = self.torch
        x = (self.x if x is None else x).detach().requires_grad_(True)
        ang = (self.angular if y is None else y).detach().requires_grad_(True)
        feat = (self.feat if f is None else f).detach().requires_grad_(True)
        out = self.model(x, ang, self.trunk(feat))
        grads = torch.autograd.grad(out, [x, ang, feat] + self.params,
                                    self.g if g is None else g)
        if self.world > 1:
            flat = torch.cat([t.reshape(-1) for t in grads[3:]])
            torch.distributed.all_reduce(flat)
        return out, grads

    def kernels(self, time_op):
        ops, m = self.ops, self.model
        torch = self.torch
        with torch.no_grad():
            hidden = self.trunk(self.feat).contiguous()
        alpha = m.radial_out.weight.detach()
        empty = alpha.new_empty(0)
        rc = m._rconfig()
        fwd = time_op(lambda: ops.radial_forward(self.x, self.angular, hidden, alpha, empty,
                                                 m.tp._table, rc, False))
        bwd = time_op(lambda: ops.radial_backward(self.x, self.angular, hidden, alpha, empty,
                                                  self.g, m.tp._table, rc, False, 15))
        flops = 2 * m.tp.weight_numel * 64 * self.edges  # affine regeneration per edge
        return {"radial_forward": (fwd, flops), "radial_backward": (bwd, 3 * flops)}, "fp32"

    def host_inputs(self):
        return (self.x, self.angular, self.feat, self.g)

    def config(self):
        return {"workload": "reference's published radial chain: radial features [N,16] -> "
                            f"MLP 16-64-64 SiLU -> fused affine (bias=False) + V=1 uvu "
                            f"C{self.channels} m6 full / angular canonical m6, forward + full "
                            "VJP (x, angular, features, every parameter)",
                "channels": self.channels,
                "edges_total": self.total, "edges_per_gpu": self.edges,
                "l2": "inputs larger than L2 (per-edge features 0.9 GB, gw block 8.4 GB)",
                "parallelism": f"edge shards on {self.world} GPU(s), one NCCL all_reduce of all "
                               "parameter gradients"}

    def step_bytes(self):
        w1 = self.x.shape[1]
        return (3 * w1 + 2 * 13 + 2 * 16 + 64 * 2) * 4 * self.edges

    def collective_numel(self):
        return sum(p.numel() for p in self.params)


class RadialM6ForceWorkload(RadialM6Workload):
    """Force-loss training through the published radial chain (second derivatives,
    the "force_parameters" metric of docs/RADIAL_PERFORMANCE.md:60-65): energy =
    sum of the layer output; forces = its gradient with respect to x, angular and the
    radial features (create_graph=True); loss = sum of the squared forces,
    differentiated with respect to the three inputs and every network parameter.
    The reference publishes the metric but not its loss, so vs_baseline stays null."""

    name = "radial_m6_force"

    @staticmethod
    def published(args):
        return None

    def step(self, x=None, y=None, f=None, g=None):
        torch = self.torch
        x = (self.x if x is None else x).detach().requires_grad_(True)
        ang = (self.angular if y is None else y).detach().requires_grad_(True)
        feat = (self.feat if f is None else f).detach().requires_grad_(True)
        energy = self.model(x, ang, self.trunk(feat)).sum()
        forces = torch.autograd.grad(energy, (x, ang, feat), create_graph=True)
        loss = sum(t.square().sum() for t in forces)
        grads = torch.autograd.grad(loss, [x, ang, feat] + self.params)
        if self.world > 1:
            flat = torch.cat([t.reshape(-1) for t in grads[3:]])
            torch.distributed.all_reduce(flat)
        return loss, grads

    def config(self):
        c = super().config()
        c["workload"] = ("force-loss training through the reference's published radial chain "
                         "(MLP 16-64-64, fused affine + V=1 uvu C{} m6): energy = sum of "
                         "outputs, forces = d energy / d (x, angular, features) with "
                         "create_graph, loss = sum of squared forces, gradients for the "
                         "inputs and every parameter").format(self.channels)
        return c


WORKLOADS = {"tp": TpWorkload, "uvu": UvuWorkload, "uvu_rowwise": UvuRowWorkload,
             "radial": RadialWorkload, "radial_mp": RadialMpWorkload,
             "radial_m6": RadialM6Workload,
             "radial_m6_force": RadialM6ForceWorkload}


# ------------------------------------------------------------------ GPU arm

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
    torch.set_float32_matmul_precision("highest")

    wl = WORKLOADS[args.workload](args, device, rank, world)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed_steps(w, steps, warmup, clocks=None):
        """Device time of `steps` steps after `warmup`, barrier and synchronize on
        both sides, max over ranks (ms per step)."""
        for _ in range(warmup):
            w.step()
        barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if clocks is not None:
            time.sleep(0.3)
        start.record()
        for _ in range(steps):
            w.step()
        end.record()
        torch.cuda.synchronize()
        if clocks is not None:
            time.sleep(0.2)
        barrier()
        return max_over_ranks(start.elapsed_time(end) / steps)

    with ClockSampler(local_rank) as clocks:
        ms = timed_steps(wl, args.steps, args.warmup, clocks)

    # Per-kernel timing for the roofline, on the launching (current) stream.
    def time_op(fn, steps=None):
        steps = steps or args.steps
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / steps

    def time_allreduce(numel):
        """The step's one all-reduce timed by itself on a buffer of its size (ms,
        max over ranks); None with one rank (no collective)."""
        if world == 1 or numel == 0:
            return None
        buf = torch.ones(numel, device=device)
        barrier()
        t = time_op(lambda: dist.all_reduce(buf), steps=20)
        return max_over_ranks(t)

    with torch.no_grad():
        kernels, bound = wl.kernels(time_op)
    kernels = {k: (max_over_ranks(t), work) for k, (t, work) in kernels.items()}
    collective = {"allreduce_bytes": 4 * wl.collective_numel(),
                  "allreduce_ms": time_allreduce(wl.collective_numel())}

    # End to end through the public API with host buffers: H2D of this step's
    # inputs from pinned memory, forward + VJP, D2H of every result.
    e2e = None
    if not args.no_e2e and hasattr(wl, "e2e_runner"):
        # the workload's host-buffer API: its own copies, overlapped with the kernels
        run, dev_in, dev_out = wl.e2e_runner()
        host_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in dev_in]
        for h, d in zip(host_in, dev_in):
            h.copy_(d)
        host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in dev_out]

        def e2e_step():
            run(*host_in, *host_out)

        e2e_steps = max(3, min(args.steps, 10))
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
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
        total_units = wl.units * world if wl.scaling == "weak" else wl.total
        e2e = {"value": total_units / (e2e_ms * 1e-3), "unit": wl.unit, "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host_in),
               "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in host_out),
               "steps": e2e_steps,
               "path": "chunked host-buffer runner, host-to-device and device-to-host "
                       "copies overlapped with each other and with the kernels"}
    elif not args.no_e2e:
        dev_in = wl.host_inputs()
        host_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in dev_in]
        for h, d in zip(host_in, dev_in):
            h.copy_(d)
        staged = [torch.empty_like(d) for d in dev_in]
        results = wl.step()
        flat_results = list(wl.e2e_outputs(results))
        host_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in flat_results]

        def e2e_step():
            for s, h in zip(staged, host_in):
                s.copy_(h, non_blocking=True)
            res = list(wl.e2e_outputs(wl.step(*staged)))
            for h, t in zip(host_out, res):
                h.copy_(t.detach(), non_blocking=True)

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
        total_units = wl.units * world if wl.scaling == "weak" else wl.total
        e2e = {"value": total_units / (e2e_ms * 1e-3), "unit": wl.unit, "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host_in),
               "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in host_out),
               "steps": e2e_steps}

    # The north-star multi-GPU target: config 5 (1,048,576 edges in total, strong
    # scaling) measured in the same run as the default workload.
    radial = None
    if args.workload == "tp" and not args.no_radial_scaling:
        del wl.x, wl.y, wl.g
        torch.cuda.empty_cache()
        rargs = argparse.Namespace(**{**vars(args), "rows": 0})
        rw = RadialWorkload(rargs, device, rank, world)
        rsteps = max(3, min(args.steps, 10))
        rms = timed_steps(rw, rsteps, 3)
        with torch.no_grad():
            rk, _ = rw.kernels(lambda fn: time_op(fn, steps=rsteps))
        rk = {k: max_over_ranks(t) for k, (t, _) in rk.items()}
        radial = {"metric": METRICS["radial"], "value": rw.total / (rms * 1e-3),
                  "unit": "edges/s", "scaling": "strong", "ms_per_step": rms, "steps": rsteps,
                  "edges_total": rw.total, "edges_per_gpu": rw.edges,
                  "kernel_ms_max_over_ranks": rk,
                  "allreduce_bytes": 4 * rw.collective_numel(),
                  "allreduce_ms": time_allreduce(rw.collective_numel())}
        del rw

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return None

    peak, peak_kind = peaks()
    hbm = float(peak["hbm_gbs"])
    name, (kms, work) = max(kernels.items(), key=lambda kv: kv[1][0])
    if bound == "hbm":
        achieved = work / (kms * 1e-3) / 1e9
        roof = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS)",
                "algorithmic_bytes_per_launch": work, "traffic": traffic_of(wl, name)[0],
                "traffic_source": traffic_of(wl, name)[1]}
    else:
        achieved = work / (kms * 1e-3) / 1e12
        roof = {"kernel": name, "bound": "fp32", "achieved": achieved, "peak": FP32_PEAK_TFLOPS,
                "unit": "TFLOP/s", "frac": achieved / FP32_PEAK_TFLOPS,
                "peak_source": "nominal FP32 FMA peak at the 1965 MHz max SM clock (strict "
                               "FP32, no tensor cores)", "algorithmic_flops_per_launch": work,
                "traffic": traffic_of(wl, name)[0], "traffic_source": traffic_of(wl, name)[1]}
    total_units = wl.units * world if wl.scaling == "weak" else wl.total
    value = total_units / (ms * 1e-3)
    result = {
        "metric": METRICS[wl.name].format(channels=args.channels),
        "value": value,
        "unit": wl.unit,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": wl.scaling,
        "vs_baseline": vs_baseline(wl, args, value),
        "dtype": "f32",
        "data": "synthetic (seeded iid N(0,1) inputs, seeded init, ones cotangent)",
        "config": wl.config(),
        "step_hbm_fraction": wl.step_bytes() * (world if wl.scaling == "weak" else 1)
                             / world / (ms * 1e-3) / 1e9 / hbm,
        "kernel_ms": {k: t for k, (t, _) in kernels.items()},
        "roofline": roof,
        "gpu_launches": wl.launches * args.steps,
        "clocks": clocks.summary(),
    }
    result["collective"] = collective
    if e2e is not None:
        result["e2e"] = e2e
    if radial is not None:
        result["radial_strong_scaling"] = radial
    return result


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one 65,536-row launch
# of the TensorProduct(128, 6, full) kernels (the default workload's own launch), from a
# one-pass ncu capture of this bench command; other row counts carry it scaled by rows,
# and the line says which.
TRAFFIC_65K_ROWS = {"tp_backward": 2.6174e9 + 1.7112e9, "tp_forward": 1.7450e9 + 0.8421e9}


def traffic_of(wl, name):
    """(bytes per launch, how obtained) for the dominant kernel, or (None, None)."""
    if wl.name == "tp" and name in TRAFFIC_65K_ROWS:
        if wl.rows == 65536:
            return (TRAFFIC_65K_ROWS[name],
                    "ncu DRAM bytes (read + write) of this 65,536-row launch of the kernel")
        return (TRAFFIC_65K_ROWS[name] * wl.rows / 65536,
                "ncu DRAM bytes of a 65,536-row launch of the same kernel, scaled by rows to "
                f"this {wl.rows}-row launch")
    return None, None


def vs_baseline(wl, args, value):
    """value / the reference's published number for this exact metric and config."""
    if hasattr(wl, "published"):
        ref = wl.published(args)
    elif wl.name == "tp" and args.rows in (0, 65536):
        ref = A100_TP_ROWS_PER_S
    else:
        ref = None
    return value / ref if ref else None


def _leaves(value):
    import torch
    if isinstance(value, torch.Tensor):
        yield value
    elif isinstance(value, (list, tuple)):
        for v in value:
            yield from _leaves(v)


# ------------------------------------------------------------------ config-3 sweep

SWEEP_CHANNELS = (32, 64, 96, 128, 256)
SWEEP_M_MAX = (1, 2, 3, 4, 5, 6)
SWEEP_PARITY = ("canonical", "full")
SWEEP_ROWS = (16384, 32768, 65536, 131072)


def run_sweep(args) -> dict:
    """Config 3: TensorProduct over m_max 1-6 x C {32, 64, 96, 128, 256} x parity x
    N {16,384, 32,768, 65,536, 131,072}, iid N(0, 1) inputs (seed per shape), ones
    cotangent; the forward and the forward + VJP are each captured in a CUDA graph
    (so host launch time does not enter the small shapes' figures) and each replay
    is timed alone with CUDA events, after an L2 flush (a 256 MB write); median of
    the steps."""
    import torch
    from ictc_o2_hp_b200 import TensorProduct, ops
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    hbm = float(peaks()[0]["hbm_gbs"])
    steps = max(3, min(args.steps, 10))
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=device)

    def median_ms(graph):
        for _ in range(2):
            graph.replay()
        times = []
        for _ in range(steps):
            flush.fill_(1.0)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b))
        return statistics.median(times)

    def capture(fn):
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(2):
                fn()  # warm-up outside the capture (allocations, smem opt-in)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        return graph

    shapes = []
    launches = 0
    with ClockSampler(0) as clocks:
        for channels in SWEEP_CHANNELS:
            for m_max in SWEEP_M_MAX:
                for parity in SWEEP_PARITY:
                    torch.manual_seed(channels * 100 + m_max * 10 + (parity == "full"))
                    tp = TensorProduct(channels, m_max, parity=parity).to(device)
                    W = tp.representation_dimension
                    top = max(SWEEP_ROWS)
                    x = torch.randn(top, W, device=device)
                    y = torch.randn(top, W, device=device)
                    g = torch.ones(top, W, device=device)
                    w = tp.weight.detach()
                    cfg = (channels, m_max, parity, "component")
                    for rows in SWEEP_ROWS:
                        xs, ys, gs = x[:rows], y[:rows], g[:rows]
                        fwd_graph = capture(lambda: ops.tp_forward(xs, ys, w, *cfg))
                        both_graph = capture(lambda: (ops.tp_forward(xs, ys, w, *cfg),
                                                      ops.tp_backward(xs, ys, w, gs, *cfg)))
                        fwd = median_ms(fwd_graph)
                        both = median_ms(both_graph)
                        del fwd_graph, both_graph
                        # each forward kernel the dispatcher chooses between, forced
                        variants = {}
                        for variant in ("grouped", "wide"):
                            os.environ["ICTC_TP_FORWARD"] = variant
                            try:
                                vg = capture(lambda: ops.tp_forward(xs, ys, w, *cfg))
                                variants[variant] = median_ms(vg)
                                del vg
                            finally:
                                del os.environ["ICTC_TP_FORWARD"]
                        launches += 5 * (steps + 2)
                        shapes.append({
                            "channels": channels, "m_max": m_max, "parity": parity,
                            "rows": rows, "width": W, "fwd_ms": fwd, "fwd_vjp_ms": both,
                            "fwd_variant_ms": variants,
                            "fwd_hbm_frac": 12 * W * rows / (fwd * 1e-3) / 1e9 / hbm,
                            "fwd_vjp_hbm_frac": 32 * W * rows / (both * 1e-3) / 1e9 / hbm})
                    del x, y, g, tp
                    torch.cuda.empty_cache()
    fracs = [s["fwd_vjp_hbm_frac"] for s in shapes]
    geo = math.exp(sum(math.log(f) for f in fracs) / len(fracs))
    total_ms = sum(s["fwd_vjp_ms"] for s in shapes)
    return {
        "metric": "TensorProduct shape sweep (config 3): geometric mean over 240 shapes of the "
                  "fwd+VJP fraction of measured HBM (32 W B per row)",
        "value": geo, "unit": "fraction of measured HBM", "n_gpus": 1, "steps": steps,
        "warmup": 2, "ms_per_step": total_ms, "higher_is_better": True, "scaling": "none",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded iid N(0,1) inputs, seeded init, ones cotangent)",
        "config": {"workload": "m_max 1-6 x C {32,64,96,128,256} x parity {canonical, full} x "
                               "N {16384, 32768, 65536, 131072}; forward and forward + VJP "
                               "(forward and backward launches) timed separately, each as a "
                               "CUDA graph replay",
                   "l2": "L2 flushed (256 MB write) before every timed replay"},
        "gpu_launches": launches, "clocks": clocks.summary(), "shapes": shapes}


# ------------------------------------------------------------------ reference arm

def run_reference(args) -> dict | None:
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    if args.workload not in CPU_ROWS:
        why = {"radial_mp": "the reference has no message-passing layer (gather and scatter "
                            "are outside its chain)",
               "sweep": "the shape sweep is timed on the GPU only; the CPU reference arm "
                        "runs on the single-config workloads"}.get(
            args.workload, "the CPU oracle has no second derivatives (force-loss metric)")
        return {"impl": "reference", "unavailable": why}
    if reference_cpu_available():
        rows = args.cpu_rows or REF_CPU_ROWS[args.workload]
        base = reference_cpu_units_per_second(args.workload, rows, args.steps,
                                              max(1, min(args.warmup, 1)), args.channels)
        how = "reference package's own CPU path"
        per_step_ms = rows / base["value"] * 1e3
    else:
        rows = args.cpu_rows or CPU_ROWS[args.workload]
        base = cpu_units_per_second(args.workload, rows, args.steps,
                                    max(1, min(args.warmup, 1)), args.channels)
        how = "reference algorithm, numpy port, per core"
        per_step_ms = rows * base["cores"] / base["value"] * 1e3
    value = base["value"]
    return {
        "metric": METRICS[args.workload].format(channels=args.channels), "impl": "reference",
        "value": value,
        "unit": base["unit"], "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_step_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded iid N(0,1) inputs, ones cotangent)",
        "config": {"workload": f"{args.workload} forward + VJP on the host CPU ({how}), "
                               f"bounded sample of {rows} rows per step"},
        "cpu_baseline": base,
        "e2e": {"value": value, "unit": base["unit"], "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ------------------------------------------------------------------ reference GPU path

def run_reference_gpu(args) -> dict | None:
    """The reference package's own public API on this GPU (its Triton kernels, which
    it picks for CUDA float32 inputs), on the same workload, seeds and timing as the
    ours arm: TensorProduct config 2 (default), uvu config 4 (shared weights) or the
    radial product of config 5 (--workload tp | uvu | radial; the radial network in
    front of the product is the same PyTorch MLP).  It needs the reference installed
    under baseline/_ref (pip install --target); without it the line says unavailable.
    One GPU, rank 0 (other ranks exit without work)."""
    import torch
    if int(os.environ.get("RANK", "0")) != 0:
        return None
    ref_dir = ROOT / "baseline" / "_ref"
    base = {"impl": "reference_gpu", "metric": METRICS.get(args.workload, args.workload)}
    if not (ref_dir / "ictc_o2_hp").is_dir():
        return {**base, "unavailable": "the reference package is not installed under "
                                       "baseline/_ref"}
    if args.workload not in ("tp", "uvu", "radial"):
        return {**base, "unavailable": f"no reference GPU leg for workload {args.workload}"}
    sys.path.insert(0, str(ref_dir))
    import ictc_o2_hp as ref
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    gen = torch.Generator(device=device)
    if args.workload == "tp":
        rows = args.rows or 65536
        torch.manual_seed(0)
        tp = ref.TensorProduct(128, 6, parity="full").to(device)
        W = tp.representation_dimension
        gen.manual_seed(1000)
        x = torch.randn(rows, W, device=device, generator=gen).requires_grad_(True)
        y = torch.randn(rows, W, device=device, generator=gen).requires_grad_(True)
        g = torch.ones(rows, W, device=device)
        params, inputs = [tp.weight], (x, y)

        def step():
            return torch.autograd.grad(tp(x, y), [x, y] + params, g)
        workload = ("TensorProduct(128, 6, parity='full') forward + VJP (dx, dy, dw), "
                    f"{rows} rows, ones cotangent")
    elif args.workload == "uvu":
        rows = args.rows or 131072
        torch.manual_seed(0)
        tp = ref.UvuTensorProduct(128, 32, 3).to(device)
        with torch.no_grad():
            tp.weight.copy_(torch.randn(tp.weight_numel, device=device) / 32 ** 0.5)
        gen.manual_seed(2000)
        x = torch.randn(rows, tp.input1_dimension, device=device, generator=gen)
        y = torch.randn(rows, tp.input2_dimension, device=device, generator=gen)
        x.requires_grad_(True)
        y.requires_grad_(True)
        g = torch.ones(rows, tp.input1_dimension, device=device)
        params = [tp.weight]

        def step():
            return torch.autograd.grad(tp(x, y), [x, y] + params, g)
        workload = (f"UvuTensorProduct(128, 32, 3, parity='full') shared weights, forward + "
                    f"VJP (dx, dy, dw), {rows} rows")
    else:
        rows = args.rows or RadialWorkload.EDGES
        torch.manual_seed(0)
        tp = ref.UvuTensorProduct(64, 1, 3, parity="full", parity_in2="canonical",
                                  shared_weights=False)
        trunk = torch.nn.Sequential(torch.nn.Linear(8, 64), torch.nn.SiLU(),
                                    torch.nn.Linear(64, 64), torch.nn.SiLU()).to(device)
        model = ref.RadialUvuTensorProduct(
            tp, torch.nn.Linear(64, tp.weight_numel, bias=False)).to(device)
        gen.manual_seed(3000)
        nodes = torch.randn(RadialWorkload.NODES, tp.input1_dimension, device=device,
                            generator=gen)
        src = torch.randint(0, RadialWorkload.NODES, (rows,), device=device, generator=gen)
        torch.randint(1, RadialWorkload.NODES, (rows,), device=device, generator=gen)
        r = torch.rand(rows, device=device, generator=gen) * 4.5 + 0.5
        theta = torch.rand(rows, device=device, generator=gen) * 2 * math.pi
        x = nodes[src].contiguous().requires_grad_(True)
        y = torch.stack([torch.ones_like(theta)] + [
            f(m * theta) for m in range(1, 4) for f in (torch.cos, torch.sin)],
            dim=-1).contiguous().requires_grad_(True)
        g = torch.ones(rows, tp.input1_dimension, device=device)
        params = list(trunk.parameters()) + list(model.parameters())
        n = torch.arange(1, 9, device=device, dtype=r.dtype)
        rc = RadialWorkload.RC

        def step():
            basis = (math.sqrt(2 / rc) * torch.sin(n * math.pi * r[:, None] / rc) / r[:, None]
                     * (0.5 * (torch.cos(math.pi * r / rc) + 1))[:, None])
            out = model(x, y, trunk(basis))
            return torch.autograd.grad(out, [x, y] + params, g)
        workload = (f"RadialUvuTensorProduct C64 m3 (config 5 product), {rows} edges, radial MLP "
                    "8-64-64 SiLU in front, forward + VJP through the radial network")
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clocks:
        time.sleep(0.3)
        a.record()
        for _ in range(args.steps):
            step()
        b.record()
        torch.cuda.synchronize()
        time.sleep(0.2)
    ms = a.elapsed_time(b) / args.steps
    unit = "edges/s" if args.workload == "radial" else "rows/s"
    return {**base, "value": rows / (ms * 1e-3), "unit": unit, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "dtype": "f32", "data": "synthetic (same seeds as the "
            "ours arm)", "config": {"workload": workload, "path": "reference public API, CUDA "
                                    "float32 inputs (its Triton kernels)"},
            "clocks": clocks.summary()}


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__,
                                     formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference", "reference_gpu"), default="ours",
                        help="reference: the reference algorithm on the host cores (the "
                             "comparison arm); reference_gpu: the reference package's own "
                             "Triton path on this GPU, when installed under baseline/_ref")
    parser.add_argument("--workload", choices=tuple(WORKLOADS) + ("sweep",), default="tp")
    parser.add_argument("--rows", type=int, default=0,
                        help="rows per GPU (tp, uvu) or total edges (radial); 0 = config")
    parser.add_argument("--channels", type=int, default=64,
                        help="radial_m6: channels C of the published chain (64, 128, 256)")
    parser.add_argument("--cpu-rows", type=int, default=0,
                        help="rows per host core per CPU-baseline step; 0 = default")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--node-partition", action="store_true",
                        help="radial_mp with N > 1: node blocks per rank (all-gather of node "
                             "features, reduce-scatter of node outputs and node gradients)")
    parser.add_argument("--no-radial-scaling", action="store_true",
                        help="tp workload: skip the config-5 strong-scaling companion line")
    args = parser.parse_args(argv)
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")

    if args.impl in ("reference", "reference_gpu"):
        result = run_reference(args) if args.impl == "reference" else run_reference_gpu(args)
        if result is not None:
            print(json.dumps(result), flush=True)
        return 0

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.workload == "sweep":
        if rank == 0:
            print(json.dumps(run_sweep(args)), flush=True)
        return 0
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.workload in CPU_ROWS:
        # The process pool starts before the first CUDA call (spawned workers).
        if reference_cpu_available():
            cpu = reference_cpu_units_per_second(
                args.workload, args.cpu_rows or REF_CPU_ROWS[args.workload], 3, 1, args.channels)
        else:
            cpu = cpu_units_per_second(args.workload, args.cpu_rows or CPU_ROWS[args.workload],
                                       3, 1, args.channels)
    result = run_gpu(args)
    if result is not None:
        if cpu is not None:
            result["cpu_baseline"] = cpu
        print(json.dumps(result), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
