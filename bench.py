#!/usr/bin/env python3
"""Benchmark of the packed-affine B3 block matmul (metric: Q4 GEMV/B3 HBM GB/s).

Workload (default `b3`): one step = one block matmul of a Q4/group-64
17408x5120 matrix with BF16 scale/bias against 3 FP32 activation rows (one
target + two MTP proposals), the R2-eligible gate/up shape.  Inputs are
seeded synthetic data with the benchmark distributions (no dataset exists for
this path).  Steps rotate over enough distinct weight copies to exceed 4x the
L2 size, so every step streams its weights from HBM.

Other workloads (--workload): b1 (same matrix, one RHS), q8b3 (Q8 config),
mlp (gate/up SwiGLU + down at B3), head (152064-row vocabulary head + argmax).

Multi-GPU: one process per GPU (torchrun); each rank runs the same workload
on its own weights (independent matrices, no data-path collective), value =
all ranks' bytes / max-over-ranks time ("scaling": "weak").

--impl reference times the reference's CPU path on the host cores instead:
the FP64 oracle restatement (oracle/), a bounded sample of rows per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import pathlib
import statistics
import subprocess
import sys
import time

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "qwen-mlx-runner_b200"))

import numpy as np  # noqa: E402

ROWS, COLS, GROUP = 17408, 5120, 64
VOCAB = 152064
METRIC = "Q4 GEMV/B3 HBM GB/s"


def matrix_bytes(rows, cols, bits, group):
    return rows * cols * bits // 8 + 2 * (rows * cols // group) * 2


def workload_spec(name):
    """(description, per-step algorithmic bytes, bits, batch)."""
    if name == "b3":
        return dict(desc="Q4/g64 BF16-metadata B3 block matmul 17408x5120", bits=4, batch=3, rows=ROWS,
                    cols=COLS)
    if name == "b1":
        return dict(desc="Q4/g64 BF16-metadata B1 GEMV 17408x5120", bits=4, batch=1, rows=ROWS, cols=COLS)
    if name == "q8b3":
        return dict(desc="Q8/g64 BF16-metadata B3 block matmul 17408x5120", bits=8, batch=3, rows=ROWS, cols=COLS)
    if name == "mlp":
        return dict(desc="Q4/g64 SwiGLU MLP at B3: fused gate/up 17408x5120 + down 5120x17408", bits=4, batch=3,
                    rows=ROWS, cols=COLS)
    if name == "head":
        return dict(desc="Q4/g64 vocabulary head 152064x5120 + argmax at B3", bits=4, batch=3, rows=VOCAB,
                    cols=COLS)
    raise SystemExit(f"unknown workload {name}")


def algorithmic_bytes(name, spec):
    b, bits = spec["batch"], spec["bits"]
    if name == "mlp":
        up = matrix_bytes(ROWS, COLS, 4, GROUP)
        down = matrix_bytes(COLS, ROWS, 4, GROUP)
        # weights+metadata of 3 matrices, x read, activation write + read, output write
        return 2 * up + down + 4 * b * COLS + 2 * 4 * b * ROWS + 4 * b * COLS
    rows, cols = spec["rows"], spec["cols"]
    return matrix_bytes(rows, cols, bits, GROUP) + 4 * b * cols + 4 * b * rows


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(workload):
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summaries (profiles/traffic.txt: `workload bytes` lines), or None."""
    p = ROOT / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) == 2 and not line.startswith("#") and parts[0] == workload:
            return float(parts[1])
    return None


class Clocks:
    """nvidia-smi sampler for the timed region (sm clock, throttle reasons)."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            self.path = f"/tmp/qmr_clocks_{os.getpid()}.csv"
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


# ---------------------------------------------------------------------------
# CPU reference arm
# ---------------------------------------------------------------------------

def cpu_sample(name, spec, rows_sample, seed=1):
    """Time the FP64 oracle on rows_sample rows of the workload; returns (seconds, bytes)."""
    import oracle
    from qmr import synth
    bits, b = spec["bits"], spec["batch"]
    cols = spec["cols"]
    mat = synth.affine_matrix(rows_sample, cols, bits, GROUP, seed=seed)
    x = synth.activations(b, cols, seed=seed + 1)
    t0 = time.perf_counter()
    oracle.matmul_f64(mat["weight"], mat["scales"], mat["biases"], x, rows_sample, cols, bits, GROUP, batch=b)
    dt = time.perf_counter() - t0
    full_rows = spec["rows"]
    nbytes = algorithmic_bytes(name, spec) * rows_sample / full_rows
    return dt, nbytes


def calibrate_rows(name, spec, target_s):
    rows = 64
    dt, _ = cpu_sample(name, spec, rows)
    per_row = max(dt / rows, 1e-7)
    return max(16, min(spec["rows"], int(target_s / per_row)))


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    import oracle
    spec = workload_spec(args.workload)
    threads = oracle.threads()
    # Bound the whole run to about a minute: per-step sample sized from K+W.
    total_steps = args.steps + args.warmup
    per_step = max(0.005, min(0.25, 60.0 / max(total_steps, 1)))
    rows = calibrate_rows(args.workload, spec, per_step)
    for _ in range(args.warmup):
        cpu_sample(args.workload, spec, rows)
    secs, nbytes = 0.0, 0.0
    for _ in range(args.steps):
        dt, nb = cpu_sample(args.workload, spec, rows)
        secs += dt
        nbytes += nb
    value = nbytes / secs / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded; benchmark distributions)",
        "config": {"workload": spec["desc"], "cpu_rows_per_step": rows},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} of {spec['rows']} rows per step, FP64 oracle (tests/quantized.rs:39-51 "
                                   "restated in oracle/oracle.c), OpenMP over rows"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def sharded(name, world):
    """The MLP and the head run row-sharded across the ranks (one model split
    over N GPUs, strong scaling); the single matrices run one replica per
    rank (weak scaling)."""
    return world > 1 and name in ("mlp", "head")


class Workload:
    def __init__(self, name, spec, device, seed, world=1, rank=0, exchange="p2p"):
        import torch

        from qmr import synth
        self.name, self.spec, self.device = name, spec, device
        self.torch = torch
        bits, b = spec["bits"], spec["batch"]
        self.batch = b
        self.sharded = sharded(name, world)
        self.exchange = exchange
        if self.sharded:
            self._init_sharded(world, rank, seed)
            return
        per_copy = (matrix_bytes(ROWS, COLS, 4, GROUP) * 3) if name == "mlp" else \
            matrix_bytes(spec["rows"], spec["cols"], bits, GROUP)
        l2 = torch.cuda.get_device_properties(device).L2_cache_size
        self.copies = max(2, math.ceil(4 * l2 / per_copy) + 1)
        self.l2 = l2
        self.x = torch.from_numpy(synth.activations(b, COLS, seed=seed + 1).ravel()).to(device)

        def dev_matrix(rows, cols, s):
            m = synth.affine_matrix(rows, cols, bits, GROUP, seed=s)
            return synth.to_device(m, rows, cols, bits, GROUP, device)

        def clone(m):
            from qmr.ops import PackedMatrix
            return PackedMatrix(m.weight.clone(), m.scales.clone(), m.biases.clone(), m.rows, m.cols, m.bits,
                                m.group)

        if name == "mlp":
            g0 = dev_matrix(ROWS, COLS, seed + 10)
            u0 = dev_matrix(ROWS, COLS, seed + 11)
            d0 = dev_matrix(COLS, ROWS, seed + 12)
            self.mats = [(clone(g0), clone(u0), clone(d0)) for _ in range(self.copies)]
            self.act = torch.empty(b * ROWS, dtype=torch.float32, device=device)
            self.y = torch.empty(b * COLS, dtype=torch.float32, device=device)
        else:
            m0 = dev_matrix(spec["rows"], spec["cols"], seed + 10)
            self.mats = [clone(m0) for _ in range(self.copies)]
            self.y = torch.empty(b * spec["rows"], dtype=torch.float32, device=device)
            self.idx = torch.empty(b, dtype=torch.int32, device=device)
        self.launches_per_step = 2 if name == "mlp" else 1

    def _init_sharded(self, world, rank, seed):
        """This rank's row shards (random init of this rank's rows only)."""
        import math

        import torch

        import qmr
        from qmr import parallel, synth
        from qmr.ops import PackedMatrix
        b, dev = self.batch, self.device
        l2 = torch.cuda.get_device_properties(dev).L2_cache_size
        self.l2 = l2

        def dev_matrix(rows, cols, s):
            m = synth.affine_matrix(rows, cols, 4, GROUP, seed=s)
            return synth.to_device(m, rows, cols, 4, GROUP, dev)

        def clone(m):
            return PackedMatrix(m.weight.clone(), m.scales.clone(), m.biases.clone(), m.rows, m.cols, m.bits,
                                m.group)

        self.x = torch.from_numpy(synth.activations(b, COLS, seed=seed + 1).ravel()).to(dev)
        s = seed + 100 * rank
        if self.name == "mlp":
            f0, f1 = parallel.shard_range(ROWS, world, rank)
            h0, h1 = parallel.shard_range(COLS, world, rank)
            g0, u0 = dev_matrix(f1 - f0, COLS, s + 10), dev_matrix(f1 - f0, COLS, s + 11)
            d0 = dev_matrix(h1 - h0, ROWS, s + 12)
            per_copy = g0.nbytes + u0.nbytes + d0.nbytes
            self.copies = max(2, math.ceil(4 * l2 / per_copy) + 1)
            self.mods = [parallel.ShardedMLP(clone(g0), clone(u0), clone(d0), COLS, ROWS, qmr.ops,
                                             exchange=self.exchange) for _ in range(self.copies)]
            self.y = torch.empty(b * COLS, dtype=torch.float32, device=dev)
            self.launches_per_step = 2
        else:
            v0, v1 = parallel.shard_range(VOCAB, world, rank)
            h = dev_matrix(v1 - v0, COLS, s + 10)
            self.copies = max(2, math.ceil(4 * l2 / h.nbytes) + 1)
            self.mods = [parallel.ShardedHead(clone(h), VOCAB, v0, qmr.ops, exchange=self.exchange)
                         for _ in range(self.copies)]
            self.y = torch.empty(b * (v1 - v0), dtype=torch.float32, device=dev)
            self.idx = torch.empty(b, dtype=torch.int32, device=dev)
            self.launches_per_step = 1

    def step(self, i, stream=None, x=None):
        """One call of the workload; x (default: the device activations) may
        be a pinned host tensor, which the kernels read over the host link."""
        import qmr
        x = self.x if x is None else x
        if self.sharded:
            mod = self.mods[i % self.copies]
            if self.name == "mlp":
                mod(x, self.batch, out=self.y)
            else:
                idx, _ = mod(x, self.batch, logits=self.y)
                self.idx.copy_(idx)
            return
        m = self.mats[i % self.copies]
        if self.name == "mlp":
            g, u, d = m
            qmr.gateup_swiglu(g, u, x, self.act, self.batch, stream=stream)
            qmr.matmul_affine(d, self.act, self.y, self.batch, stream=stream)
        elif self.name == "head":
            qmr.head_argmax(m, x, self.y, self.idx, self.batch, stream=stream)
        elif self.batch == 1:
            qmr.matvec_affine(m, x, self.y, stream=stream)
        else:
            qmr.matmul_affine(m, x, self.y, self.batch, stream=stream)


def kernel_only_ms(wl, stream, steps):
    """Average duration of the streaming kernel alone: prepare the activations
    once, then time `steps` launches (rotating weight copies) in one graph."""
    import torch

    import qmr
    spec = wl.spec
    prepared = qmr.ops.alloc_prepared(spec["bits"], spec["cols"], wl.batch, wl.device)
    n = min(steps, 1000)
    with torch.cuda.stream(stream):
        qmr.ops.prepare_activations(wl.x, spec["cols"], spec["bits"], wl.batch, prepared, stream=stream)
        for i in range(3):
            qmr.ops.matmul_prepared(wl.mats[i % wl.copies], prepared, wl.y, wl.batch, stream=stream)
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(n):
            qmr.ops.matmul_prepared(wl.mats[i % wl.copies], prepared, wl.y, wl.batch, overlap=True, stream=stream)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        g.replay()
        e0.record(stream)
        g.replay()
        e1.record(stream)
    stream.synchronize()
    return e0.elapsed_time(e1) / n


def run_gpu(args):
    import torch
    import torch.distributed as dist

    import qmr
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    qmr.ops.init(local)
    spec = workload_spec(args.workload)
    wl = Workload(args.workload, spec, device, seed=1000 + 17 * rank, world=world, rank=rank, exchange=args.exchange)
    nbytes = algorithmic_bytes(args.workload, spec)
    # Replicas: every rank processes nbytes per step.  Shards: the ranks
    # together process one model's nbytes per step.
    job_factor = 1 if wl.sharded else world

    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            wl.step(i, stream)
    torch.cuda.synchronize()

    # Capture the timed steps into CUDA graphs of at most CHUNK steps each.
    CHUNK = 1000
    graphs = []
    done = 0
    while done < args.steps:
        n = min(CHUNK, args.steps - done)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                wl.step(done + i, stream)
        graphs.append(g)
        done += n
    # Warm the graphs (untimed).
    for g in graphs[:1]:
        g.replay()
    torch.cuda.synchronize()

    clocks = Clocks(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    # CUDAGraph.replay launches on the current stream: keep events and
    # replays on the same stream.
    with torch.cuda.stream(stream):
        start.record(stream)
        for g in graphs:
            g.replay()
        end.record(stream)
    stream.synchronize()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    # Keep the GPU in the same loop until the clock sampler has seen >= 1.5 s
    # of it (untimed; only the first pass above is reported).  The count comes
    # from the slowest rank's time, so every rank replays the same exchanges.
    extra = 0 if args.quick else min(400, int(math.ceil(1500.0 / max(ms_max, 1e-3))))
    with torch.cuda.stream(stream):
        for _ in range(extra):
            for g in graphs:
                g.replay()
    stream.synchronize()
    clk = clocks.stop()
    torch.cuda.synchronize()
    kernel_ms = kernel_only_ms(wl, stream, args.steps) if args.workload in ("b3", "b1", "q8b3") else None
    ms_per_step = ms_max / args.steps
    value = job_factor * nbytes * args.steps / (ms_max * 1e-3) / 1e9

    # End to end through the public API: pinned host x in, result out, every
    # step.  The call takes x straight from pinned host memory (the prep
    # kernel reads it over the host link: the step's host-to-device
    # transfer); qmr_copy_f32 writes the result into pinned host memory (the
    # device-to-host transfer, a kernel chained behind the call).
    e2e_steps = min(args.steps, 200 if args.quick else 2000)
    h2d = wl.x.numel() * 4
    out = wl.y if args.workload != "head" else wl.idx
    d2h = out.numel() * out.element_size()
    xh = torch.empty(wl.x.numel(), dtype=torch.float32, pin_memory=True)
    xh.copy_(wl.x.cpu())
    yh = torch.empty(out.numel(), dtype=out.dtype, pin_memory=True)
    with torch.cuda.stream(stream):
        for i in range(3):
            wl.step(i, stream, x=xh)
            qmr.ops.copy_f32(out, yh, out.numel(), stream=stream)
    stream.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(e2e_steps):
            wl.step(i, stream, x=xh)
            qmr.ops.copy_f32(out, yh, out.numel(), stream=stream)
        e1.record(stream)
    stream.synchronize()
    te = torch.tensor([e0.elapsed_time(e1)], device=device)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = job_factor * nbytes * e2e_steps / (float(te.item()) * 1e-3) / 1e9

    peak, peak_kind = load_peaks()
    if kernel_ms is not None:
        kernel_nbytes = nbytes  # the streaming kernel reads weights, x' and writes y
        achieved = kernel_nbytes / (kernel_ms * 1e-3) / 1e9
        timing_note = "streaming kernel alone: activations prepared once, K launches in one graph"
    else:
        # per GPU: its share of the job's bytes over the step time
        achieved = job_factor * nbytes / world / (ms_per_step * 1e-3) / 1e9
        timing_note = "whole call" + (f", sharded step incl. the {wl.exchange} exchange" if wl.sharded else "")
    traffic = profile_traffic(args.workload)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
        "scaling": "strong" if wl.sharded else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded; benchmark distributions)",
        "config": {"workload": spec["desc"], "batch": spec["batch"], "rows": spec["rows"], "cols": spec["cols"],
                   "bits": spec["bits"], "group": GROUP, "metadata": "bf16", "weight_copies": wl.copies,
                   "l2_bytes": wl.l2, "l2_policy": f"{wl.copies} distinct weight copies rotated (> 4x L2)",
                   "bytes_per_step": nbytes,
                   "parallelism": (f"rowshard{world} ({'peer-memory exchange in the kernels' if wl.exchange == 'p2p' else 'NCCL all-gather'})"
                                   if wl.sharded else
                                   f"replicas{world}" if world > 1 else "single")},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} hbm_gbs", "timing": timing_note,
                     "kernel_ms": None if kernel_ms is None else round(kernel_ms, 6)},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.quick):
        import oracle
        rows = calibrate_rows(args.workload, spec, 2.0)
        secs, nb = 0.0, 0.0
        for i in range(5):
            dt, b = cpu_sample(args.workload, spec, rows, seed=3 + i)
            secs += dt
            nb += b
        line["cpu_baseline"] = {"value": round(nb / secs / 1e9, 4), "unit": "GB/s", "cores": oracle.threads(),
                                "kind": "port",
                                "sample": f"5 x {rows} of {spec['rows']} rows, FP64 oracle, OpenMP over rows"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        # Every graph that holds NCCL calls must be gone before the process
        # group is destroyed (the loop variable above holds one too).
        g = None
        graphs.clear()
        del graphs, g
        import gc
        gc.collect()
        torch.cuda.synchronize()
        if wl.sharded:
            for m in wl.mods:
                m.close()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="qmr", choices=["qmr", "reference"])
    ap.add_argument("--workload", default="b3", choices=["b3", "b1", "q8b3", "mlp", "head"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="sharded workloads: output exchange over peer memory in the kernels, or NCCL all-gathers")
    ap.add_argument("--quick", action="store_true",
                    help="profiling runs: no clock-sampling loop, short e2e, no CPU baseline")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
