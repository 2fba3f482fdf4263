#!/usr/bin/env python3
"""Benchmark of the packed-affine B3 block matmul (metric: Q4 GEMV/B3 HBM GB/s).

Headline workload (`b3`): one step = one block matmul of a Q4/group-64
17408x5120 matrix with BF16 scale/bias against 3 FP32 activation rows (one
target + two MTP proposals), the R2-eligible gate/up shape.  Inputs are
seeded synthetic data with the benchmark distributions (no dataset exists for
this path).  Steps rotate over enough distinct weight copies to exceed 4x the
L2 size, so every step streams its weights from HBM.

The same JSON line also carries, measured in the same run:
  * `workloads`: the B1 GEMV (config 0) and the Q8 B3 block (config 1), each
    as whole-call GB/s and as the streaming kernel alone, over a fixed 200
    calls;
  * `sharded`: the SwiGLU MLP (config 2) and the vocabulary head + argmax
    (config 3).  At N=1 the unsharded call; under torchrun (N>1) the rows are
    split over the ranks (strong scaling, outputs exchanged over peer memory
    inside the kernels), timed as the max over ranks, and checked against the
    1-GPU call on rank 0;
  * `reps200`: the headline call timed over a fixed 200 calls, comparable
    between runs whatever --steps is;
  * `decode`: config 4, the synthetic 64-layer 27B-shaped hybrid: prefill a
    seeded 512-token prompt and greedily decode 128 tokens at context 4096
    through the engine (qmr_model_generate), decode tokens/s; under
    torchrun the model split tensor-parallel over the ranks (one token
    stream for the job, strong scaling).

Multi-GPU headline: one process per GPU (torchrun); each rank runs the b3
call on its own weights (independent matrices, no data-path collective),
value = all ranks' bytes / max-over-ranks time ("scaling": "weak").

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
ARITH = ("tensor cores (mma.sync m16n8k16): exact fp16-subnormal Q4/Q8 weights x activations split into "
         "fp16 high + low parts with a per-group exponent (about 22 significant bits), f32 accumulation and "
         "f32 scale/bias fold; FP32 activations in, FP32 outputs")
FIXED_REPS = 200


def matrix_bytes(rows, cols, bits, group):
    return rows * cols * bits // 8 + 2 * (rows * cols // group) * 2


def workload_spec(name):
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


def config_of(spec):
    """The `config` object both arms print for a workload."""
    return {"workload": spec["desc"], "batch": spec["batch"], "rows": spec["rows"], "cols": spec["cols"],
            "bits": spec["bits"], "group": GROUP, "metadata": "bf16"}


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

def host_threads():
    """Every host core this process may run on (torchrun sets OMP_NUM_THREADS=1
    for its children; the CPU baseline is measured on all cores regardless)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


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
    oracle.set_threads(host_threads())
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
    config = config_of(spec)
    config["cpu_rows_per_step"] = rows
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded; benchmark distributions)",
        "config": config,
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{rows} of {spec['rows']} rows per step (the same workload, a bounded row "
                                   "sample), FP64 oracle (tests/quantized.rs:39-51 restated in oracle/oracle.c), "
                                   "OpenMP over rows on all host cores"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def _synth_matrix(rows, cols, bits, seed, device):
    from qmr import synth
    m = synth.affine_matrix(rows, cols, bits, GROUP, seed=seed)
    return synth.to_device(m, rows, cols, bits, GROUP, device)


def _clone(m):
    from qmr.ops import PackedMatrix
    return PackedMatrix(m.weight.clone(), m.scales.clone(), m.biases.clone(), m.rows, m.cols, m.bits, m.group)


def _copies(l2, per_copy):
    return max(2, math.ceil(4 * l2 / per_copy) + 1)


class Workload:
    """One workload on this rank: its weight copies (> 4x L2 in total), its
    input and outputs, and one call per step through the public API."""

    def __init__(self, name, device, seed, world=1, rank=0, shard=False, exchange="p2p"):
        import torch

        from qmr import synth
        spec = workload_spec(name)
        self.name, self.spec, self.device = name, spec, device
        self.batch = b = spec["batch"]
        self.sharded = shard and world > 1
        self.exchange = exchange
        self.world, self.rank, self.seed = world, rank, seed
        self.l2 = torch.cuda.get_device_properties(device).L2_cache_size
        self.x = torch.from_numpy(synth.activations(b, COLS, seed=seed + 1).ravel()).to(device)
        if self.sharded:
            self._init_sharded()
            return
        bits = spec["bits"]
        if name == "mlp":
            g0 = _synth_matrix(ROWS, COLS, bits, seed + 10, device)
            u0 = _synth_matrix(ROWS, COLS, bits, seed + 11, device)
            d0 = _synth_matrix(COLS, ROWS, bits, seed + 12, device)
            self.copies = _copies(self.l2, g0.nbytes + u0.nbytes + d0.nbytes)
            self.mats = [(_clone(g0), _clone(u0), _clone(d0)) for _ in range(self.copies)]
            self.act = torch.empty(b * ROWS, dtype=torch.float32, device=device)
            self.y = torch.empty(b * COLS, dtype=torch.float32, device=device)
            # fused gate/up, down: each streaming kernel builds its activation image
            self.launches_per_step = 2
        else:
            m0 = _synth_matrix(spec["rows"], spec["cols"], bits, seed + 10, device)
            self.copies = _copies(self.l2, m0.nbytes)
            self.mats = [_clone(m0) for _ in range(self.copies)]
            self.y = torch.empty(b * spec["rows"], dtype=torch.float32, device=device)
            self.idx = torch.empty(b, dtype=torch.int32, device=device)
            # the streaming kernel (building its activation image); the head's
            # argmax epilogue keeps the separate activation prep
            self.launches_per_step = 2 if name == "head" else 1

    def shard_seed(self, r):
        return self.seed + 100 * r

    def _init_sharded(self):
        """This rank's row shards (random init of this rank's rows only)."""
        import torch

        import qmr
        from qmr import parallel
        b, dev, world, rank = self.batch, self.device, self.world, self.rank
        s = self.shard_seed(rank)
        if self.name == "mlp":
            f0, f1 = parallel.shard_range(ROWS, world, rank)
            h0, h1 = parallel.shard_range(COLS, world, rank)
            g0, u0 = _synth_matrix(f1 - f0, COLS, 4, s + 10, dev), _synth_matrix(f1 - f0, COLS, 4, s + 11, dev)
            d0 = _synth_matrix(h1 - h0, ROWS, 4, s + 12, dev)
            self.copies = _copies(self.l2, g0.nbytes + u0.nbytes + d0.nbytes)
            self.mods = [parallel.ShardedMLP(_clone(g0), _clone(u0), _clone(d0), COLS, ROWS, qmr.ops,
                                             exchange=self.exchange) for _ in range(self.copies)]
            self.y = torch.empty(b * COLS, dtype=torch.float32, device=dev)
            # p2p: prep + gate/up + exchange wait, prep + down + exchange wait;
            # nccl: gate/up and down, each building its image (+ NCCL's own kernels)
            self.launches_per_step = 6 if self.exchange == "p2p" else 2
        else:
            v0, v1 = parallel.shard_range(VOCAB, world, rank)
            h = _synth_matrix(v1 - v0, COLS, 4, s + 10, dev)
            self.copies = _copies(self.l2, h.nbytes)
            self.mods = [parallel.ShardedHead(_clone(h), VOCAB, v0, qmr.ops, exchange=self.exchange)
                         for _ in range(self.copies)]
            self.y = torch.empty(b * (v1 - v0), dtype=torch.float32, device=dev)
            self.idx = torch.empty(b, dtype=torch.int32, device=dev)
            self.launches_per_step = 3 if self.exchange == "p2p" else 2  # prep + head (+ wait)

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

    def close(self):
        if self.sharded:
            for m in self.mods:
                m.close()


def capture(wl, stream, n, start=0):
    """CUDA graphs (at most 1000 calls each) of n consecutive steps."""
    import torch
    graphs, done = [], 0
    while done < n:
        k = min(1000, n - done)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(k):
                wl.step(start + done + i, stream)
        graphs.append(g)
        done += k
    return graphs


def replay_ms(graphs, stream):
    """Device time of one replay of every graph, with events on the replay stream."""
    import torch
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for g in graphs:
            g.replay()
        e1.record(stream)
    stream.synchronize()
    return e0.elapsed_time(e1)


def max_over_ranks(v, device, world):
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(v)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


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
    replay_ms([g], stream)
    return replay_ms([g], stream) / n


def warm(wl, stream, n=3):
    import torch
    with torch.cuda.stream(stream):
        for i in range(n):
            wl.step(i, stream)
    torch.cuda.synchronize()


def fixed_call_ms(wl, stream, world, reps=FIXED_REPS):
    """Whole-call device time per step over a fixed number of calls (one
    graph, replayed once untimed), max over ranks."""
    warm(wl, stream)
    graphs = capture(wl, stream, reps)
    replay_ms(graphs, stream)
    barrier(world)
    ms = replay_ms(graphs, stream) / reps
    graphs.clear()
    return max_over_ranks(ms, wl.device, world)


def single_record(name, device, seed, stream, world, peak):
    """Whole call and streaming kernel alone for one single-matrix workload
    (one replica per rank)."""
    wl = Workload(name, device, seed)
    nbytes = algorithmic_bytes(name, wl.spec)
    call_ms = fixed_call_ms(wl, stream, world)
    kern_ms = max_over_ranks(kernel_only_ms(wl, stream, FIXED_REPS), device, world)
    rec = {"workload": wl.spec["desc"], "bytes_per_call": nbytes, "calls": FIXED_REPS,
           "us_per_call": round(call_ms * 1e3, 3), "gbs": round(world * nbytes / (call_ms * 1e-3) / 1e9, 2),
           "call_frac": round(nbytes / (call_ms * 1e-3) / 1e9 / peak, 4),
           "kernel_us": round(kern_ms * 1e3, 3), "kernel_frac": round(nbytes / (kern_ms * 1e-3) / 1e9 / peak, 4),
           "weight_copies": wl.copies, "replicas": world}
    del wl
    return rec


# ---- the sharded MLP / head record ---------------------------------------

def _dequant_torch(m):
    """fp32 [rows, cols] dequantisation of a device PackedMatrix with torch
    (for the consistency bound of the sharded check; the kernels never use
    it)."""
    import torch
    w = m.weight.view(torch.int32)
    per = 32 // m.bits
    shifts = torch.arange(per, device=w.device, dtype=torch.int32) * m.bits
    q = ((w.unsqueeze(-1) >> shifts) & ((1 << m.bits) - 1)).reshape(m.rows, m.cols).float()
    if m.meta_bf16:
        s = (m.scales.view(torch.int16).to(torch.int32) << 16).view(torch.float32)
        b = (m.biases.view(torch.int16).to(torch.int32) << 16).view(torch.float32)
    else:
        s, b = m.scales, m.biases
    s = s.reshape(m.rows, m.cols // m.group).repeat_interleave(m.group, dim=1)
    b = b.reshape(m.rows, m.cols // m.group).repeat_interleave(m.group, dim=1)
    return q * s + b


def _full_matrix(wl, rows_total, cols, seed_off):
    """Rank 0: the full matrix assembled from every rank's shard (each
    shard's seeded synthetic data regenerated here)."""
    from qmr import parallel, synth
    parts = []
    for r in range(wl.world):
        r0, r1 = parallel.shard_range(rows_total, wl.world, r)
        parts.append(synth.affine_matrix(r1 - r0, cols, 4, GROUP, seed=wl.shard_seed(r) + seed_off))
    cat = {k: np.concatenate([p[k] for p in parts], axis=0) for k in ("weight", "scales", "biases")}
    return synth.to_device(cat, rows_total, cols, 4, GROUP, wl.device)


def sharded_check(wl, stream):
    """Rank 0 compares the sharded outputs with the 1-GPU call on the full
    matrices: every output within twice the north-star bound (both sides
    are within 2e-5 * sum|w x| of FP64), argmax identical unless the top two
    logits are within that bound.  Returns a dict for the JSON line."""
    import torch
    import torch.distributed as dist

    import qmr
    b, dev = wl.batch, wl.device
    with torch.cuda.stream(stream):
        wl.step(0, stream)
    stream.synchronize()
    if wl.name == "head":
        lg = torch.empty(wl.world * wl.y.numel(), dtype=torch.float32, device=dev)
        dist.all_gather_into_tensor(lg, wl.y)
        got_logits = lg.view(wl.world, b, -1).permute(1, 0, 2).reshape(b, VOCAB)
        got_idx = wl.idx.clone()
    torch.cuda.synchronize()
    if wl.rank != 0:
        return None
    x = wl.x.view(b, COLS)
    if wl.name == "mlp":
        g = _full_matrix(wl, ROWS, COLS, 10)
        u = _full_matrix(wl, ROWS, COLS, 11)
        d = _full_matrix(wl, COLS, ROWS, 12)
        act = torch.empty(b * ROWS, dtype=torch.float32, device=dev)
        y = torch.empty(b * COLS, dtype=torch.float32, device=dev)
        qmr.gateup_swiglu(g, u, wl.x, act, b)
        qmr.matmul_affine(d, act, y, b)
        mod = wl.mods[0]
        act_s = mod.xa.output(mod.xa.parity ^ 1, dev)[:b * ROWS].view(b, ROWS)
        y_s = wl.y.view(b, COLS)
        torch.cuda.synchronize()
        G, U, D = _dequant_torch(g), _dequant_torch(u), _dequant_torch(d)
        ax = x.abs()
        gv, uv = x @ G.T, x @ U.T
        sg, su = ax @ G.abs().T, ax @ U.abs().T
        a1 = act.view(b, ROWS)
        mag_a = uv.abs() * 1.1 * sg + (gv * torch.sigmoid(gv)).abs() * su + 0.05 * a1.abs()
        ra = ((act_s - a1).abs() / (2 * 2e-5 * mag_a)).max().item()
        # y_s came from act_s: its distance to y allows the down bound twice plus |D| |act_s - act|.
        mag_y = a1.abs() @ D.abs().T
        slack = (act_s - a1).abs() @ D.abs().T
        ry = ((y_s - y.view(b, COLS)).abs() / (2 * 2e-5 * mag_y + slack)).max().item()
        worst = max(ra, ry)
        return {"vs_1gpu": "ok" if worst <= 1.0 else "FAILED", "worst_ratio": round(worst, 4),
                "bound": "2 x 2e-5 sum|w x| per output (act and y)"}
    h = _full_matrix(wl, VOCAB, COLS, 10)
    logits = torch.empty(b * VOCAB, dtype=torch.float32, device=dev)
    idx = torch.empty(b, dtype=torch.int32, device=dev)
    qmr.head_argmax(h, wl.x, logits, idx, b)
    torch.cuda.synchronize()
    H = _dequant_torch(h)
    mag = x.abs() @ H.abs().T
    L = logits.view(b, VOCAB)
    worst = ((got_logits - L).abs() / (2 * 2e-5 * mag)).max().item()
    ids_ok = True
    for bi in range(b):
        gi, wi = int(got_idx[bi]), int(idx[bi])
        if gi != wi:
            # acceptable only for a near tie within the bound
            ids_ok &= bool(abs(float(L[bi, gi]) - float(L[bi, wi])) <= 4 * 2e-5 * float(mag[bi, wi]))
    ok = worst <= 1.0 and ids_ok
    return {"vs_1gpu": "ok" if ok else "FAILED", "worst_ratio": round(worst, 4),
            "argmax": got_idx.tolist(), "argmax_1gpu": idx.tolist(), "argmax_identical": got_idx.tolist() == idx.tolist(),
            "bound": "2 x 2e-5 sum|w x| per logit"}


def sharded_record(name, device, seed, stream, world, rank, peak):
    """The MLP or head: unsharded at N=1, row-sharded over the ranks with the
    peer-memory exchange at N>1 (strong scaling: one model's bytes per step)."""
    wl = Workload(name, device, seed, world=world, rank=rank, shard=True, exchange="p2p")
    nbytes = algorithmic_bytes(name, wl.spec)
    ms = fixed_call_ms(wl, stream, world)
    rec = {"workload": wl.spec["desc"], "bytes_per_step": nbytes, "steps": FIXED_REPS,
           "us_per_step": round(ms * 1e3, 3), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 2),
           "gbs_per_gpu": round(nbytes / world / (ms * 1e-3) / 1e9, 2),
           "frac_per_gpu": round(nbytes / world / (ms * 1e-3) / 1e9 / peak, 4),
           "exchange": "peer-memory stores in the streaming kernel + bounded wait kernel" if wl.sharded else None,
           "split": ("gate/up and down by output rows, activations and outputs exchanged" if name == "mlp" else
                     "vocabulary rows, per-shard argmax keys exchanged and merged") if wl.sharded else "unsharded",
           "gpus_active": world, "launches_per_step": wl.launches_per_step, "weight_copies": wl.copies}
    if wl.sharded:
        chk = sharded_check(wl, stream)
        if chk is not None:
            rec["check"] = chk
    barrier(world)
    import torch
    torch.cuda.synchronize()
    wl.close()
    del wl
    return rec


# ---- config 4: the synthetic 64-layer hybrid decode -------------------------

DECODE_CONTEXT = 4096


def decode_bytes_per_token(cfg):
    """Algorithmic bytes of one decode step: every packed matrix once (Q4
    words + BF16 scale and bias per 64 columns), the embedding row, the
    DeltaNet state read and written, the conv history."""
    H, F, V = cfg["hidden"], cfg["inter"], cfg["vocab"]
    KD, VD = cfg["lin_key_heads"] * cfg["lin_key_dim"], cfg["lin_value_heads"] * cfg["lin_value_dim"]
    QD, KVD = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    mat = lambda r, c: r * c // 2 + r * c // 64 * 4  # noqa: E731
    total = mat(V, H) + H * 4 // 8  # head, embedding row
    for att in cfg["is_attn"]:
        total += 3 * mat(F, H)
        if att:
            total += mat(2 * QD + 2 * KVD, H) + mat(H, QD)
        else:
            total += mat(2 * KD + 2 * VD + 2 * cfg["lin_value_heads"], H) + mat(H, VD)
            total += 2 * cfg["lin_value_heads"] * cfg["lin_value_dim"] * cfg["lin_key_dim"] * 4
    return total


def decode_record(device, world, rank, peak, cpu_baseline, n_prompt=512, n_new=128):
    """Config 4: prefill a seeded 512-token prompt, then greedily decode 128
    tokens at context 4096.  One GPU: the whole model.  N GPUs: the model
    split tensor-parallel over the N ranks (qmr_model_synthetic_sharded:
    heads, MLP rows and vocabulary divided, partial sums all-reduced by the
    streaming kernels' peer-memory exchange), one token stream for the job,
    so tokens/s is strong-scaling."""
    DECODE_PROMPT, DECODE_NEW = n_prompt, n_new
    import torch

    import qmr
    from qmr import engine as qeng
    from qmr import synth
    torch.cuda.empty_cache()
    cfg = qeng.qwen27b_config()
    if world > 1:
        eng = qmr.Engine.synthetic_sharded(cfg, 4242, DECODE_CONTEXT)
    else:
        eng = qmr.Engine.synthetic(cfg, 4242, DECODE_CONTEXT)
    prompt = [int(v % cfg["vocab"]) for v in synth.splitmix64(77, DECODE_PROMPT)]
    eng.generate(prompt[:16], 8)  # untimed warm-up
    eng.reset()
    barrier(world)
    toks, pre_ms, dec_ms = eng.generate(prompt, DECODE_NEW)
    pre_max = max_over_ranks(pre_ms, device, world)
    dec_max = max_over_ranks(dec_ms, device, world)
    with_head, without = eng.step_launches()
    # B3 verification rounds (MTP-style decoding): the synthetic model has no
    # trained drafter, so the drafts are (i) the greedy continuation just
    # decoded (every draft accepted: 3 tokens per round) and (ii) wrong
    # tokens (every draft rejected: 1 token per round).  Both must emit the
    # plain greedy tokens.
    table = [0] * DECODE_CONTEXT
    for k, t in enumerate(toks):
        table[DECODE_PROMPT + k] = t
    mtp = {}
    for label, drafts in (("drafts_accepted", table), ("drafts_rejected", [(t + 1) % cfg["vocab"] for t in table])):
        eng.reset()
        barrier(world)
        m_toks, rounds, acc, _, m_dec = eng.mtp_generate(prompt, DECODE_NEW, 3, drafts)
        m_max = max_over_ranks(m_dec, device, world)
        mtp[label] = {"rounds": rounds, "drafts_accepted": acc, "rounds_per_s": round(rounds / (m_max * 1e-3), 2),
                      "tok_s": round((DECODE_NEW - 1) / (m_max * 1e-3), 2),
                      "ms_per_round": round(m_max / rounds, 4), "same_tokens_as_plain": m_toks == toks}
    same_tokens = True
    if world > 1:
        import torch.distributed as dist
        every = [None] * world
        dist.all_gather_object(every, toks)
        same_tokens = all(t == every[0] for t in every)
    eng.close()
    nbytes = decode_bytes_per_token(cfg)
    tps = (DECODE_NEW - 1) / (dec_max * 1e-3)
    rec = {"workload": "synthetic 64-layer Qwen3.5-27B-shaped hybrid (3:1 DeltaNet:attention), Q4/g64 BF16 "
                       "metadata, distinct seeded weights, vocabulary 152064, FP32 activations/state/KV",
           "prompt_tokens": DECODE_PROMPT, "new_tokens": DECODE_NEW, "context": DECODE_CONTEXT,
           "decode_tok_s": round(tps, 2), "ms_per_token": round(dec_max / (DECODE_NEW - 1), 4),
           "prefill_tok_s": round(DECODE_PROMPT / (pre_max * 1e-3), 2),
           "bytes_per_token": nbytes, "gbs_per_gpu": round(nbytes / world * tps / 1e9, 2),
           "frac_per_gpu": round(nbytes / world * tps / 1e9 / peak, 4),
           "launches_per_token": with_head, "launches_per_prefill_token": without,
           "parallelism": f"tp{world}" if world > 1 else "single", "scaling": "strong",
           "tokens_identical_across_ranks": same_tokens,
           "first_tokens": toks[:8],
           "mtp_b3": dict(mtp, block=3, note="tok/s counts the 127 tokens after the first (the prompt's last step "
                                             "emits it); timed over the verification rounds")}
    if cpu_baseline and rank == 0 and world == 1:
        # The reference's CPU arithmetic for this graph: the FP64 oracle on the
        # same synthetic model, all host cores, two steps of the prompt.
        import oracle
        oracle.set_threads(host_threads())
        o = oracle.synthetic_decode_oracle(cfg, 4242, 8, qeng.synthetic_mid, qeng.MID_EMBED, qeng.MID_HEAD)
        t0 = time.perf_counter()
        for t in prompt[:2]:
            o.forward(t)
        secs = (time.perf_counter() - t0) / 2
        rec["cpu_baseline"] = {"value": round(1.0 / secs, 5), "unit": "tok/s", "cores": oracle.threads(),
                               "kind": "port", "s_per_token": round(secs, 3),
                               "sample": "2 decode steps (positions 0-1) of the same model, FP64 oracle "
                                         "(oracle/decode.c), OpenMP over matrix rows"}
    return rec


def run_decode(args):
    """--workload decode: the config-4 record alone (profiling runs)."""
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
    peak, _ = load_peaks()
    rec = decode_record(device, world, rank, peak, not (args.no_cpu_baseline or args.quick), args.decode_prompt,
                        args.decode_new)
    if rank == 0:
        print(json.dumps({"metric": "synthetic decode tokens/s", "value": rec["decode_tok_s"], "unit": "tok/s",
                          "n_gpus": world, "higher_is_better": True, "scaling": "strong", "decode": rec}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_gpu(args):
    import torch
    import torch.distributed as dist

    import qmr
    if args.workload == "decode":
        return run_decode(args)
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    qmr.ops.init(local)
    spec = workload_spec(args.workload)
    peak, peak_kind = load_peaks()
    shard = args.workload in ("mlp", "head")
    wl = Workload(args.workload, device, seed=1000 + 17 * rank, world=world, rank=rank, shard=shard,
                  exchange=args.exchange)
    nbytes = algorithmic_bytes(args.workload, spec)
    # Replicas: every rank processes nbytes per step.  Shards: the ranks
    # together process one model's nbytes per step.
    job_factor = 1 if wl.sharded else world

    stream = torch.cuda.Stream(device)
    torch.cuda.synchronize()
    warm(wl, stream, max(args.warmup, 3))
    graphs = capture(wl, stream, args.steps)
    replay_ms(graphs[:1], stream)  # untimed warm replay
    torch.cuda.synchronize()

    clocks = Clocks(local)
    barrier(world)
    torch.cuda.synchronize()
    clocks.start()
    time.sleep(0.3)
    ms_max = max_over_ranks(replay_ms(graphs, stream), device, world)
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
    graphs.clear()
    single = args.workload in ("b3", "b1", "q8b3")
    kernel_ms = kernel_only_ms(wl, stream, args.steps) if single else None
    reps_ms = fixed_call_ms(wl, stream, world) if not args.quick else None
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
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(e2e_steps):
            wl.step(i, stream, x=xh)
            qmr.ops.copy_f32(out, yh, out.numel(), stream=stream)
        e1.record(stream)
    stream.synchronize()
    te = max_over_ranks(e0.elapsed_time(e1), device, world)
    e2e_value = job_factor * nbytes * e2e_steps / (te * 1e-3) / 1e9

    if kernel_ms is not None:
        achieved = nbytes / (kernel_ms * 1e-3) / 1e9  # the streaming kernel reads weights, x' and writes y
        timing_note = "streaming kernel alone: activations prepared once, K launches in one graph"
    else:
        # per GPU: its share of the job's bytes over the step time
        achieved = job_factor * nbytes / world / (ms_per_step * 1e-3) / 1e9
        timing_note = "whole call" + (f", sharded step incl. the {wl.exchange} exchange" if wl.sharded else "")
    traffic = profile_traffic(args.workload)
    config = config_of(spec)
    config.update({"weight_copies": wl.copies, "l2_bytes": wl.l2,
                   "l2_policy": f"{wl.copies} distinct weight copies rotated (> 4x L2)",
                   "bytes_per_step": nbytes,
                   "parallelism": (f"rowshard{world} ({'peer-memory exchange in the kernels' if wl.exchange == 'p2p' else 'NCCL all-gather'})"
                                   if wl.sharded else f"replicas{world}" if world > 1 else "single")})
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 6), "higher_is_better": True,
        "scaling": "strong" if wl.sharded else "weak",
        "vs_baseline": None, "dtype": "f32", "arith": ARITH,
        "data": "synthetic (seeded; benchmark distributions)",
        "config": config,
        "call_frac": round(job_factor * nbytes / world / (ms_per_step * 1e-3) / 1e9 / peak, 4),
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} hbm_gbs", "timing": timing_note,
                     "kernel_ms": None if kernel_ms is None else round(kernel_ms, 6)},
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clk,
    }
    if reps_ms is not None:
        line["reps200"] = {"calls": FIXED_REPS, "us_per_call": round(reps_ms * 1e3, 3),
                           "value": round(job_factor * nbytes / (reps_ms * 1e-3) / 1e9, 2)}
    wl.close()
    del wl

    if args.workload == "b3" and not args.quick:
        line["workloads"] = {n: single_record(n, device, 2000 + 17 * rank, stream, world, peak)
                             for n in ("b1", "q8b3")}
        line["sharded"] = {n: sharded_record(n, device, 3000, stream, world, rank, peak) for n in ("mlp", "head")}
        line["decode"] = decode_record(device, world, rank, peak, not args.no_cpu_baseline)
        line["gpu_launches_decode_per_token"] = line["decode"]["launches_per_token"]

    if rank == 0 and world == 1 and not (args.no_cpu_baseline or args.quick):
        import oracle
        oracle.set_threads(host_threads())
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
        import gc
        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="qmr", choices=["qmr", "reference"])
    ap.add_argument("--workload", default="b3", choices=["b3", "b1", "q8b3", "mlp", "head", "decode"])
    ap.add_argument("--decode-prompt", type=int, default=512, help="config-4 prompt tokens")
    ap.add_argument("--decode-new", type=int, default=128, help="config-4 generated tokens")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="sharded workloads: output exchange over peer memory in the kernels, or NCCL all-gathers")
    ap.add_argument("--quick", action="store_true",
                    help="profiling runs: no clock-sampling loop, no sub-records, short e2e, no CPU baseline")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        if args.workload == "decode":
            args.workload = "b3"
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
