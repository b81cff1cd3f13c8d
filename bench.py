#!/usr/bin/env python3
"""Benchmark: one emitted IR kernel per step, on 1..N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c2] [--impl ours|reference]

A *step* is one pass of the hot path over one batch of synthetic input: the compiled kernel
(plus, for the full-array sum at N > 1, the ncclAllReduce of the per-GPU partial).  The default
workload is BASELINE config 2 — the f32 sum of 2**28 elements — whose metric is HBM GB/s.

Printed (rank 0, one JSON line):
  value        whole-job algorithmic bytes (or FLOP) per second, inputs resident in HBM;
  e2e          the same metric through the C-ABI path with pinned HOST buffers: every step copies
               its inputs host->device, runs, and copies its outputs back;
  roofline     the kernel's achieved GB/s (TFLOP/s) from CUDA events around each launch, against
               the measured peak in MEASURED_PEAKS.json, and its DRAM traffic from ncu;
  cpu_baseline the CPU oracle (a numpy restatement of the reference semantics) on host cores;
  clocks       nvidia-smi samples taken during the timed region.

``--impl reference`` times the reference's CPU implementation of the path — the oracle port —
on all host cores (spawned worker processes), on the same workload, and prints the same line
with ``"impl": "reference"``.  Multi-GPU runs use torchrun: one process per GPU; the units are
sharded (weak scaling: each rank owns a full-size shard), time is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "c1": ("softmax f32 [4096,1024]", "HBM GB/s", "GB/s"),
    "c2": ("sum f32 [2^28]", "HBM GB/s", "GB/s"),
    "c2i": ("sum i32 [2^28]", "HBM GB/s", "GB/s"),
    "c3": ("fused relu(a*b+c)*exp(d) bf16 [8192,8192]", "HBM GB/s", "GB/s"),
    "c4": ("bmm bf16 [16,4096,4096]x[16,4096,4096] -> f32", "tensor TFLOP/s", "TFLOP/s"),
    "c5": ("causal attention bf16 [8,32,4096,128]", "tensor TFLOP/s", "TFLOP/s"),
}

def _small_for_profile():
    from emmy_ptx_b200 import irgen
    return {
        "c1": lambda **kw: irgen.softmax_ir(4096, 1024, **kw),
        "c2": lambda **kw: irgen.sum_ir(1 << 26, "f32", **kw),
        "c2i": lambda **kw: irgen.sum_ir(1 << 26, "i32", **kw),
        "c3": lambda **kw: irgen.fused_ir(4096, 8192, **kw),
        "c4": lambda **kw: irgen.bmm_ir(2, 4096, 4096, 4096, **kw),
        "c5": lambda **kw: irgen.attention_ir(2, 16, 4096, 128, **kw),
    }


class _Lazy(dict):
    def __missing__(self, k):
        self.update(_small_for_profile())
        return dict.__getitem__(self, k)


SMALL_FOR_PROFILE = _Lazy()

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) from one ncu capture of each
# kernel on a reduced instance, scaled to the full launch by the units processed (traffic grows in
# proportion for these streaming / tiled kernels); the captures are summarised under profiles/.
TRAFFIC = {
    "c2": (268.443904e6 + 4.902912e6) * 4,       # 2^26 -> 2^28 elements
    "c2i": (268.443904e6 + 4.902912e6) * 4,      # same kernel shape, i32 elements
    "c3": (201.394176e6 + 44.741632e6) * 2,      # 4096 -> 8192 rows
    "c4": (192.727040e6 + 105.907456e6) * 8,     # 2 -> 16 batches
    "c1": 16.793088e6 + 0.0,                     # captured at full size (y stays in L2 at kernel end)
    "c5": (143.738112e6 + 14.620416e6) * 8,      # 32 -> 256 (batch, head) pairs
}


def work_units(p) -> tuple[float, str]:
    """Algorithmic bytes (HBM-bound kernels) or FLOP (tensor kernels) of one launch."""
    fam = p.family
    q = p.params
    if fam == "softmax":
        return 2.0 * q["rows"] * q["cols"] * 4, "B"
    if fam == "sum":
        return q["n"] * 4.0 + 4.0, "B"
    if fam == "fused":
        ob = 2 if q.get("out_dtype", "bf16") in ("bf16", "f16") else 4
        return 3.0 * q["rows"] * q["cols"] * 2 + q["cols"] * 4 + q["rows"] * q["cols"] * ob, "B"
    if fam == "bmm":
        return 2.0 * q["batch"] * q["m"] * q["n"] * q["k"], "FLOP"
    if fam == "attention":
        s = q["seq"]
        pairs = s * (s + 1) / 2 if q.get("causal", True) else s * s
        return 4.0 * q["batch"] * q["heads"] * q["dim"] * pairs, "FLOP"
    raise ValueError(fam)


def load_peaks() -> tuple[dict, str]:
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        return json.loads(f.read_text()), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "sm_max_mhz": 1965.0}, "fallback"


# ---- clocks -------------------------------------------------------------------------------------

CLOCK_FIELDS = ["index", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
                "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
                "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]


class ClockSampler:
    """nvidia-smi sampling every 200 ms while the timed region runs."""

    def __init__(self):
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + ",".join(CLOCK_FIELDS),
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) != len(CLOCK_FIELDS):
                continue
            rows.append(dict(zip(CLOCK_FIELDS, parts)))
        os.unlink(self.file.name)
        if not rows:
            return None

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        by_gpu = {}
        for r in rows:
            by_gpu.setdefault(r["index"], []).append(r)
        # the GPU(s) under load: highest median power
        med_power = {g: statistics.median([num(r["power.draw"]) or 0 for r in rs]) for g, rs in by_gpu.items()}
        top = max(med_power.values())
        busy = [g for g, pw in med_power.items() if pw >= 0.6 * top]
        samples = [r for g in busy for r in by_gpu[g]]
        loaded = [r for r in samples if (num(r["power.draw"]) or 0) >= 0.5 * top] or samples
        reasons = set()
        for r in loaded:
            for k in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"):
                if r["clocks_event_reasons." + k].lower().startswith("active"):
                    reasons.add(k)
        sm = [num(r["clocks.sm"]) for r in loaded if num(r["clocks.sm"])]
        mx = [num(r["clocks.max.sm"]) for r in loaded if num(r["clocks.max.sm"])]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(loaded), "gpus": sorted(busy)}


# ---- the CPU oracle (baseline and reference arm) --------------------------------------------------

def _oracle_worker(args):
    """Interpret a block range of the problem's kernel; returns the output arrays (spawned process)."""
    key, ir_kw, files, block_lo, block_hi = args
    import numpy as np
    from emmy_ptx_b200 import irgen
    from emmy_ptx_b200.ir import Graph
    from oracle.interp import Interpreter, storage_dtype
    p = irgen.FULL[key](**ir_kw)
    bufs = {}
    for a in p.args:
        n = 1
        for s in a.shape:
            n *= s
        if a.output:
            bufs[a.name] = np.zeros(n, dtype=storage_dtype(a.dtype))
        else:
            bufs[a.name] = np.memmap(files[a.name], dtype=storage_dtype(a.dtype), mode="r", shape=(n,))
    Interpreter(Graph.from_dict(p.graph)).run(bufs, p.grid, p.block, blocks=range(block_lo, block_hi))
    return {a.name: bufs[a.name].copy() for a in p.outputs}


class OraclePool:
    """The oracle over a bounded sample of the workload, on ``workers`` spawned processes."""

    def __init__(self, key: str, tensors: dict, workers: int, sample_blocks: int, ir_kw: dict | None = None):
        import multiprocessing as mp
        from emmy_ptx_b200 import irgen
        from emmy_ptx_b200.data import to_numpy_storage
        self.key = key
        self.ir_kw = dict(ir_kw or {})
        self.p = irgen.FULL[key](**self.ir_kw)
        # inputs shared with the workers as read-only memory-mapped files (page cache, not /dev/shm)
        self.dir = tempfile.TemporaryDirectory(prefix="emmy_oracle_")
        self.files = {}
        for a in self.p.inputs:
            f = os.path.join(self.dir.name, a.name + ".bin")
            to_numpy_storage(tensors[a.name]).tofile(f)
            self.files[a.name] = f
        self.workers = workers
        self.sample_blocks = min(sample_blocks, self.p.grid)
        self.pool = mp.get_context("spawn").Pool(workers) if workers > 1 else None

    def chunks(self):
        n = self.sample_blocks
        w = max(1, min(self.workers, n))
        edges = [n * i // w for i in range(w + 1)]
        return [(self.key, self.ir_kw, self.files, edges[i], edges[i + 1]) for i in range(w)]

    def step(self):
        if self.pool is None:
            return [_oracle_worker(c) for c in self.chunks()]
        return self.pool.map(_oracle_worker, self.chunks())

    def close(self):
        if self.pool is not None:
            self.pool.close()
            self.pool.join()
        self.dir.cleanup()


def sample_blocks_for(key: str, p, workers: int = 1) -> int:
    """Thread blocks of the grid the oracle interprets per pass (its bounded sample).

    The interpreter's cost is per statement executed, nearly independent of how many lanes run
    it, so the sample is set per kernel: the whole grid for the streaming kernels (a few seconds),
    a handful of blocks for the contraction kernels (about 10 s for one process)."""
    per = {"c1": p.grid, "c2": p.grid, "c2i": p.grid, "c3": p.grid // 2, "c4": 8, "c5": 8}.get(key, 8)
    if key in ("c4", "c5"):
        per = per * max(1, workers // 4) if workers > 1 else per
    return max(1, min(p.grid, per))


# ---- main -----------------------------------------------------------------------------------------

def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every step from the host instead of CUDA graphs")
    ap.add_argument("--size", default="full", choices=["full", "small"],
                    help="small: a reduced instance of the same kernel (still larger than L2) for ncu captures")
    ap.add_argument("--opt", action="append", default=[], metavar="KEY=VALUE",
                    help="a compile option (value read as JSON when it parses), e.g. --opt attn_persistent=true")
    ap.add_argument("--ir", action="append", default=[], metavar="KEY=VALUE",
                    help="an argument of the workload's IR builder, e.g. --ir recip=true for config 1")
    return ap.parse_args()


def compile_options(pairs) -> dict:
    """``--opt KEY=VALUE`` flags as the compiler's options dict."""
    out = {}
    for item in pairs:
        key, sep, val = item.partition("=")
        if not sep or not key:
            raise SystemExit(f"--opt wants KEY=VALUE, got {item!r}")
        try:
            out[key] = json.loads(val)
        except ValueError:
            out[key] = val
    return out


def use_graphs(world: int, no_graph: bool) -> bool:
    """Whether this run captures CUDA graphs at all: single-GPU runs only.  Multi-GPU runs launch from
    the host, the multi-GPU path measured on B200, so no capture runs beside the process group's NCCL
    watchdog and no NCCL call is ever captured."""
    return not no_graph and world == 1


def capture_steps(collective: bool, no_graph: bool, world: int = 1) -> bool:
    """Whether the timed steps are replayed from a CUDA graph: yes, unless graphs are off, the run has
    several ranks, or a step holds the ncclAllReduce.  NCCL calls stay out of graphs: a live graph
    that holds one keeps the communicator's teardown waiting."""
    return use_graphs(world, no_graph) and not collective


def reference_arm(args, world, rank):
    """The reference's CPU implementation of the path (the oracle port) on every host core."""
    if rank != 0:
        return 0
    import torch
    from emmy_ptx_b200 import irgen, data
    key = args.config
    p = irgen.FULL[key]()
    units, kind = work_units(p)
    _, metric, unit = CONFIGS[key]
    cores = os.cpu_count() or 1
    workers = max(1, min(cores, 64))
    tensors = data.make_inputs(p, "cpu")
    blocks = sample_blocks_for(key, p, workers)
    pool = OraclePool(key, tensors, workers, blocks)
    frac = pool.sample_blocks / p.grid
    try:
        for _ in range(max(args.warmup, 0)):
            pool.step()
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            pool.step()
            times.append(time.perf_counter() - t0)
    finally:
        pool.close()
    ms = 1000.0 * sum(times) / len(times)
    scale = 1e9 if unit == "GB/s" else 1e12
    value = units * frac / (ms / 1000.0) / scale
    sample = (f"{pool.sample_blocks} of {p.grid} thread blocks ({100 * frac:.1f}% of the workload) per step, "
              f"{workers} spawned worker processes")
    line = {
        "impl": "reference", "metric": f"{CONFIGS[key][0]} {metric}", "value": value, "unit": unit,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": p.args[0].dtype,
        "data": "synthetic (seeded, CPU-generated)",
        "config": {"workload": key, "description": CONFIGS[key][0]},
        "cpu_baseline": {"value": value, "unit": unit, "cores": workers, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def main() -> int:
    args = parse()
    from emmy_ptx_b200 import dist as edist
    world, rank, local = edist.env()
    if args.impl == "reference":
        return reference_arm(args, world, rank)
    import torch
    from emmy_ptx_b200 import irgen, data
    from emmy_ptx_b200.compiler import compile_graph
    from emmy_ptx_b200.ir import Graph
    from emmy_ptx_b200.runtime import Executable
    dist = edist.init(world, local)
    max_over_ranks = edist.max_over_ranks
    key = args.config
    ir_kw = compile_options(args.ir)
    p = (SMALL_FOR_PROFILE[key] if args.size == "small" else irgen.FULL[key])(**ir_kw)
    units, kind = work_units(p)
    desc, metric, unit = CONFIGS[key]
    scale = 1e9 if unit == "GB/s" else 1e12
    peaks, peak_src = load_peaks()

    options = compile_options(args.opt)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), options)
    ex = Executable(mod, device=local)
    dev = ex.dev
    stream = torch.cuda.current_stream().cuda_stream

    # inputs: seeded per rank (rank r owns shard r of the weak-scaled global problem)
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    rotate = 1
    if units < 2 * 126e6 and kind == "B":      # L2-resident working set: rotate buffer sets past 2x L2
        rotate = int(max(2, (2 * 126e6 * 2) // units + 1))
    sets = []
    for r in range(rotate):
        t = {}
        for a in p.args:
            shape = tuple(a.shape)
            if a.output:
                t[a.name] = torch.zeros(shape, dtype=data.torch_dtype(a.dtype), device="cuda")
            elif a.dist[0] == "normal":
                t[a.name] = (torch.randn(shape, generator=gen, device="cuda") * a.dist[1]).to(data.torch_dtype(a.dtype))
            elif a.dist[0] == "uniform":
                t[a.name] = (torch.rand(shape, generator=gen, device="cuda") * (a.dist[2] - a.dist[1]) + a.dist[1]).to(
                    data.torch_dtype(a.dtype))
            else:
                t[a.name] = torch.randint(a.dist[1], a.dist[2], shape, generator=gen, device="cuda",
                                          dtype=torch.int32)
        sets.append(t)

    collective = p.family == "sum" and world > 1
    allreduce = edist.AllReducePartials(dev, dist, rank, world) if collective else None

    def step(t, s=None):
        s = stream if s is None else s
        ex(t, s)
        if collective:
            allreduce(t["out"], p.params["dtype"], s)

    for i in range(max(args.warmup, 3)):
        step(sets[i % rotate])
    torch.cuda.synchronize()
    if dist:
        dist.barrier()

    launches0 = dev.launches
    reps = args.steps if units * 1.0 > 1e11 or kind == "FLOP" else max(args.steps, 200)
    # single-GPU runs replay launch-bound steps from CUDA graphs: exactly K steps in one graph, and a
    # kernel-only graph of `reps` back-to-back launches for the per-launch duration.  Multi-GPU runs,
    # and any step holding the ncclAllReduce, launch from the host (see use_graphs / capture_steps).
    step_graph = None
    kern_graph = None
    if use_graphs(world, args.no_graph):
        if capture_steps(collective, args.no_graph, world):
            step_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(step_graph):
                cs = torch.cuda.current_stream().cuda_stream
                for i in range(args.steps):
                    step(sets[i % rotate], cs)
            step_graph.replay()
        kern_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(kern_graph):
            cs = torch.cuda.current_stream().cuda_stream
            for i in range(reps):
                ex.run(sets[i % rotate], cs, zero=False)   # every entry of the module (a pre-pass included)
        kern_graph.replay()
        torch.cuda.synchronize()
    gpu_launches = args.steps * len(mod.kernels)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clocks = ClockSampler() if local == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0.record()
    if step_graph is not None:
        step_graph.replay()
    else:
        for i in range(args.steps):
            step(sets[i % rotate])
    e1.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    # the kernel alone, back to back on the same stream (CUDA events around the whole sequence)
    k0 = torch.cuda.Event(enable_timing=True)
    k1 = torch.cuda.Event(enable_timing=True)
    k0.record()
    if kern_graph is not None:
        kern_graph.replay()
    else:
        for i in range(reps):
            ex.run(sets[i % rotate], stream, zero=False)
    k1.record()
    torch.cuda.synchronize()
    clock = clocks.stop() if clocks else None
    ms_step = max_over_ranks(dist, ms / args.steps)
    kern_ms = max_over_ranks(dist, k0.elapsed_time(k1) / reps)
    value = world * units / (ms_step / 1000.0) / scale

    # correctness of what was timed (rank-local shard)
    check = None
    t = sets[0]
    ex(t, stream)
    torch.cuda.synchronize()
    if p.family == "sum":
        want = t["x"].double().sum().item() if p.params["dtype"] == "f32" else int(t["x"].long().sum().item())
        got = t["out"].item()
        check = {"abs_err": abs(got - want), "rel_err": abs(got - want) / max(abs(want), 1e-30)}
        if collective:
            # the exchange step too: kernel + ncclAllReduce against the all-reduced float64 shard sums
            step(t)
            torch.cuda.synchronize()
            tot = torch.tensor([float(want)], dtype=torch.float64, device="cuda")
            dist.all_reduce(tot)
            g_all = t["out"].item()
            check["global_rel_err"] = abs(g_all - tot.item()) / max(abs(tot.item()), 1e-30)
    elif p.family == "softmax":
        want = torch.softmax(t["x"].double(), -1)
        check = {"max_rel_err": ((t["y"].double() - want).abs() / want.abs().clamp_min(1e-30)).max().item()}
    elif p.family == "fused":
        want = torch.relu(t["a"].double() * t["b"].double() + t["c"].double()) * torch.exp(t["d"].double())
        check = {"max_rel_err_vs_f64": ((t["y"].double() - want).abs() / want.abs().clamp_min(1e-6)).max().item()}
    elif p.family == "bmm":
        # batch 0 in float64: the error relative to max(|ref|, rms), the matmul tolerance's measure
        want = t["A"][0].double() @ t["B"][0].double()
        den = torch.clamp(want.abs(), min=want.pow(2).mean().sqrt().item())
        check = {"batch0_max_err_over_rms_floor": ((t["C"][0].double() - want).abs() / den).max().item()}
    elif p.family == "attention":
        # (batch 0, head 0) in float64: the error in bf16 units of max(|ref|, row rms)
        q, k, v = (t[n][0, 0].double() for n in ("Q", "K", "V"))
        s_ = (q @ k.T) * p.params["scale"]
        if p.params.get("causal", True):
            s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
        want = torch.softmax(s_, -1) @ v
        den = torch.maximum(want.abs(), want.pow(2).mean(-1, keepdim=True).sqrt()) * 2.0 ** -7
        check = {"head00_max_err_bf16_units": ((t["O"][0, 0].double() - want).abs() / den).max().item()}
    code = int(max_over_ranks(dist, float(ex.error_code())))
    if code:
        # a tensor-core kernel whose bounded wait gave up returned early: its timing means nothing
        if rank == 0:
            print(json.dumps({"error": f"kernel status word {code}: a pipeline wait timed out", "config": key}),
                  file=sys.stderr, flush=True)
        step_graph = kern_graph = None
        torch.cuda.synchronize()
        if collective:
            allreduce.close()
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return 3

    # e2e: pinned host buffers, copies inside the timed region, through the C ABI
    e2e = None
    if not args.no_e2e:
        host = {a.name: sets[0][a.name].cpu().pin_memory() for a in p.args}
        t = sets[0]
        h2d = sum(host[a.name].numel() * host[a.name].element_size() for a in p.inputs)
        d2h = sum(host[a.name].numel() * host[a.name].element_size() for a in p.outputs)
        e2e_steps = max(3, min(args.steps, 10))

        def e2e_step():
            for a in p.inputs:
                dev.htod(t[a.name].data_ptr(), host[a.name].data_ptr(), host[a.name].numel() * host[a.name].element_size(), stream)
            step(t)
            for a in p.outputs:
                dev.dtoh(host[a.name].data_ptr(), t[a.name].data_ptr(), host[a.name].numel() * host[a.name].element_size(), stream)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(e2e_steps):
            e2e_step()
        a1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(dist, a0.elapsed_time(a1) / e2e_steps)
        e2e = {"value": world * units / (e2e_ms / 1000.0) / scale, "unit": unit, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "steps": e2e_steps,
               "path": "pinned host -> cuMemcpyHtoDAsync -> kernel -> cuMemcpyDtoHAsync (libemmy_launch.so)"}

    # context for small byte-bound launches: a plain device copy moving the same number of bytes
    # (half read, half written), rotated and graph-replayed like the kernel, shows what this launch
    # size allows; the roofline fraction itself stays against the measured 1 GiB copy peak
    copy_ref = None
    if kind == "B" and use_graphs(world, args.no_graph):
        nb = int(units // 2) // 4
        pairs = [(torch.ones(nb, dtype=torch.float32, device="cuda"), torch.empty(nb, dtype=torch.float32, device="cuda"))
                 for _ in range(rotate)]
        # an elementwise kernel on the SMs (torch's copy_ of same-dtype tensors may go to a copy engine)
        for a_, b_ in pairs:
            torch.mul(a_, 1.0, out=b_)
        g_copy = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_copy):
            for i in range(reps):
                torch.mul(pairs[i % rotate][0], 1.0, out=pairs[i % rotate][1])
        g_copy.replay()
        torch.cuda.synchronize()
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record()
        g_copy.replay()
        c1.record()
        torch.cuda.synchronize()
        copy_ms = max_over_ranks(dist, c0.elapsed_time(c1) / reps)
        del g_copy, pairs
        torch.cuda.synchronize()
        copy_ref = {"achieved": units / (copy_ms / 1000.0) / scale, "ms_per_launch": copy_ms,
                    "how": "torch elementwise y = x * 1 over the same bytes (half read, half written), same rotation, graph replay"}

    achieved = units / (kern_ms / 1000.0) / scale
    if copy_ref:
        copy_ref["kernel_frac_of_copy"] = achieved / copy_ref["achieved"]
    if unit == "GB/s":
        peak = peaks["hbm_gbs"]
        bound = "hbm"
    else:
        peak = peaks.get("bf16_tflops_sustained" if kern_ms > 100 else "bf16_tflops", 1590.0)
        bound = "tensor"
    traffic = TRAFFIC.get(key)
    roof = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
            "traffic": traffic, "peak_source": f"{peak_src} (MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback",
            "kernel": mod.kernels[-1]["entry"], "kernel_ms": kern_ms, "kernel_launches_timed": reps,
            "kernel_entries_timed": [k["entry"] for k in mod.kernels],
            "algorithmic_per_launch": units, "algorithmic_unit": kind, "same_bytes_copy": copy_ref}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tc = {a.name: sets[0][a.name].cpu() for a in p.args}
        blocks = sample_blocks_for(key, p, 1)
        pool = OraclePool(key, tc, 1, blocks, ir_kw)
        t0 = time.perf_counter()
        pool.step()
        dt = time.perf_counter() - t0
        pool.close()
        frac = pool.sample_blocks / p.grid
        cpu = {"value": units * frac / dt / scale, "unit": unit, "cores": 1, "kind": "port",
               "sample": f"{pool.sample_blocks} of {p.grid} thread blocks ({100 * frac:.1f}% of one step) "
                         f"through the numpy oracle, one process", "seconds": dt}

    step_graph = kern_graph = None          # release the graphs before any teardown
    torch.cuda.synchronize()
    if rank == 0:
        line = {
            "metric": f"{desc} {metric}", "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": p.args[0].dtype, "data": "synthetic (seeded on device)",
            "config": {"workload": key, "description": desc, "per_rank_units": units, "unit_kind": kind,
                       "parallelism": f"dp{world} ({'sharded + ncclAllReduce of the partial' if collective else 'sharded, no collective'})",
                       "l2": ("inputs exceed L2 (126 MB)" if rotate == 1 else f"{rotate} rotating buffer sets exceed 2x L2"),
                       "grid": p.grid, "block": p.block, **({"compile_options": options} if options else {}),
                       **({"ir_options": ir_kw} if ir_kw else {})},
            "gpu_launches": gpu_launches,
            "timing": ("CUDA graph replay of the K steps" if capture_steps(collective, args.no_graph, world)
                       else "host launches (kernel + ncclAllReduce per step)" if collective else "host launches"),
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "clocks": clock,
            "check": check, "kernel_kind": mod.kernels[-1].get("kind"),
        }
        print(json.dumps(line), flush=True)
    if collective:
        allreduce.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
