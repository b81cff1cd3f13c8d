#!/usr/bin/env python3
"""Benchmark: every BASELINE configuration's emitted IR kernel, on 1..N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config all|c1|c2|c2i|c3|c4|c5]
                    [--impl ours|reference] [--scaling strong|weak]

A *step* is one pass of the hot path over one batch of synthetic input: the compiled kernel(s) of a
configuration (plus, for the full-array sum at N > 1, the exchange of the per-GPU partials: the
peer-exchange kernel over NVLink by default, or one ncclAllReduce with ``--exchange nccl``).
By default one run measures all six configurations one after another in one process and prints
ONE JSON line (rank 0): the headline fields are config 2's — the f32 sum of 2**28 elements, metric
HBM GB/s — and ``per_config`` holds every configuration's own record.

Per configuration:
  value        whole-job algorithmic bytes (or FLOP) per second over exactly K steps, inputs resident
               in HBM, max over ranks;
  e2e          the same metric through the C-ABI path with pinned HOST buffers: every step copies its
               inputs host->device, runs, and copies its outputs back;
  roofline     the kernel's achieved GB/s (TFLOP/s) from CUDA events around back-to-back launches,
               against the measured peak in MEASURED_PEAKS.json, and its DRAM traffic from ncu;
  ref_emitter  the reference emitter's own PTX for the same full-size IR (tests/golden/ref_ptx_full),
               launched with the same geometry, buffers and rotation, and the time ratio to ours;
  cpu_baseline the source expression in torch on all host cores (a bounded, stated sample);
  cpu_port     the CPU oracle (a numpy restatement of the reference semantics), one process;
  check        the timed output against float64, held to the path's tolerance: a configuration
               outside it makes the run exit 4 without printing a line;
  clocks       nvidia-smi samples taken while the configuration ran.

Multi-GPU runs use torchrun, one process per GPU.  ``--scaling strong`` (the default) partitions each
configuration's one global problem: rank r owns shard r of 4096 rows / 2**28 elements / 8192 rows /
16 batches / 8 batches of 32 heads, sliced from inputs generated once with the global seeds.
``--scaling weak`` gives every rank a full-size problem of its own.  Time is the max over ranks.

``--impl reference`` times the reference's CPU implementation of the path — the oracle port — on all
host cores (spawned worker processes), on the same configurations, and prints the same line with
``"impl": "reference"``.
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
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
ALL_KEYS = ["c1", "c2", "c2i", "c3", "c4", "c5"]
HEADLINE = "c2"

# Strong scaling: the global unit count of each configuration along its sharded axis, and the
# tensors cut along that axis (the others — c3's row vector, the sum's scalar — are replicated).
SHARD_UNITS = {"c1": 4096, "c2": 1 << 28, "c2i": 1 << 28, "c3": 8192, "c4": 16, "c5": 8}
SHARDED = {"c1": ("x", "y"), "c2": ("x",), "c2i": ("x",), "c3": ("a", "b", "d", "y"), "c4": ("A", "B", "C"),
           "c5": ("Q", "K", "V", "O")}


def build_problem(key: str, units: int | None = None, **kw):
    """Config ``key`` with ``units`` of its sharded axis (the full configuration when None)."""
    from emmy_ptx_b200 import irgen
    if units is None:
        return irgen.FULL[key](**kw)
    return {
        "c1": lambda: irgen.softmax_ir(units, 1024, **{"recip": True, **kw}),
        "c2": lambda: irgen.sum_ir(units, "f32", **kw),
        "c2i": lambda: irgen.sum_ir(units, "i32", **kw),
        "c3": lambda: irgen.fused_ir(units, 8192, **kw),
        "c4": lambda: irgen.bmm_ir(units, 4096, 4096, 4096, **kw),
        "c5": lambda: irgen.attention_ir(units, 32, 4096, 128, **kw),
    }[key]()


def _small_for_profile():
    from emmy_ptx_b200 import irgen
    return {
        "c1": lambda **kw: irgen.softmax_ir(4096, 1024, **{"recip": True, **kw}),
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

# DRAM bytes per launch of the full configuration (dram__bytes_read.sum + dram__bytes_write.sum)
# from one ncu capture of each kernel on a reduced instance, scaled to the full launch by the units
# processed (traffic grows in proportion for these streaming / tiled kernels); the captures are
# summarised under profiles/.  Config 5 is the value pre-pass plus the attention kernel.
TRAFFIC = {
    "c2": (268.443904e6 + 4.902912e6) * 4,       # 2^26 -> 2^28 elements
    "c2i": (268.443904e6 + 4.902912e6) * 4,      # same kernel shape, i32 elements
    "c3": (201.394176e6 + 44.741632e6) * 2,      # 4096 -> 8192 rows
    "c4": (195.336192e6 + 104.641024e6) * 8,     # 2 -> 16 batches (the CTA-pair kernel)
    "c1": 16.793088e6 + 0.0,                     # captured at full size (y stays in L2 at kernel end)
    "c5": (143.738112e6 + 14.620416e6) * 8 + 2 * 268.435456e6,   # 32 -> 256 (b,h) pairs, + pre-pass
}

# The reference emitter's PTX for each full-size configuration (tests/golden/make_golden.py).
REF_PTX_FULL = ROOT / "tests" / "golden" / "ref_ptx_full"


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


# ---- tolerance (the bars the north star states) --------------------------------------------------

def check_verdict(key: str, check: dict) -> tuple[bool, str]:
    """Whether a configuration's ``check`` is inside its tolerance: bit-exact for the i32 sum, 1e-5
    relative for the f32 sum and softmax, one bf16 unit for bf16 outputs (the fused kernel; the
    attention against max(|ref|, row rms)), 1e-4 of max(|ref|, rms) for the matmul."""
    if key == "c2i":
        ok = check["abs_err"] == 0 and check.get("global_abs_err", 0) == 0
        return ok, "bit-exact"
    if key == "c2":
        # the configuration's output is the global scalar: at N > 1 the bound applies to the exchanged
        # total; a rank's partial is an intermediate whose shard may cancel to near zero, where a
        # relative bound on it says nothing about the kernel (its error is reported all the same)
        if "global_rel_err" in check:
            return check["global_rel_err"] <= 1e-5, "1e-5 relative on the global total"
        return check["rel_err"] <= 1e-5, "1e-5 relative"
    if key == "c1":
        return check["max_err_over_bound"] <= 1.0, "1e-5 relative (floor 1e-5 of the largest |y|)"
    if key == "c3":
        return check["max_err_over_bound"] <= 1.0, "one bf16 ulp (2^-7 relative) + 1e-6"
    if key == "c4":
        return check["max_err_over_bound"] <= 1.0, "1e-4 of max(|ref|, rms)"
    if key == "c5":
        return check["max_err_over_bound"] <= 1.0, "one bf16 ulp of max(|ref|, row rms)"
    raise ValueError(key)


# ---- clocks -------------------------------------------------------------------------------------

CLOCK_FIELDS = ["timestamp", "index", "uuid", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.active",
                "clocks_event_reasons.hw_slowdown", "clocks_event_reasons.hw_thermal_slowdown",
                "clocks_event_reasons.sw_thermal_slowdown", "clocks_event_reasons.sw_power_cap"]


class ClockSampler:
    """nvidia-smi sampling every 200 ms for the whole run; ``summary(t0, t1)`` reads a time window.
    ``uuids`` (set by the caller) restricts the summary to the GPUs the job's ranks run on, so a job on
    4 GPUs of an 8-GPU box reports its own clocks, not the idle GPUs'."""

    def __init__(self):
        self.proc = None
        self.file = None
        self.rows = None
        self.uuids: set | None = None

    def start(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", "--query-gpu=" + ",".join(CLOCK_FIELDS),
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=self.file, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> None:
        if self.proc is None:
            return
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
            r = dict(zip(CLOCK_FIELDS, parts))
            try:
                r["t"] = datetime.datetime.strptime(r["timestamp"], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                r["t"] = None
            rows.append(r)
        os.unlink(self.file.name)
        self.rows = rows

    def summary(self, t0: float | None = None, t1: float | None = None) -> dict | None:
        """Median SM clock and the throttle reasons seen under load, over [t0, t1] (the whole run
        when no window is given, or when the window holds no sample)."""
        if not self.rows:
            return None
        rows = self.rows
        if t0 is not None:
            win = [r for r in rows if r["t"] is not None and t0 - 0.25 <= r["t"] <= t1 + 0.25]
            rows = win or rows

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        if self.uuids:
            mine = [r for r in rows if r["uuid"].removeprefix("GPU-").lower() in self.uuids]
            rows = mine or rows
        by_gpu = {}
        for r in rows:
            by_gpu.setdefault(r["index"], []).append(r)
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


# ---- the CPU oracle (the port leg and the reference arm) ----------------------------------------

def _oracle_worker(args):
    """Interpret a block range of the problem's kernel (spawned process).  Returns how many output
    elements the range wrote: the outputs themselves are full-size arrays (zero pages until written),
    and shipping them back to the parent would time a pickle of up to 1 GB instead of the kernel."""
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
    return sum(int(np.count_nonzero(bufs[a.name])) for a in p.outputs)


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
    it, so the sample is set per kernel: the whole grid for the sums (about 3 s in one process), a
    part of it for the softmax and the fused kernel (1-4 s), and one block per worker for the
    contraction kernels (3-4 s per block)."""
    per = {"c1": p.grid // 16, "c2": p.grid, "c2i": p.grid, "c3": p.grid // 8}.get(key)
    if per is None:
        per = max(1, workers)
    elif workers > 1:
        per = min(p.grid, per * 2)
    return max(1, min(p.grid, per))


# ---- the torch-CPU baseline ---------------------------------------------------------------------

def torch_cpu_leg(key: str, p, t: dict, units: float, unit: str, budget_s: float = 6.0) -> dict:
    """The configuration's source expression in torch on every host core, on a stated sample of the
    workload (whole tensors for the streaming configs, some batches / heads for the contractions),
    repeated until ``budget_s`` has passed (at least twice after a warm-up)."""
    import torch
    import torch.nn.functional as F
    threads0 = torch.get_num_threads()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    try:
        frac = 1.0
        if key == "c1":
            x = t["x"]
            fn, sample = (lambda: torch.softmax(x, -1)), "the whole [4096,1024] tensor: torch.softmax(x, -1)"
        elif key in ("c2", "c2i"):
            x = t["x"]
            fn, sample = (lambda: x.sum()), f"the whole {tuple(x.shape)} tensor: x.sum()"
        elif key == "c3":
            a, b, c, d = (t[n] for n in "abcd")
            fn = lambda: (torch.relu(a.float() * b.float() + c) * torch.exp(d.float())).to(torch.bfloat16)
            sample = "the whole [8192,8192] problem: relu(a*b+c)*exp(d) in fp32 from bf16, cast to bf16"
        elif key == "c4":
            nb = 1
            A, B = t["A"][:nb].float(), t["B"][:nb].float()
            frac = nb / t["A"].shape[0]
            fn = lambda: torch.bmm(A, B)
            sample = f"{nb} of {t['A'].shape[0]} batches: torch.bmm in fp32 from bf16 inputs (scaled linearly)"
        elif key == "c5":
            nh = 8
            q, k, v = (t[n][0, :nh].float() for n in ("Q", "K", "V"))
            frac = nh / (t["Q"].shape[0] * t["Q"].shape[1])
            fn = lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True).to(torch.bfloat16)
            sample = (f"{nh} of {t['Q'].shape[0] * t['Q'].shape[1]} (batch, head) pairs: "
                      "scaled_dot_product_attention(is_causal=True) in fp32 from bf16 (scaled linearly)")
        else:
            raise ValueError(key)
        fn()
        times = []
        t_end = time.perf_counter() + budget_s
        while len(times) < 2 or (time.perf_counter() < t_end and len(times) < 20):
            t0 = time.perf_counter()
            fn()
            times.append(time.perf_counter() - t0)
        sec = statistics.median(times)
    finally:
        torch.set_num_threads(threads0)
    scale = 1e9 if unit == "GB/s" else 1e12
    return {"value": units * frac / sec / scale, "unit": unit, "cores": cores, "kind": "torch",
            "sample": sample, "seconds_per_sample": sec, "repeats": len(times),
            "cpu": _cpu_model()}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_port_leg(key: str, p, t_cpu: dict, units: float, unit: str, ir_kw: dict) -> dict:
    """The numpy oracle on a bounded sample of the thread blocks, one process."""
    blocks = sample_blocks_for(key, p, 1)
    pool = OraclePool(key, t_cpu, 1, blocks, ir_kw)
    t0 = time.perf_counter()
    pool.step()
    dt = time.perf_counter() - t0
    pool.close()
    frac = pool.sample_blocks / p.grid
    scale = 1e9 if unit == "GB/s" else 1e12
    return {"value": units * frac / dt / scale, "unit": unit, "cores": 1, "kind": "port",
            "sample": f"{pool.sample_blocks} of {p.grid} thread blocks ({100 * frac:.2f}% of one step) "
                      f"through the numpy oracle, one process", "seconds": dt}


# ---- main -----------------------------------------------------------------------------------------

def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="all", choices=["all"] + ALL_KEYS)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong: the ranks share one global problem; weak: every rank runs a full-size one")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="how the sum's partials combine at N>1: the peer-exchange kernel over NVLink (falls back "
                         "to NCCL when the ranks cannot map each other's memory) or one ncclAllReduce")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-ref-emitter", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="launch every step from the host instead of CUDA graphs")
    ap.add_argument("--size", default="full", choices=["full", "small"],
                    help="small: a reduced instance of the same kernel (still larger than L2) for ncu captures")
    ap.add_argument("--opt", action="append", default=[], metavar="KEY=VALUE",
                    help="a compile option (value read as JSON when it parses), e.g. --opt attn_persistent=true")
    ap.add_argument("--ir", action="append", default=[], metavar="KEY=VALUE",
                    help="an argument of the workload's IR builder, e.g. --ir recip=true for config 1")
    return ap.parse_args(argv)


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
    """Whether this run captures CUDA graphs: unless switched off, at any number of ranks.  Captures
    use thread-local capture mode (the process group's watchdog thread may query events meanwhile)
    and never hold an NCCL call."""
    return not no_graph


def capture_steps(collective: bool, no_graph: bool, world: int = 1) -> bool:
    """Whether the timed steps are replayed from a CUDA graph: yes, unless graphs are off or a step
    holds the ncclAllReduce.  NCCL calls stay out of graphs: a live graph that holds one keeps the
    communicator's teardown waiting."""
    return use_graphs(world, no_graph) and not collective


def keys_for(config: str) -> list[str]:
    return list(ALL_KEYS) if config == "all" else [config]


def reference_arm(args, world, rank):
    """The reference's CPU implementation of the path (the oracle port) on every host core, for each
    configuration of the run; one line like ours, with ``"impl": "reference"``."""
    if rank != 0:
        return 0
    from emmy_ptx_b200 import irgen, data
    cores = os.cpu_count() or 1
    workers = max(1, min(cores, 64))
    per = {}
    for key in keys_for(args.config):
        p = irgen.FULL[key]()
        units, kind = work_units(p)
        desc, metric, unit = CONFIGS[key]
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
        sample = (f"{pool.sample_blocks} of {p.grid} thread blocks ({100 * frac:.2f}% of the workload) per step, "
                  f"{workers} spawned worker processes")
        per[key] = {"metric": f"{desc} {metric}", "value": value, "unit": unit, "ms_per_step": ms,
                    "cpu_baseline": {"value": value, "unit": unit, "cores": workers, "kind": "port", "sample": sample},
                    "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        del tensors
    head = per[HEADLINE] if HEADLINE in per else per[keys_for(args.config)[0]]
    hk = HEADLINE if HEADLINE in per else keys_for(args.config)[0]
    line = {
        "impl": "reference", "metric": head["metric"], "value": head["value"], "unit": head["unit"],
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": head["ms_per_step"],
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": irgen.FULL[hk]().args[0].dtype, "data": "synthetic (seeded, CPU-generated)",
        "config": {"workload": hk, "description": CONFIGS[hk][0], "configs": list(per)},
        "cpu_baseline": head["cpu_baseline"], "e2e": head["e2e"], "per_config": per,
    }
    print(json.dumps(line), flush=True)
    return 0


class CheckFailed(Exception):
    pass


class KernelTimedOut(Exception):
    pass


def _gen_tensor(spec, shape, gen_seed: int, device: str):
    """One input drawn on the device from its spec's distribution with a fixed seed."""
    import torch
    from emmy_ptx_b200 import data
    gen = torch.Generator(device=device).manual_seed(gen_seed & 0x7FFFFFFFFFFFFFFF)
    if spec.dist[0] == "normal":
        t = torch.randn(shape, generator=gen, device=device) * spec.dist[1]
    elif spec.dist[0] == "uniform":
        t = torch.rand(shape, generator=gen, device=device) * (spec.dist[2] - spec.dist[1]) + spec.dist[1]
    else:
        return torch.randint(spec.dist[1], spec.dist[2], shape, generator=gen, device=device, dtype=torch.int32)
    return t.to(data.torch_dtype(spec.dtype))


def make_sets(key, p, p_global, rotate, world, rank, scaling, shard_lo, shard_hi):
    """``rotate`` input sets on the device.  Strong scaling: every rank draws the GLOBAL tensors with
    the global seeds and keeps its slice along the sharded axis; weak scaling: every rank draws its own
    full-size tensors with rank-dependent seeds."""
    import torch
    from emmy_ptx_b200 import data
    sets = []
    for r in range(rotate):
        t = {}
        for a in p.args:
            if a.output:
                t[a.name] = torch.zeros(tuple(a.shape), dtype=data.torch_dtype(a.dtype), device="cuda")
                continue
            if scaling == "strong":
                g = p_global.spec(a.name)
                full = _gen_tensor(g, tuple(g.shape), g.seed + 7919 * r, "cuda")
                if a.name in SHARDED[key] and world > 1:
                    full = full[shard_lo:shard_hi].contiguous()
                t[a.name] = full
            else:
                t[a.name] = _gen_tensor(a, tuple(a.shape), a.seed + 7919 * r + 104729 * rank, "cuda")
        sets.append(t)
    return sets


def correctness(key, p, t, ex, step, dist, collective, stream, fused: bool = False) -> dict:
    """The timed output (rank-local shard) against float64, as the tolerance measures it."""
    import torch
    ex(t, stream)
    torch.cuda.synchronize()
    fam = p.family
    if fam == "sum":
        want = t["x"].double().sum().item() if p.params["dtype"] == "f32" else int(t["x"].long().sum().item())
        got = t["out"].item()
        if fused:
            # the kernel's output is already the exchanged total of every rank's partial
            tot = torch.tensor([float(want)], dtype=torch.float64, device="cuda")
            dist.all_reduce(tot)
            e = abs(got - tot.item())
            r = e / max(abs(tot.item()), 1e-30)
            return {"abs_err": e, "rel_err": r, "global_abs_err": e, "global_rel_err": r,
                    "partial": "exchanged inside the kernel (no rank-local partial to check)"}
        check = {"abs_err": abs(got - want), "rel_err": abs(got - want) / max(abs(want), 1e-30)}
        if collective:
            # the exchange step too: kernel + ncclAllReduce against the all-reduced float64 shard sums
            step(t)
            torch.cuda.synchronize()
            tot = torch.tensor([float(want)], dtype=torch.float64, device="cuda")
            dist.all_reduce(tot)
            g_all = t["out"].item()
            check["global_abs_err"] = abs(g_all - tot.item())
            check["global_rel_err"] = abs(g_all - tot.item()) / max(abs(tot.item()), 1e-30)
        return check
    if fam == "softmax":
        want = torch.softmax(t["x"].double(), -1)
        err = (t["y"].double() - want).abs()
        bound = 1e-5 * want.abs() + 1e-5 * 1e-5 * want.abs().max()
        return {"max_rel_err": (err / want.abs().clamp_min(1e-30)).max().item(),
                "max_err_over_bound": (err / bound).max().item()}
    if fam == "fused":
        want = torch.relu(t["a"].double() * t["b"].double() + t["c"].double()) * torch.exp(t["d"].double())
        err = (t["y"].double() - want).abs()
        bound = 2.0 ** -7 * want.abs() + 1e-6
        return {"max_rel_err_vs_f64": (err / want.abs().clamp_min(1e-6)).max().item(),
                "max_err_over_bound": (err / bound).max().item()}
    if fam == "bmm":
        # the first and the last batch of this shard (the persistent GEMM's first and last tiles)
        worst = 0.0
        batches = sorted({0, p.params["batch"] - 1})
        for b in batches:
            want = t["A"][b].double() @ t["B"][b].double()
            den = torch.clamp(want.abs(), min=want.pow(2).mean().sqrt().item())
            worst = max(worst, ((t["C"][b].double() - want).abs() / den).max().item())
        return {"batches_checked": batches, "max_err_over_rms_floor": worst,
                "max_err_over_bound": worst / 1e-4}
    if fam == "attention":
        # (first batch, head 0) and (last batch, last head) of this shard against float64
        worst = 0.0
        pairs = sorted({(0, 0), (p.params["batch"] - 1, p.params["heads"] - 1)})
        for b, h in pairs:
            q, k, v = (t[n][b, h].double() for n in ("Q", "K", "V"))
            s_ = (q @ k.T) * p.params["scale"]
            if p.params.get("causal", True):
                s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
            want = torch.softmax(s_, -1) @ v
            den = torch.maximum(want.abs(), want.pow(2).mean(-1, keepdim=True).sqrt()) * 2.0 ** -7
            worst = max(worst, ((t["O"][b, h].double() - want).abs() / den).max().item())
        return {"heads_checked": [list(x) for x in pairs], "max_err_bf16_units": worst,
                "max_err_over_bound": worst}
    raise ValueError(fam)


def graph_of(fn, capture=True):
    """A CUDA graph of ``fn(stream)`` captured in thread-local mode (None when ``capture`` is false)."""
    import torch
    if not capture:
        return None
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        fn(torch.cuda.current_stream().cuda_stream)
    g.replay()
    torch.cuda.synchronize()
    return g


def timed(fn, dist, max_over_ranks, n: int = 1) -> float:
    """Milliseconds per unit of ``fn()`` (which queues ``n`` units on the current stream): CUDA events
    around it, a barrier and a synchronize on both sides, max over ranks."""
    import torch
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    fn()
    e1.record()
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    return max_over_ranks(dist, e0.elapsed_time(e1) / n)


def ref_emitter_leg(key, p, sets, rotate, reps_hint, no_graph) -> dict | None:
    """The reference emitter's PTX for this full-size IR, launched like ours: same geometry, buffers,
    rotation and graph replay.  Returns its per-launch time and a float64 check of its output."""
    import torch
    from emmy_ptx_b200.launcher import Device
    f = REF_PTX_FULL / f"{key}.ptx"
    if not f.exists():
        return {"unavailable": f"no reference PTX for {key} (see tests/golden/ref_ptx_full/manifest.json)"}
    dev = Device.get(torch.cuda.current_device())
    mod = dev.load_ptx(f.read_text())
    fn = dev.function(mod, p.entry)
    smem = int(p.smem_bytes or 0)
    if smem > 48 * 1024:
        dev.set_max_dyn_smem(fn, smem)

    def launch(t, s):
        for name in p.zero_outputs:
            nb = t[name].numel() * t[name].element_size()
            dev.memset_d32(t[name].data_ptr(), 0, nb // 4, s)
        dev.launch_u64(fn, [p.grid, 1, 1], [p.block, 1, 1], smem, s, [t[n].data_ptr() for n in p.arg_order])

    stream = torch.cuda.current_stream().cuda_stream
    launch(sets[0], stream)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    launch(sets[0], stream)
    torch.cuda.synchronize()
    one = time.perf_counter() - t0
    reps = max(2, min(reps_hint, int(2.0 / max(one, 1e-6))))      # about two seconds at most
    g = graph_of(lambda s: [launch(sets[i % rotate], s) for i in range(reps)], capture=not no_graph)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    if g is not None:
        g.replay()
    else:
        for i in range(reps):
            launch(sets[i % rotate], stream)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    del g
    dev.unload(mod)
    return {"kernel": p.entry, "ref_kernel_ms": ms, "launches_timed": reps,
            "ptx": f"tests/golden/ref_ptx_full/{key}.ptx (the reference compile.py, run unmodified)"}


def run_config(key, args, world, rank, local, dist, peaks, peak_src, clocks) -> dict:
    """Everything measured for one configuration; raises CheckFailed / KernelTimedOut."""
    import torch
    from emmy_ptx_b200 import dist as edist
    from emmy_ptx_b200.compiler import compile_graph
    from emmy_ptx_b200.ir import Graph
    from emmy_ptx_b200.runtime import Executable
    max_over_ranks = edist.max_over_ranks
    t_start = time.time()
    ir_kw = compile_options(args.ir)
    options = compile_options(args.opt)
    strong = args.scaling == "strong" and world > 1 and args.size == "full"
    if args.size == "small":
        p_global = SMALL_FOR_PROFILE[key](**ir_kw)
        p = p_global
        lo, hi = 0, 0
    else:
        p_global = build_problem(key, None, **ir_kw)
        if strong:
            sh = edist.shard(SHARD_UNITS[key], world, rank)
            lo, hi = sh.start, sh.stop
            p = build_problem(key, hi - lo, **ir_kw)
        else:
            lo, hi = 0, SHARD_UNITS[key]
            p = p_global
    units, kind = work_units(p)                      # this rank's work per step
    g_units = work_units(p_global)[0] if strong else world * units
    desc, metric, unit = CONFIGS[key]
    scale = 1e9 if unit == "GB/s" else 1e12

    from emmy_ptx_b200.launcher import Device
    dev = Device.get(local)
    collective = p.family == "sum" and world > 1
    allreduce, exchange, fused = None, None, False
    if collective:
        if args.exchange == "peer":
            try:
                allreduce = edist.PeerAllReduce(dev, dist, rank, world, p.params["dtype"])
                exchange, fused = "peer (NVLink exchange fused into the reduction kernel)", True
            except RuntimeError as exc:         # the same on every rank (the set-up agrees)
                exchange = f"nccl (peer exchange unavailable: {exc})"
        if allreduce is None:
            allreduce = edist.AllReducePartials(dev, dist, rank, world)
            exchange = exchange or "nccl"
    nccl_in_step = collective and not fused
    build_opts = dict(options)
    if fused:
        # the last block of the reduction publishes the partial and adds every rank's (kernels/peer_sum.py)
        build_opts["exchange"] = {"rank": rank, "world": world, "partial": "out", "dtype": p.params["dtype"]}
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), build_opts)
    ex = Executable(mod, device=local)
    stream = torch.cuda.current_stream().cuda_stream

    rotate = 1
    if units < 2 * 126e6 and kind == "B":      # L2-resident working set: rotate buffer sets past 2x L2
        rotate = int(max(2, (2 * 126e6 * 2) // units + 1))
    sets = make_sets(key, p, p_global, rotate, world, rank, "strong" if strong else "weak", lo, hi)
    if fused:
        for t_ in sets:
            t_["__xch"], t_["__peers"] = allreduce.xch, allreduce.table
    try:
        def step(t, s=None):
            s = stream if s is None else s
            ex(t, s)
            if nccl_in_step:
                allreduce(t["out"], p.params["dtype"], s)

        for i in range(max(args.warmup, 3)):
            step(sets[i % rotate])
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

        reps = args.steps if units * 1.0 > 1e11 or kind == "FLOP" else max(args.steps, 200)
        graphs = use_graphs(world, args.no_graph)
        step_graph = graph_of(lambda s: [step(sets[i % rotate], s) for i in range(args.steps)],
                              capture=capture_steps(nccl_in_step, args.no_graph, world))
        kern_graph = graph_of(lambda s: [ex.run(sets[i % rotate], s, zero=False) for i in range(reps)],
                              capture=graphs)
        t_timed0 = time.time()
        if step_graph is not None:
            ms_step = timed(step_graph.replay, dist, max_over_ranks, args.steps)
        else:
            ms_step = timed(lambda: [step(sets[i % rotate]) for i in range(args.steps)], dist, max_over_ranks,
                            args.steps)
        if kern_graph is not None:
            kern_ms = timed(kern_graph.replay, dist, max_over_ranks, reps)
        else:
            kern_ms = timed(lambda: [ex.run(sets[i % rotate], stream, zero=False) for i in range(reps)], dist,
                            max_over_ranks, reps)
        allreduce_ms = None
        if nccl_in_step:
            n_ar = 50
            allreduce_ms = timed(lambda: [allreduce(sets[0]["out"], p.params["dtype"], stream) for _ in range(n_ar)],
                                 dist, max_over_ranks, n_ar)
        elif fused:
            # the exchange's cost: the fused kernel against the same reduction without its epilogue
            plain = Executable(compile_graph(Graph.from_dict(p.graph), p.meta(), options), device=local)
            g_plain = graph_of(lambda s: [plain.run(sets[i % rotate], s, zero=False) for i in range(reps)],
                               capture=graphs)
            plain_ms = timed(g_plain.replay if g_plain is not None else
                             (lambda: [plain.run(sets[i % rotate], stream, zero=False) for i in range(reps)]),
                             dist, max_over_ranks, reps)
            allreduce_ms = kern_ms - plain_ms
            g_plain = None
            plain.close()
        t_timed1 = time.time()
        step_graph = kern_graph = None
        value = g_units / (ms_step / 1000.0) / scale

        check = correctness(key, p, sets[0], ex, step, dist, collective, stream, fused)
        ok, tol = check_verdict(key, check)
        check["tolerance"] = tol
        check["ok"] = ok
        bad = int(max_over_ranks(dist, 0.0 if ok else 1.0))
        code = int(max_over_ranks(dist, float(max(ex.error_code(),
                                                  allreduce.error_code() if hasattr(allreduce, "error_code") else 0))))
        if code:
            raise KernelTimedOut(f"{key}: kernel status word {code}: a pipeline wait timed out")
        if bad:
            per_rank = [check]
            if dist:
                per_rank = [None] * world
                dist.all_gather_object(per_rank, check)
            raise CheckFailed(f"{key}: result outside the tolerance ({tol}) on some rank; checks by rank: "
                              f"{json.dumps(per_rank)}")

        # e2e: pinned host buffers, copies inside the timed region, through the C ABI.  Two device
        # buffer sets: step i's outputs travel back to the host on a second stream while step i+1's
        # inputs come over on the first (PCIe carries both directions at once); every step still
        # copies its own inputs in and its own outputs out inside the timed region
        e2e = None
        if not args.no_e2e:
            t = sets[0]
            t2 = dict(sets[1]) if rotate > 1 else dict(t)
            if rotate == 1:
                for a in p.args:
                    t2[a.name] = torch.empty_like(t[a.name])
            tb = [t, t2]
            host = {a.name: t[a.name].cpu().pin_memory() for a in p.args}
            h2d = sum(host[a.name].numel() * host[a.name].element_size() for a in p.inputs)
            d2h = sum(host[a.name].numel() * host[a.name].element_size() for a in p.outputs)
            e2e_steps = max(3, min(args.steps, 10))
            s_out = dev.stream()
            computed = [dev.sync_event(), dev.sync_event()]
            returned = [dev.sync_event(), dev.sync_event()]
            used = [False, False]

            def e2e_step(i):
                b = i % 2
                tt = tb[b]
                if used[b]:
                    dev.wait_event(stream, returned[b])      # set b's last outputs are on the host
                for a in p.inputs:
                    dev.htod(tt[a.name].data_ptr(), host[a.name].data_ptr(),
                             host[a.name].numel() * host[a.name].element_size(), stream)
                step(tt)
                dev.record(computed[b], stream)
                dev.wait_event(s_out, computed[b])
                for a in p.outputs:
                    dev.dtoh(host[a.name].data_ptr(), tt[a.name].data_ptr(),
                             host[a.name].numel() * host[a.name].element_size(), s_out)
                dev.record(returned[b], s_out)
                used[b] = True

            def e2e_run(n):
                for i in range(n):
                    e2e_step(i)
                for b in range(2):                          # the timed region ends after the last copy out
                    if used[b]:
                        dev.wait_event(stream, returned[b])

            e2e_run(2)
            e2e_ms = timed(lambda: e2e_run(e2e_steps), dist, max_over_ranks, e2e_steps)
            dev.sync()
            for ev in computed + returned:
                dev.destroy_event(ev)
            dev.destroy_stream(s_out)
            e2e = {"value": g_units / (e2e_ms / 1000.0) / scale, "unit": unit, "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "ms_per_step": e2e_ms, "steps": e2e_steps,
                   "path": "pinned host -> cuMemcpyHtoDAsync -> kernel -> cuMemcpyDtoHAsync (libemmy_launch.so); "
                           "two device buffer sets, step i's copy out on a second stream beside step i+1's copy in"}
            del host, tb, t2

        # context for small byte-bound launches: a plain device copy moving the same number of bytes
        copy_ref = None
        if kind == "B" and graphs:
            nb = int(units // 2) // 4
            pairs = [(torch.ones(nb, dtype=torch.float32, device="cuda"), torch.empty(nb, dtype=torch.float32, device="cuda"))
                     for _ in range(rotate)]
            g_copy = graph_of(lambda s: [torch.mul(pairs[i % rotate][0], 1.0, out=pairs[i % rotate][1])
                                         for i in range(reps)])
            copy_ms = timed(g_copy.replay, dist, max_over_ranks, reps)
            del g_copy, pairs
            copy_ref = {"achieved": units / (copy_ms / 1000.0) / scale, "ms_per_launch": copy_ms,
                        "how": "torch elementwise y = x * 1 over the same bytes (half read, half written), "
                               "same rotation, graph replay"}

        achieved = units / (kern_ms / 1000.0) / scale
        if copy_ref:
            copy_ref["kernel_frac_of_copy"] = achieved / copy_ref["achieved"]
        if unit == "GB/s":
            peak, bound, peak_key = peaks["hbm_gbs"], "hbm", "hbm_gbs"
        else:
            peak_key = "bf16_tflops_sustained" if kern_ms > 100 else "bf16_tflops"
            peak, bound = peaks.get(peak_key, 1590.0), "tensor"
        traffic = TRAFFIC.get(key) if not strong and args.size == "full" else None
        if traffic is not None and strong:
            traffic = traffic * units / work_units(p_global)[0]
        roof = {"bound": bound, "achieved": achieved, "peak": peak, "unit": unit, "frac": achieved / peak,
                "traffic": traffic,
                "peak_source": f"{peak_src} ({peak_key}, MEASURED_PEAKS.json)" if peak_src == "measured" else "fallback",
                "kernel": mod.kernels[-1]["entry"], "kernel_ms": kern_ms, "kernel_launches_timed": reps,
                "kernel_entries_timed": [k["entry"] for k in mod.kernels],
                "algorithmic_per_launch": units, "algorithmic_unit": kind, "same_bytes_copy": copy_ref}

        ref = None
        if world == 1 and args.size == "full" and not args.no_ref_emitter and not ir_kw:
            ref = ref_emitter_leg(key, p, sets, rotate, reps, args.no_graph)
            if ref and "ref_kernel_ms" in ref:
                ref["kernel_ms_over_ref_kernel_ms"] = kern_ms / ref["ref_kernel_ms"]
                ref["ref_achieved"] = units / (ref["ref_kernel_ms"] / 1000.0) / scale

        cpu = port = None
        if rank == 0 and world == 1 and not args.no_cpu_baseline and args.size == "full":
            tc = {a.name: sets[0][a.name].cpu() for a in p.args}
            cpu = torch_cpu_leg(key, p, tc, units, unit)
            port = cpu_port_leg(key, p, tc, units, unit, ir_kw)
            del tc
        t_end = time.time()
    finally:
        torch.cuda.synchronize()
        if collective:
            if dist:
                dist.barrier()               # every rank is done with the peers' exchange buffers
            allreduce.close()
        ex.close()
        del sets
        torch.cuda.empty_cache()

    rec = {
        "metric": f"{desc} {metric}", "value": value, "unit": unit, "ms_per_step": ms_step, "dtype": p.args[0].dtype,
        "config": {"workload": key, "description": desc, "per_rank_units": units, "global_units": g_units,
                   "unit_kind": kind,
                   "parallelism": f"dp{world} ({'sharded + ' + exchange + ' of the partial' if collective else 'sharded, no collective'})",
                   "shard": ([lo, hi] if strong else None),
                   "l2": ("inputs exceed L2 (126 MB)" if rotate == 1 else f"{rotate} rotating buffer sets exceed 2x L2"),
                   "grid": p.grid, "block": p.block, **({"compile_options": options} if options else {}),
                   **({"ir_options": ir_kw} if ir_kw else {})},
        "gpu_launches": args.steps * len(mod.kernels),
        "timing": ("CUDA graph replay of the K steps" if capture_steps(nccl_in_step, args.no_graph, world)
                   else "host launches (kernel + ncclAllReduce per step)" if nccl_in_step else "host launches"),
        "roofline": roof, "ref_emitter": ref, "cpu_baseline": cpu, "cpu_port": port, "e2e": e2e,
        "check": check, "kernel_kind": mod.kernels[-1].get("kind"),
        "clocks_window": [t_timed0, t_timed1], "wall_s": t_end - t_start,
    }
    if allreduce_ms is not None:
        rec["exchange"] = exchange
        rec["exchange_ms"] = allreduce_ms
        rec["kernel_ms"] = kern_ms
    return rec


def main(argv=None) -> int:
    args = parse(argv)
    from emmy_ptx_b200 import dist as edist
    world, rank, local = edist.env()
    if args.impl == "reference":
        return reference_arm(args, world, rank)
    import torch
    dist = edist.init(world, local)
    peaks, peak_src = load_peaks()
    clocks = ClockSampler() if local == 0 else None
    # the GPUs this job runs on (every rank's), for the clock summary
    uuid = str(torch.cuda.get_device_properties(local).uuid).removeprefix("GPU-").lower()
    uuids = [uuid]
    if dist:
        uuids = [None] * world
        dist.all_gather_object(uuids, uuid)
    if clocks:
        clocks.uuids = set(uuids)
        clocks.start()
        time.sleep(0.3)
    per = {}
    failure = None
    rc = 0
    try:
        for key in keys_for(args.config):
            per[key] = run_config(key, args, world, rank, local, dist, peaks, peak_src, clocks)
    except KernelTimedOut as exc:
        failure, rc = str(exc), 3
    except CheckFailed as exc:
        failure, rc = str(exc), 4
    finally:
        if clocks:
            clocks.stop()
    if failure:
        if rank == 0:
            print(json.dumps({"error": failure}), file=sys.stderr, flush=True)
        if dist:
            dist.barrier()
            dist.destroy_process_group()
        return rc
    for key, rec in per.items():
        w = rec.pop("clocks_window")
        rec["clocks"] = clocks.summary(*w) if clocks else None
    if rank == 0:
        hk = HEADLINE if HEADLINE in per else next(iter(per))
        h = per[hk]
        line = {
            "metric": h["metric"], "value": h["value"], "unit": h["unit"], "n_gpus": world, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": h["ms_per_step"], "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": h["dtype"],
            "data": "synthetic (seeded on device)", "config": {**h["config"], "configs": list(per)},
            "gpu_launches": h["gpu_launches"], "timing": h["timing"], "roofline": h["roofline"],
            "cpu_baseline": h["cpu_baseline"], "e2e": h["e2e"],
            "clocks": clocks.summary() if clocks else None, "check": h["check"], "kernel_kind": h["kernel_kind"],
            "ref_emitter": h["ref_emitter"],
            "per_config": {k: {kk: vv for kk, vv in rec.items()} for k, rec in per.items()},
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
