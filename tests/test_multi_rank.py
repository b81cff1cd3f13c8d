"""Multi-process host logic on CPU: two gloo ranks, no GPU.

Covers the sharding of units, the unique-id broadcast, the max-over-ranks timing reduction, the
weak-scaled sum (partials combined by an all-reduce, bit-exact for integers), and failure detection: a
rank that leaves before the collective makes the others fail within the process-group timeout instead
of hanging.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from emmy_ptx_b200 import dist as edist


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _setup(rank, world, port, timeout_s=30.0):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    return edist.init(world, rank, backend="gloo", timeout_s=timeout_s)


def _worker_basic(rank, world, port, q):
    d = _setup(rank, world, port)
    try:
        uid = edist.share_unique_id(d, rank, lambda: bytes(range(128)))
        mx = edist.max_over_ranks(d, float(rank + 1) * 1.5)
        # weak-scaled integer sum: each rank owns a full shard, partials all-reduced
        g = torch.Generator().manual_seed(100 + rank)
        x = torch.randint(-1000, 1001, (1 << 16,), generator=g, dtype=torch.int32)
        part = torch.tensor([int(x.long().sum())], dtype=torch.int64)
        d.all_reduce(part)
        q.put((rank, uid == bytes(range(128)), mx, int(part.item())))
    finally:
        d.destroy_process_group()


def test_two_gloo_ranks_share_uid_max_and_partials():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_basic, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    want = 0
    for r in range(world):
        g = torch.Generator().manual_seed(100 + r)
        want += int(torch.randint(-1000, 1001, (1 << 16,), generator=g, dtype=torch.int32).long().sum())
    for rank, uid_ok, mx, total in res:
        assert uid_ok and mx == 3.0 and total == want


def _worker_dies(rank, world, port, q):
    d = _setup(rank, world, port, timeout_s=5.0)
    if rank == 1:
        os._exit(0)                      # leaves between steps, before the collective
    try:
        edist.max_over_ranks(d, 1.0)
        q.put("returned")
    except Exception as exc:             # the process-group timeout ends the collective with an error
        q.put("error:" + type(exc).__name__)


def test_a_rank_that_leaves_fails_the_collective_instead_of_hanging():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_dies, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error:")


@pytest.mark.parametrize("n,world", [(4096, 2), (4096, 8), (16, 3), (7, 4), (256, 8)])
def test_shards_cover_every_unit_once(n, world):
    seen = np.zeros(n, dtype=int)
    for r in range(world):
        for i in edist.shard(n, world, r):
            seen[i] += 1
    assert (seen == 1).all()


def test_nccl_steps_are_never_captured_in_a_graph():
    """The sum's multi-GPU step holds an ncclAllReduce; bench.py times it with host launches, since a
    live CUDA graph that holds an NCCL call keeps the communicator's teardown waiting.  Steps without
    a collective are graph-replayed, at any number of ranks, unless graphs are switched off."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("bench_mod", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench.capture_steps(collective=True, no_graph=False) is False
    assert bench.capture_steps(collective=True, no_graph=False, world=8) is False
    assert bench.capture_steps(collective=False, no_graph=False) is True
    assert bench.capture_steps(collective=False, no_graph=True) is False
    assert bench.capture_steps(collective=False, no_graph=False, world=8) is True
    assert bench.use_graphs(world=2, no_graph=False) is True
    assert bench.use_graphs(world=1, no_graph=True) is False


def test_bench_compile_options_parse():
    import bench
    assert bench.compile_options(["attn_persistent=true", "sms=148", "name=x"]) == {
        "attn_persistent": True, "sms": 148, "name": "x"}
    with pytest.raises(SystemExit):
        bench.compile_options(["novalue"])


def test_bench_reference_arm_runs_on_the_host():
    # the reference arm (the oracle port on host cores) needs no GPU: one line from rank 0, with the
    # contract's keys; another rank of a multi-GPU launch prints nothing and exits 0
    import json
    import os
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    cmd = [sys.executable, str(root / "bench.py"), "--impl", "reference", "--config", "c1", "--steps", "1",
           "--warmup", "0"]
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "GB/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["h2d_bytes_per_step"] == 0
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300,
                       env={**env, "RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert r.returncode == 0 and not r.stdout.strip()


def test_clock_summary_reads_only_the_jobs_gpus():
    """A job on some GPUs of a larger box summarises the clocks of its own GPUs (matched by UUID), not
    those of idle GPUs beside it."""
    import bench
    rows = []
    for idx, uu, mhz, pw in [("0", "GPU-AAAA-1", "1900", "700"), ("1", "GPU-BBBB-2", "300", "90"),
                             ("0", "GPU-AAAA-1", "1950", "710"), ("2", "GPU-CCCC-3", "345", "95")]:
        r = dict(zip(bench.CLOCK_FIELDS, ["2026/12/02 06:00:00.000", idx, uu, mhz, "1965", pw] + ["Not Active"] * 5))
        r["t"] = None
        rows.append(r)
    c = bench.ClockSampler()
    c.rows = rows
    c.uuids = {"aaaa-1"}
    s = c.summary()
    assert s["gpus"] == ["0"] and s["sm_mhz"] == 1925.0
    c.uuids = {"bbbb-2", "cccc-3"}
    assert c.summary()["gpus"] == ["1", "2"]
