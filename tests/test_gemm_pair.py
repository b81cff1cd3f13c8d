"""The CTA-pair GEMM (``tcgen05.mma.cta_group::2``, option ``gemm_pair``).

On the CPU the emitted PTX runs in the cluster emulator (:mod:`tests.tcemu_pair`): both CTAs of each
cluster scheduled together, their TMA halves completing CTA 0's barriers, the pair MMA reading both
CTAs' shared memory and writing both tensor memories.  It is compared with the oracle on tile
multiples, edge tiles and several tiles per cluster, with completions deferred until no thread can
run, and a planted mistake (a missing commit to the partner's ``empty`` barrier) must deadlock.  On
the B200 the same kernel runs against the oracle and against float64 at full size.
"""
import re

import numpy as np
import pytest
import torch

from emmy_ptx_b200 import data, irgen
from emmy_ptx_b200.compiler import CompiledModule
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.kernels import tc_gemm_pair as gp
from oracle.run import oracle_outputs
from tests.checks import compare
from tests.ptxemu import Memory
from tests.tcemu_pair import PairEmulator
from tests.test_tc_emulated import _np

OPTS = {"gemm_pair": True, "sms": 4}


def _run(p, mod, defer=False, seed=None):
    rec = mod.kernels[0]
    t = data.make_inputs(p)
    mem = Memory()
    addr = {n: mem.alloc(_np(x).copy()) for n, x in t.items()}
    err = mem.alloc(np.zeros(16, np.uint8))
    tm = {f"p_{s['name']}": (addr[s["tensor"]], s) for s in rec["tmaps"]}
    emu = PairEmulator(mod.ptx, rec["entry"], tm, defer=defer, seed=seed)
    args = {"p_A": addr["A"], "p_B": addr["B"], "p_C": addr["C"], **emu.tmap_args(), "p_err": err}
    emu.run(rec["grid"][0], rec["block"][0], args, mem, rec["dyn_smem"])
    got = torch.from_numpy(mem.array(addr["C"], np.float32, tuple(t["C"].shape)).copy())
    return t, got, int(mem.array(err, np.int32, (4,))[0])


@pytest.mark.parametrize("shape,defer", [
    ((1, 256, 256, 128), False),
    ((2, 512, 512, 256), False),       # 8 tiles over 2 clusters, the 7-stage ring wraps
    ((1, 300, 264, 72), False),        # edge tiles in M, N and K
    ((3, 130, 520, 200), False),
    ((2, 256, 512, 512), True),        # completions deferred until no thread can run
    ((1, 200, 264, 136), True),
    ((1, 1, 8, 8), False),             # one row, one 8-column group, one K step of 8
])
def test_pair_gemm_emulated_matches_oracle(shape, defer):
    p = irgen.bmm_naive_ir(*shape)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), OPTS)
    rec = mod.kernels[0]
    assert rec["kind"] == "tcgen05_gemm_pair" and rec["cluster"] == [2, 1, 1] and rec["grid"][0] % 2 == 0
    t, got, code = _run(p, mod, defer)
    assert code == 0
    compare(got, oracle_outputs(p, t)["C"], "f32", 1e-4, f"pair {shape}")


@pytest.mark.parametrize("stages", [2, 7])
def test_pair_gemm_ring_depths(stages):
    p = irgen.bmm_naive_ir(2, 256, 512, 512)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {**OPTS, "gemm_stages": stages})
    t, got, code = _run(p, mod, seed=stages)
    assert code == 0
    compare(got, oracle_outputs(p, t)["C"], "f32", 1e-4, f"pair stages {stages}")


@pytest.mark.parametrize("seed", range(6))
def test_pair_gemm_random_orders(seed):
    # threads stepped in a random order, loads landing in random subsets, the tensor core running a
    # random number of its queued MMAs and commits at a time: the same result every time
    p = irgen.bmm_naive_ir(2, 256, 512, 512) if seed % 2 == 0 else irgen.bmm_naive_ir(1, 300, 264, 200)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), OPTS)
    t, got, code = _run(p, mod, seed=seed)
    assert code == 0
    compare(got, oracle_outputs(p, t)["C"], "f32", 1e-4, f"pair seed {seed}")


def test_planted_missing_commit_to_the_partner_deadlocks():
    p = irgen.bmm_naive_ir(2, 256, 512, 512)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), OPTS)
    lines = mod.ptx.splitlines()
    commits = [i for i, ln in enumerate(lines) if "tcgen05.commit" in ln]
    assert len(commits) == 4                       # empty x 2 CTAs, tmem_full x 2 CTAs
    bad = "\n".join(lines[:commits[1]] + lines[commits[1] + 1:])   # CTA 1's empty barrier never arrives
    with pytest.raises(RuntimeError, match="deadlock"):
        _run(p, CompiledModule(bad, mod.kernels))


def test_planted_full_barrier_expecting_one_half_fails():
    # CTA 0's full barrier armed for its own half only: in random orders the accounting breaks
    # (the stage completes before the partner's bytes, or a later phase never completes)
    p = irgen.bmm_naive_ir(2, 256, 512, 512)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), OPTS)
    bad = mod.ptx.replace(f", {gp.TX_PAIR};", f", {gp.TX_PAIR // 2};")
    assert bad != mod.ptx
    for seed in range(3):
        try:
            t, got, code = _run(p, CompiledModule(bad, mod.kernels), seed=seed)
        except RuntimeError:
            continue
        want = oracle_outputs(p, t)["C"]
        assert code != 0 or (got.double() - want.double()).abs().max().item() > 1e-2


def test_pair_kernel_uses_no_multicast_and_assembles():
    import shutil
    import subprocess
    import tempfile
    from pathlib import Path
    from emmy_ptx_b200.codegen.module import module_text
    txt = module_text([gp.gemm_pair_entry("bmm", 16, 4096, 4096, 4096)])
    assert "multicast" not in txt
    assert len(re.findall(r"tcgen05\.mma\.cta_group::2", txt)) == 4
    ptxas = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
    with tempfile.TemporaryDirectory() as td:
        f = Path(td) / "k.ptx"
        f.write_text(txt)
        r = subprocess.run([ptxas, "-arch=sm_100a", "-v", str(f), "-o", str(Path(td) / "k.cubin")],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        assert "0 bytes spill" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1, 256, 256, 128), (2, 512, 512, 256), (1, 300, 264, 72), (3, 1000, 1000, 1000),
                                   (1, 1, 8, 8), (5, 257, 264, 520), (1, 4096, 8, 4096), (2, 130, 4096, 64)])
def test_pair_gemm_on_the_gpu(shape):
    from emmy_ptx_b200.runtime import Executable
    p = irgen.bmm_naive_ir(*shape)
    ex = Executable(compile_graph(Graph.from_dict(p.graph), p.meta(), {"gemm_pair": True}))
    t_cpu = data.make_inputs(p)
    t = {k: v.cuda() for k, v in t_cpu.items()}
    t["C"].fill_(float("nan"))
    ex(t)
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    want = (t_cpu["A"].double() @ t_cpu["B"].double())
    compare(t["C"].cpu(), want, "f32", 1e-4, f"pair {shape}")
    ex.close()


@pytest.mark.gpu
def test_pair_gemm_full_size_sampled():
    """Config 4 at full size through the pair kernel: batches 0, 7 and 15 against float64."""
    from emmy_ptx_b200.runtime import Executable
    p = irgen.FULL["c4"]()
    ex = Executable(compile_graph(Graph.from_dict(p.graph), p.meta(), {"gemm_pair": True}))
    assert ex.records[0]["kind"] == "tcgen05_gemm_pair"
    t = {k: v.cuda() for k, v in data.make_inputs(p).items()}
    ex(t)
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    for b in (0, 7, 15):
        want = t["A"][b].double() @ t["B"][b].double()
        compare(t["C"][b], want, "f32", 1e-4, f"pair c4 batch {b}")
    ex.close()


@pytest.mark.gpu
@pytest.mark.parametrize("opts", [{"gemm_stages": 2}, {"sms": 4}, {"sms": 6, "gemm_stages": 3}])
def test_pair_gemm_ring_and_cluster_counts_on_the_gpu(opts):
    """The shallowest ring, and two or three clusters walking many tiles each (the tile loop strides by
    the launched cluster count), against float64."""
    from emmy_ptx_b200.runtime import Executable
    p = irgen.bmm_naive_ir(3, 520, 776, 264)
    ex = Executable(compile_graph(Graph.from_dict(p.graph), p.meta(), {"gemm_pair": True, **opts}))
    t_cpu = data.make_inputs(p)
    t = {k: v.cuda() for k, v in t_cpu.items()}
    t["C"].fill_(float("nan"))
    ex(t)
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    compare(t["C"].cpu(), t_cpu["A"].double() @ t_cpu["B"].double(), "f32", 1e-4, f"pair {opts}")
    ex.close()


@pytest.mark.gpu
def test_pair_gemm_random_shapes_against_float64():
    """Fifteen seeded random shapes (any M, N and K multiples of 8) through the default GEMM lowering."""
    import random
    from emmy_ptx_b200.runtime import Executable
    rng = random.Random(1202)
    for n in range(15):
        shape = (rng.randint(1, 3), rng.randint(1, 700), 8 * rng.randint(1, 90), 8 * rng.randint(1, 90))
        p = irgen.bmm_naive_ir(*shape)
        ex = Executable(compile_graph(Graph.from_dict(p.graph), p.meta()))
        assert ex.records[0]["kind"] == "tcgen05_gemm_pair"
        t_cpu = data.make_inputs(p)
        t = {k: v.cuda() for k, v in t_cpu.items()}
        t["C"].fill_(float("nan"))
        ex(t)
        torch.cuda.synchronize()
        assert ex.error_code() == 0, shape
        compare(t["C"].cpu(), t_cpu["A"].double() @ t_cpu["B"].double(), "f32", 1e-4, f"random pair {shape}")
        ex.close()
