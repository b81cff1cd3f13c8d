"""IR ``CpAsyncCopy`` stripes promoted to TMA tile loads on the CUDA-core path.

The CUDA-core batched matmul stages 64 x 32 and 32 x 64 operand stripes with one 16-byte ``cp.async``
per thread; its lanes together copy one dense box each, so the emitter issues each stripe as one
``cp.async.bulk.tensor`` from thread 0 with an mbarrier per commit group.  These tests check the
promotion decision, the emitted instructions, the results in the tensor-core emulator (also with
TMA completions held back until a thread waits, which exposes a missing or early wait) and that a
copy whose lanes do not form a box keeps ``cp.async``.
"""
import copy

import numpy as np
import pytest
import torch

from emmy_ptx_b200 import data, irgen
from emmy_ptx_b200.codegen import tma_stripes
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph, dt_name
from oracle.run import oracle_outputs
from tests.checks import compare
from tests.ptxemu import Memory
from tests.tcemu import TcEmulator


def _compile(p, **opts):
    return compile_graph(Graph.from_dict(p.graph), p.meta(), {"patterns": False, **opts})


def test_bmm_stripes_become_tma_loads():
    p = irgen.bmm_ir(2, 128, 128, 96)
    mod = _compile(p)
    rec = mod.kernels[0]
    assert [t["tensor"] for t in rec["tmaps"]] == ["A", "B"]          # one descriptor per source box
    assert rec["tmaps"][0]["box"] == [32, 64, 1] and rec["tmaps"][1]["box"] == [64, 32, 1]
    assert all(t["swizzle"] == "none" for t in rec["tmaps"])
    assert rec["extra"] == [{"kind": "errword", "name": "__err"}]
    assert "cp.async.bulk.tensor.3d" in mod.ptx and "mbarrier.try_wait.parity" in mod.ptx
    assert "cp.async.cg" not in mod.ptx and "cp.async.wait_group" not in mod.ptx
    assert "multicast" not in mod.ptx
    off = _compile(p, tma_stripes=False)
    assert "cp.async.cg" in off.ptx and "cp.async.bulk" not in off.ptx and "tmaps" not in off.kernels[0]


def _run(p, mod, defer=False):
    t = data.make_inputs(p)
    mem = Memory()
    addr = {}
    for a in p.args:
        arr = (t[a.name].view(torch.int16).numpy() if t[a.name].dtype == torch.bfloat16 else t[a.name].numpy()).copy()
        if a.output:
            arr.view(np.uint8)[...] = 0x7F
        addr[a.name] = mem.alloc(arr)
    rec = mod.kernels[0]
    tm = {f"p_{s['name']}": (addr[s["tensor"]], s) for s in rec["tmaps"]}
    emu = TcEmulator(mod.ptx, rec["entry"], tm, defer=defer)
    args = {f"p_{n}": addr[n] for n in rec["params"]}
    args.update(emu.tmap_args())
    err = mem.alloc(np.zeros(16, np.uint8))
    args["p_err"] = err
    emu.run(rec["grid"][0], rec["block"][0], args, mem, rec.get("dyn_smem", 0))
    got = torch.from_numpy(mem.array(addr["C"], np.float32, tuple(t["C"].shape)).copy())
    return t, got, int(mem.array(err, np.int32, (4,))[0])


@pytest.mark.parametrize("defer", [False, True])
def test_promoted_bmm_matches_oracle(defer):
    p = irgen.bmm_ir(1, 64, 128, 96)
    t, got, code = _run(p, _compile(p), defer)
    assert code == 0
    compare(got, oracle_outputs(p, t)["C"], "f32", 1e-4, f"tma stripes defer={defer}")


def test_a_copy_that_is_not_one_box_keeps_cp_async():
    # lane rows and columns swapped in A's copies: the lanes no longer tile a dense 64 x 32 box, so
    # every copy of the kernel stays cp.async (and the kernel still computes what its IR says)
    p = irgen.bmm_ir(1, 64, 64, 64)
    d = copy.deepcopy(p.graph)

    def edit(stmts):
        for st in stmts:
            if st.get("kind") == "CpAsyncCopy" and st["src"] == "A":
                st["lane_index"] = [st["lane_index"][1], st["lane_index"][0]]
            for key in ("body", "else_body"):
                if isinstance(st.get(key), list):
                    edit(st[key])
    edit(d["nodes"]["bmm_bf16"]["op_fields"]["body"])
    smem = {"sA": ((2, 64, 32), "bf16", 16), "sB": ((2, 32, 64), "bf16", 16)}

    def plan_of(graph_dict):
        g_ = Graph.from_dict(graph_dict)
        node = g_.kernels()[0]
        shapes = {v.name: tuple(int(x) for x in v.shape) for nd in g_.nodes.values() for v in nd.outputs}
        dtypes = {v.name: dt_name(v.dtype) for nd in g_.nodes.values() for v in nd.outputs}
        return tma_stripes.plan(node.op.body, p.block, shapes, dtypes, smem)
    assert plan_of(p.graph) is not None
    assert plan_of(d) is None
    g = Graph.from_dict(d)
    mod = compile_graph(g, p.meta(), {"patterns": False})
    assert "cp.async.cg" in mod.ptx and "cp.async.bulk" not in mod.ptx


def test_full_size_cuda_core_bmm_is_promoted():
    p = irgen.FULL["c4"]()
    rec = _compile(p).kernels[0]
    assert rec["kind"] == "generic" and [t["tensor"] for t in rec["tmaps"]] == ["A", "B"]
