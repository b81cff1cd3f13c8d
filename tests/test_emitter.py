"""The sm_100a emitter and the drop-in CLI — CPU only (ptxas cross-assembles without a GPU)."""
import json
import os
import re
import shutil
import subprocess
import sys
from pathlib import Path

import pytest

from emmy_ptx_b200 import irgen
from emmy_ptx_b200.compiler import compile_graph, compile_ir
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.codegen.module import parse_records

ROOT = Path(__file__).resolve().parents[1]
PTXAS = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"


def _compile(key, table=irgen.SMALL, **opts):
    p = table[key]()
    return p, compile_graph(Graph.from_dict(p.graph), p.meta(), opts)


def _assemble(ptx: str, tmp_path) -> str:
    if not os.path.exists(PTXAS):
        pytest.skip("ptxas not available")
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run([PTXAS, "-arch=sm_100a", "-v", str(f), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return r.stderr


@pytest.mark.parametrize("key", sorted(irgen.SMALL))
def test_small_configs_assemble_for_sm100a(key, tmp_path):
    _, mod = _compile(key)
    assert mod.ptx.startswith(".version 8.8\n.target sm_100a")
    info = _assemble(mod.ptx, tmp_path)
    assert "0 bytes spill" in info or "spill" not in info


@pytest.mark.parametrize("key", sorted(irgen.FULL))
def test_full_configs_assemble_for_sm100a(key, tmp_path):
    _, mod = _compile(key, irgen.FULL)
    _assemble(mod.ptx, tmp_path)


def test_fused_uses_packed_128bit_traffic_and_single_narrowing():
    _, mod = _compile("c3", irgen.FULL)
    ptx = mod.ptx
    assert len(re.findall(r"ld\.global\.nc\.v4\.b32", ptx)) == 3        # a, b, d: 8 x bf16 each
    assert "ld.global.nc.v4.f32" in ptx                                 # c: 4 x f32
    assert len(re.findall(r"cvt\.rn\.bf16x2\.f32", ptx)) == 4           # one narrowing per pair
    assert "st.global.v4.b32" in ptx
    assert "ld.global.b16" not in ptx and "div" not in ptx              # no scalar 16-bit, no index div


def test_block_softmax_reductions_use_redux_and_one_smem_pass():
    block = {"b": lambda: irgen.softmax_ir(4096, 1024, schedule="block")}
    _, mod = _compile("b", block)
    ptx = mod.ptx
    assert "redux.sync.max.f32" in ptx
    assert ptx.count("bar.sync") == 2                                    # the IR's two Syncs, no tree barriers
    _, ref = _compile("b", block, tree_barriers=True)
    assert ref.ptx.count("bar.sync") == 2 + 2 * 3                        # log2(8 warps) per TreeHalve


def test_warp_softmax_keeps_eight_loads_in_flight_without_barriers():
    p, mod = _compile("c1", irgen.FULL)
    ptx = mod.ptx
    assert p.params["schedule"] == "warp"
    assert ptx.count("ld.global.nc.v4.f32") == 8 and ptx.count("st.global.v4.f32") == 8
    assert "bar.sync" not in ptx and "redux.sync.max.f32" in ptx


def test_sum_kernel_unrolls_grid_stride_loads():
    _, mod = _compile("c2", irgen.FULL)
    assert len(re.findall(r"ld\.global\.nc\.v4\.f32", mod.ptx)) == 5      # 4 unrolled + remainder
    assert "red.global.add.f32" in mod.ptx
    _, modi = _compile("c2i", irgen.FULL)
    assert "red.global.add.s32" in modi.ptx and "redux.sync.add.s32" in modi.ptx


def test_launch_record_round_trips_through_the_ptx_text():
    p, mod = _compile("c2")
    (rec,) = parse_records(mod.ptx)
    assert rec["entry"] == p.entry and rec["params"] == p.arg_order
    assert rec["grid"] == [p.grid, 1, 1] and rec["block"] == [p.block, 1, 1]
    assert rec["zero_outputs"] == ["out"]
    assert ".reqntid 256, 1, 1" in mod.ptx


def test_multi_kernel_module_namespaces_shared_symbols():
    a, b = irgen.SMALL["c1b"](), irgen.SMALL["c2"]()
    g = dict(a.graph)
    g["nodes"] = {**a.graph["nodes"], **{k: v for k, v in b.graph["nodes"].items()}}
    mod = compile_graph(Graph.from_dict(g), None)
    assert "row_softmax__red_m" in mod.ptx and "array_sum_f32__red" in mod.ptx
    assert len(mod.kernels) == 2


def _write_problem(tmp_path, key):
    p = irgen.SMALL[key]()
    ir = tmp_path / f"{p.entry}.ir.json"
    ir.write_text(json.dumps(p.graph))
    (tmp_path / "meta.json").write_text(json.dumps(p.meta()))
    return p, ir


def test_cli_writes_ascii_ptx_and_reads_meta(tmp_path):
    p, ir = _write_problem(tmp_path, "c3")
    r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(ir)], capture_output=True)
    assert r.returncode == 0, r.stderr
    text = r.stdout.decode("ascii")
    assert ".visible .entry fused_relu_exp(" in text and ".reqntid 256" in text
    r2 = subprocess.run([sys.executable, "-m", "emmy_ptx", str(ir)], capture_output=True, cwd=str(ROOT))
    assert r2.returncode == 0 and r2.stdout == r.stdout


def test_cli_usage_and_errors(tmp_path):
    r = subprocess.run([sys.executable, str(ROOT / "compile.py")], capture_output=True, text=True)
    assert r.returncode == 1 and "usage" in r.stderr
    empty = tmp_path / "e.ir.json"
    empty.write_text(json.dumps({"nodes": {}, "inputs": [], "outputs": []}))
    r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(empty)], capture_output=True, text=True)
    assert r.returncode == 1 and "no KernelOp" in r.stderr
    bad = irgen.SMALL["c4"]()
    tile_body = bad.graph["nodes"]["bmm_bf16"]["op_fields"]["body"][2]["body"]
    next(st for st in tile_body if st["kind"] == "CpAsyncCopy")["swizzle"] = "SW128"
    f = tmp_path / "bad.ir.json"
    f.write_text(json.dumps(bad.graph))
    r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(f)], capture_output=True, text=True,
                       env=dict(os.environ, EMMY_B200_PATTERNS="0"))
    assert r.returncode == 1 and "swizzle" in r.stderr


def test_python_module_api_returns_ptx():
    import emmy_ptx
    p = irgen.SMALL["c1b"]()
    text = emmy_ptx.compile_ir(p.graph, p.meta())
    assert text.startswith(".version") and "row_softmax" in text


def test_vector_width_falls_back_when_alignment_is_unprovable():
    """A 4-wide f32 load at an odd element offset cannot be one 16-byte access."""
    from emmy_ptx_b200.irgen import Tile, Axis, Load, Write, Bin, V, TensorSpec, _graph
    body = [Tile([Axis("g", 64)], [
        Load(["a", "b", "c", "d"], "x", [Bin("+", Bin("*", V("g"), 4), 1)], "f32"),
        Write("y", ["a", "b", "c", "d"], [Bin("*", V("g"), 4)], "f32"),
    ])]
    args = [TensorSpec("x", (260,), "f32"), TensorSpec("y", (256,), "f32", output=True)]
    meta = {"kernels": [{"entry": "k", "grid": [1, 1, 1], "block": [64, 1, 1]}]}
    mod = compile_graph(Graph.from_dict(_graph("k", args, body)), meta)
    assert "ld.global.nc.v4" not in mod.ptx and "ld.global.nc.v2.f32" in mod.ptx
    assert "st.global.v4.f32" in mod.ptx


def test_programmatic_dependent_launch_is_opt_in_and_waits_before_memory():
    p = irgen.SMALL["c3"]()
    plain = compile_graph(Graph.from_dict(p.graph), p.meta())
    assert "griddepcontrol" not in plain.ptx and not plain.kernels[0].get("pdl")
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"pdl": True})
    assert mod.kernels[0]["pdl"] is True
    body = mod.ptx.split("griddepcontrol.wait;", 1)
    assert len(body) == 2 and "ld.global" not in body[0] and "st.global" not in body[0]
    assert "griddepcontrol.launch_dependents;" in body[1]


def test_attention_cubic_exp2_meets_its_error_bound():
    """The FMA-pipe 2^x of the attention softmax (range reduction by the 1.5*2^23 rounding trick, a
    cubic on [-1/2, 1/2], exponent added as an integer), evaluated with f32 / i32 arithmetic."""
    import numpy as np
    from emmy_ptx_b200.kernels import tc_attention as T
    c = [np.frombuffer(bytes.fromhex(h[2:])[::-1], dtype=np.float32)[0] for h in T.EXP2_C]
    f = np.linspace(-0.5, 0.5, 200001).astype(np.float32)
    r = c[3] * f + c[2]
    r = (r * f + c[1]).astype(np.float32)
    r = (r * f + c[0]).astype(np.float32)
    assert np.max(np.abs(r.astype(np.float64) / 2.0 ** f.astype(np.float64) - 1)) < 7.8e-5
    x = np.linspace(-119.9, 8.0, 400001).astype(np.float32)
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    j = (t - magic).astype(np.float32)
    fr = (x - j).astype(np.float32)
    r = (c[3] * fr + c[2]).astype(np.float32)
    r = (r * fr + c[1]).astype(np.float32)
    r = (r * fr + c[0]).astype(np.float32)
    bits = r.view(np.int32) + (t.view(np.int32) << 23)
    p = bits.view(np.float32).astype(np.float64)
    assert np.max(np.abs(p / 2.0 ** x.astype(np.float64) - 1)) < 8e-5


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("precise,half", [(True, True), (True, False), (False, False)])
def test_attention_variants_only_use_initialised_barriers(causal, precise, half):
    """Every mbarrier the attention kernel waits on or arrives at is one it initialises, and the
    launch geometry matches the warp roles of the variant (a variant that waited on a barrier nobody
    arrives at would stall until its bounded waits ran out)."""
    import math
    import re
    from emmy_ptx_b200.codegen.ptxcheck import undefined_uses
    from emmy_ptx_b200.kernels import tc_attention as T
    e = T.attention_entry("k", 2, 4, 1024, causal, 1 / math.sqrt(128), precise=precise, half=half)
    body = "\n".join(e["raw_entry"])
    base = re.search(r"add\.u32 (%r\d+), %r\d+, " + str(T.TILES * T.Q_BYTES + T.STAGES * T.KV_BYTES) + ";", body).group(1)
    inited = {int(m) for m in re.findall(r"mbarrier\.init\.shared::cta\.b64 \[" + re.escape(base) + r"\+(\d+)\]", body)}
    used = {int(m) for m in re.findall(r"mbarrier\.(?:try_wait\.parity|arrive)[^\[]*\[" + re.escape(base) + r"\+(\d+)\]", body)}
    used |= {int(m) for m in re.findall(r"tcgen05\.commit[^\[]*\[" + re.escape(base) + r"\+(\d+)\]", body)}
    assert used and used <= inited, sorted(used - inited)
    assert e["block"][0] == 384
    assert undefined_uses(".version 8.8\n.target sm_100a\n.address_size 64\n" + body) == []
