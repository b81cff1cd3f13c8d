"""IR contract (Graph.from_dict) and the symbolic integer machinery — CPU only."""
import json
import random

import pytest

from emmy_ptx_b200 import irgen
from emmy_ptx_b200.ir import Graph, IRError, load_graph
from emmy_ptx_b200.codegen.affine import Affine, reg_atom, div_const, rem_const, recombine


def test_graph_round_trip_keeps_class_names_and_fields():
    p = irgen.SMALL["c4"]()
    g = Graph.from_dict(p.graph)
    (k,) = g.kernels()
    assert type(k.op).__name__ == "KernelOp" and k.op.name == "bmm_bf16"
    tile = [s for s in k.op.body if type(s).__name__ == "Tile"][0]
    assert [a.name for a in tile.axes] == ["b", "tm", "tn", "t"]
    again = Graph.from_dict(json.loads(json.dumps(g.to_dict())))
    assert json.dumps(again.to_dict(), sort_keys=True) == json.dumps(g.to_dict(), sort_keys=True)


def test_optional_fields_get_reference_defaults():
    d = {"nodes": {"k": {"op": "KernelOp", "op_fields": {"name": "k", "body": [
        {"kind": "Sync"}, {"kind": "CpAsyncWait"},
        {"kind": "WarpShuffle", "state": ["a"]}]}, "inputs": [], "outputs": []}}}
    k = Graph.from_dict(d).kernels()[0]
    sync, wait, shf = k.op.body
    assert sync.warp is False and sync.barrier_id == 0 and sync.count is None
    assert wait.group == 0
    assert shf.length == 32 and shf.prefix is False


@pytest.mark.parametrize("bad", [
    {"nodes": {"k": {"op": "Bogus"}}},
    {"nodes": {"k": {"op": "KernelOp", "op_fields": {"name": "k", "body": [{"kind": "Load", "names": ["x"]}]}}}},
    {"nodes": {"k": {"op": "KernelOp", "op_fields": {"name": "k", "body": [{"kind": "NoSuchStmt"}]}}}},
])
def test_malformed_ir_is_refused(bad):
    with pytest.raises(IRError):
        Graph.from_dict(bad)


def test_load_graph_accepts_path(tmp_path):
    p = irgen.SMALL["c1"]()
    f = tmp_path / "k.ir.json"
    f.write_text(json.dumps(p.graph))
    assert load_graph(f).kernels()[0].op.name == "row_softmax"


def _trunc_div(a, b):
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def _eval(aff: Affine, env: dict) -> int:
    total = aff.c
    for atom, k in aff.terms.items():
        if atom.kind == "reg":
            v = env[atom.reg]
        elif atom.kind == "div":
            v = _trunc_div(_eval(atom.num, env), atom.d)
        else:
            n = _eval(atom.num, env)
            v = n - _trunc_div(n, atom.d) * atom.d
        total += k * v
    return total


def test_tile_decode_and_relinearise_cancels():
    """gid = 256*ctaid + tid decoded as (i: R, j8: C/8) and re-linearised as i*C + 8*j8 is 8*gid."""
    tid = Affine.of(reg_atom("%t", 0, 255))
    cta = Affine.of(reg_atom("%c", 0, 32767))
    gid = cta.scale(256) + tid
    i = div_const(gid, 1024)
    j8 = rem_const(gid, 1024)
    lin = recombine(i.scale(8192) + j8.scale(8))
    assert lin.key == (cta.scale(2048) + tid.scale(8)).key


@pytest.mark.parametrize("seed", range(20))
def test_div_rem_rewrites_are_exact(seed):
    rnd = random.Random(seed)
    T = rnd.choice([32, 64, 128, 256, 512])
    G = rnd.randint(1, 5000)
    tid = Affine.of(reg_atom("%t", 0, T - 1))
    cta = Affine.of(reg_atom("%c", 0, G - 1))
    k = Affine.of(reg_atom("%k", None, None))
    forms = [cta.scale(T) + tid, tid.scale(rnd.choice([1, 4, 8])) + rnd.randint(0, 64),
             cta.scale(rnd.choice([64, 1024, 4096])) + tid, k.scale(3) + tid - 7]
    for num in forms:
        for d in (1, 2, 3, 4, 8, 16, 24, 32, 256, 1000, 1024, 4096, 65536):
            q = div_const(num, d)
            r = rem_const(num, d)
            for _ in range(30):
                env = {"%t": rnd.randrange(T), "%c": rnd.randrange(G), "%k": rnd.randint(-10 ** 6, 10 ** 6)}
                n = _eval(num, env)
                assert _eval(q, env) == _trunc_div(n, d), (num, d, env)
                assert _eval(r, env) == n - _trunc_div(n, d) * d, (num, d, env)
                assert _eval(recombine(q.scale(d) + r), env) == n


def test_alignment_proof():
    tid = Affine.of(reg_atom("%t", 0, 255))
    assert tid.scale(8).scale(2).divisible_by(16)
    assert not (tid.scale(8) + 1).scale(2).divisible_by(16)
