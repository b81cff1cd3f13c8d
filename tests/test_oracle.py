"""The CPU oracle, pinned against the committed golden vectors and the source expressions."""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from emmy_ptx_b200 import irgen, data
from oracle.run import oracle_outputs
from oracle import torch_ref
from oracle.interp import f32_to_bf16_bits, bf16_bits_to_f32
from tests.checks import compare, rtol_for
from tests.golden.make_golden import ir_hash, input_digest

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())


@pytest.mark.parametrize("key", sorted(irgen.SMALL))
def test_golden_fixture_matches_current_ir_and_inputs(key):
    p = irgen.SMALL[key]()
    rec = MANIFEST[key]
    assert rec["ir"] == ir_hash(p.graph, p.meta()), "IR changed: regenerate tests/golden (make_golden.py)"
    assert rec["inputs"] == input_digest(data.make_inputs(p)), "seeded inputs changed"
    assert (GOLDEN / "ref_ptx" / f"{key}.ptx").read_text().startswith(".version")


@pytest.mark.parametrize("key", sorted(irgen.SMALL))
def test_oracle_matches_golden_vectors(key):
    p = irgen.SMALL[key]()
    t = data.make_inputs(p)
    got = oracle_outputs(p, t)
    vec = np.load(GOLDEN / "vectors" / f"{key}.npz")
    for a in p.outputs:
        ref = torch.from_numpy(vec[a.name])
        compare(got[a.name], ref, a.dtype if a.dtype != "i32" else "i32", rtol_for(p), f"{key}.{a.name}")


def test_golden_vectors_are_the_source_expressions():
    """The committed vectors are what torch computes for the source expressions today."""
    for key in ("c1b", "c2i", "c3"):
        p = irgen.SMALL[key]()
        t = data.make_inputs(p)
        ref = torch_ref.reference(p, t)
        vec = np.load(GOLDEN / "vectors" / f"{key}.npz")
        for name, v in ref.items():
            assert np.allclose(vec[name], v.double().numpy(), rtol=1e-12, atol=0)


def test_bf16_rounding_is_round_to_nearest_even():
    x = torch.randn(10000) * 100
    ours = bf16_bits_to_f32(f32_to_bf16_bits(x.numpy()))
    assert np.array_equal(ours, x.to(torch.bfloat16).float().numpy())


def test_oracle_accum_seeding_follows_emission_order():
    """An accumulator bound before a loop is not re-seeded by it (compile.py:1299-1300)."""
    from emmy_ptx_b200.irgen import (Tile, Axis, Init, StridedLoop, Accum, Write, Lit, V, TensorSpec, _graph)
    from emmy_ptx_b200.ir import Graph
    from oracle.interp import Interpreter
    body = [Tile([Axis("g", 32)], [
        Init("acc", "f32", 5.0),
        StridedLoop("i", 4, 0, 1, [Accum("acc", "add", Lit(1.0))], end=4),
        StridedLoop("j", 4, 0, 1, [Accum("acc2", "add", Lit(2.0))], end=4),
        Write("o", ["acc", "acc2"], [Bin_("g")], "f32"),
    ])]
    args = [TensorSpec("o", (64,), "f32", output=True)]
    g = Graph.from_dict(_graph("k", args, body))
    bufs = {"o": np.zeros(64, np.float32)}
    Interpreter(g).run(bufs, 1, 32)
    assert bufs["o"][0] == 9.0 and bufs["o"][1] == 8.0


def Bin_(name):
    from emmy_ptx_b200.irgen import Bin, V
    return Bin("*", V(name), 2)


def test_oracle_sample_of_blocks_is_partial():
    p = irgen.SMALL["c2i"]()
    t = data.make_inputs(p)
    full = oracle_outputs(p, t)["out"]
    half = oracle_outputs(p, t, blocks=range(p.grid // 2))["out"]
    assert int(half) != int(full)
