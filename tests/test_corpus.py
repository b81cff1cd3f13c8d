"""The coverage corpus on CPU: fixtures current, oracle against the source expressions, every kernel
assembles for sm_100a, and the corpus plus the benchmark IRs together use every IR construct."""
import json
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

from emmy_ptx_b200 import corpus, irgen, data, ir
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from oracle.run import oracle_outputs
from oracle import torch_ref
from tests.checks import compare
from tests.golden.make_golden import ir_hash, input_digest

GOLDEN = Path(__file__).resolve().parent / "golden"
MANIFEST = json.loads((GOLDEN / "manifest.json").read_text())
PTXAS = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
KEYS = sorted(corpus.CORPUS)


def _src_compare(got, ref, a, what):
    """Oracle against the float64 source expression: f32 evaluation error, so a relative 1e-4 of
    max(|ref|, rms) for f32 / f64, one unit of the 16-bit type for f16 / bf16, exact for integers."""
    compare(got, ref, a.dtype, 1e-4, what)


@pytest.mark.parametrize("key", KEYS)
def test_corpus_fixture_is_current(key):
    p = corpus.CORPUS[key]()
    rec = MANIFEST[key]
    assert rec["ir"] == ir_hash(p.graph, p.meta()), "IR changed: regenerate tests/golden (make_golden.py)"
    assert rec["inputs"] == input_digest(data.make_inputs(p))
    has_ptx = (GOLDEN / "ref_ptx" / f"{key}.ptx").exists()
    assert has_ptx == ("ref_error" not in rec and "ref_unsafe" not in rec)


@pytest.mark.parametrize("key", KEYS)
def test_corpus_oracle_matches_source_expression(key):
    p = corpus.CORPUS[key]()
    t = data.make_inputs(p)
    got = oracle_outputs(p, t)
    vec = np.load(GOLDEN / "vectors" / f"{key}.npz")
    for a in p.outputs:
        ref = torch.from_numpy(vec[a.name]).reshape(a.shape)
        _src_compare(got[a.name], ref, a, f"{key}.{a.name}")


@pytest.mark.parametrize("key", KEYS)
def test_corpus_vectors_are_todays_source_expressions(key):
    p = corpus.CORPUS[key]()
    ref = torch_ref.reference(p, data.make_inputs(p))
    vec = np.load(GOLDEN / "vectors" / f"{key}.npz")
    for name, v in ref.items():
        assert np.array_equal(vec[name], v.double().numpy(), equal_nan=True)


@pytest.mark.parametrize("key", KEYS)
def test_corpus_assembles_for_sm100a(key, tmp_path):
    if not Path(PTXAS).exists():
        pytest.skip("ptxas not available")
    p = corpus.CORPUS[key]()
    mod = compile_graph(Graph.from_dict(p.graph), p.meta())
    src = tmp_path / f"{key}.ptx"
    src.write_text(mod.ptx)
    r = subprocess.run([PTXAS, "-arch=sm_100a", str(src), "-o", str(tmp_path / "k.cubin")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    # a tensor-core attention adds its value pre-pass launch before the kernel's own entry
    entries = [rec["entry"] for rec in mod.kernels if rec.get("kind") != "value_prepass"]
    want = [ln[0] for ln in getattr(p, "launches", [])] or [p.entry]
    assert entries == want


def test_reference_cond_else_ptx_is_not_kept():
    """The reference's PTX for a Cond with an else branch stores through an address register that
    only the then-branch computes (its expression cache is not cleared between the two bodies,
    compile.py:1480-1496); on a B200 that raised an illegal address.  The fixture is withheld."""
    rec = MANIFEST["k_cond"]
    assert "%rd4 read before any write" in rec["ref_unsafe"]
    assert not (GOLDEN / "ref_ptx" / "k_cond.ptx").exists()


def test_reference_predicate_store_is_recorded():
    """The reference stores a predicate register straight to a byte (``st.global.u8 [..], %p``),
    which ptxas rejects; this backend selects 0/1 first."""
    assert "ptxas" in MANIFEST["k_mask"]["ref_error"]


def test_every_kept_reference_fixture_assembles_for_sm100a(tmp_path):
    if not Path(PTXAS).exists():
        pytest.skip("ptxas not available")
    for path in sorted((GOLDEN / "ref_ptx").glob("*.ptx")):
        r = subprocess.run([PTXAS, "-arch=sm_100a", str(path), "-o", str(tmp_path / "k.cubin")],
                           capture_output=True, text=True)
        assert r.returncode == 0, (path.name, r.stderr)


def test_reference_hypot_failure_is_recorded():
    """The reference emitter cannot build ``hypot`` (a two-operand helper given one operand); this
    backend builds it and the source expression pins it."""
    assert "TypeError" in MANIFEST["k_hypot"]["ref_error"]


def _walk(obj, kinds, ops, dtypes):
    if isinstance(obj, dict):
        k = obj.get("kind")
        if k:
            kinds.add(k)
            if k == "Assign":
                ops.add(obj["op"]["name"])
            if k in ("Load", "Write"):
                dtypes.add(obj.get("dtype") or obj.get("value_dtype"))
            if k == "WarpShuffle" and obj.get("prefix"):
                kinds.add("WarpShuffle(prefix)")
            if k == "Cond" and obj.get("else_body"):
                kinds.add("Cond(else)")
            if k == "Select" and len(obj["branches"]) > 2:
                kinds.add("Select(3+)")
            if k == "Write" and obj.get("atomic"):
                kinds.add("Write(atomic)")
        for v in obj.values():
            _walk(v, kinds, ops, dtypes)
    elif isinstance(obj, list):
        for v in obj:
            _walk(v, kinds, ops, dtypes)


def test_corpus_and_benchmarks_cover_every_construct():
    kinds, ops, dtypes = set(), set(), set()
    multi = 0
    for mk in {**irgen.SMALL, **corpus.CORPUS}.values():
        p = mk()
        _walk(p.graph, kinds, ops, dtypes)
        multi += len(Graph.from_dict(p.graph).kernels()) > 1
    missing = (set(ir.STATEMENTS) | set(ir.EXPRESSIONS)) - kinds
    assert not missing, f"no test IR uses {sorted(missing)}"
    for extra in ("WarpShuffle(prefix)", "Cond(else)", "Select(3+)", "Write(atomic)"):
        assert extra in kinds
    assert {"f32", "f16", "bf16", "f64", "i32", "u8"} <= dtypes
    assert multi >= 2
    assert {"exp", "log", "tanh", "erf", "gelu", "gelu_tanh", "sigmoid", "bitwise_and", "left_shift",
            "where", "logical_and", "logical_not", "greater"} <= ops
