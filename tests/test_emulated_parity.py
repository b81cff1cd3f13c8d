"""CPU parity of the emitted PTX itself: this backend's CUDA-core kernels and the reference emitter's
PTX for the same IR, run by the SIMT emulator (:mod:`tests.ptxemu`), against the oracle.

The GPU tests run the same comparisons on a B200; these run everywhere, on the small configurations
and the coverage corpus, so an emitter change is checked before any GPU time.  Outputs start filled
with a 0x7F byte pattern, so an element a kernel fails to write shows up as a mismatch.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from emmy_ptx_b200 import corpus, data, irgen
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from oracle.run import oracle_outputs
from tests.checks import atol_for, compare, rms_floor_for, rtol_for
from tests.ptxemu import Emulator, Memory
from tests.tcemu import TcEmulator

GOLDEN = Path(__file__).resolve().parent / "golden"
SMALL_KEYS = ["c1", "c1b", "c1w", "c2", "c2i", "c2odd", "c3"]
CORPUS_KEYS = sorted(corpus.CORPUS)
# corpus kernels whose extra CUDA-core forms (this emitter's plain form, the reference emitter's PTX)
# take the better part of a minute or more each in the scalar emulator: the GPU corpus tests run those
# forms against the oracle, and the default form of each still runs here (the tensor-core form for
# k_sdpa_big), so the CPU suite stays a few minutes long
HEAVY_CUDA_CORE = {"k_sdpa_big", "k_sdpa_causal", "k_sdpa_scale", "k_sdpa_causal2"}


def _np(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()


def _setup(p):
    t = data.make_inputs(p)
    mem = Memory()
    addr = {}
    for a in p.args:
        arr = _np(t[a.name]).copy()
        if a.output:
            arr.view(np.uint8)[...] = 0x7F
        addr[a.name] = mem.alloc(arr)
    return t, mem, addr


def _outputs(p, t, mem, addr):
    out = {}
    for a in p.outputs:
        ref = t[a.name]
        arr = mem.array(addr[a.name], _np(ref).dtype, tuple(ref.shape)).copy()
        g = torch.from_numpy(arr)
        out[a.name] = g.view(torch.bfloat16) if ref.dtype == torch.bfloat16 else g
    return out


def _zero(mem, addr, names):
    for n in names:
        mem.array(addr[n], np.uint8, (-1,))[:] = 0


def _run_ours(p, opts=None):
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), opts or {})
    assert all(r["kind"] == "generic" for r in mod.kernels)
    t, mem, addr = _setup(p)
    for rec in mod.kernels:
        _zero(mem, addr, rec.get("zero_outputs", []))
        args = {f"p_{n}": addr[n] for n in rec["params"]}
        if rec.get("tmaps"):
            # CpAsyncCopy stripes promoted to TMA: the tensor-core emulator runs the TMA loads and
            # the commit groups' mbarriers
            tm = {f"p_{spec['name']}": (addr[spec["tensor"]], spec) for spec in rec["tmaps"]}
            emu = TcEmulator(mod.ptx, rec["entry"], tm)
            args.update(emu.tmap_args())
            err = mem.alloc(np.zeros(16, np.uint8))
            args["p_err"] = err
            emu.run(rec["grid"][0], rec["block"][0], args, mem, rec.get("dyn_smem", 0))
            assert int(mem.array(err, np.int32, (4,))[0]) == 0, "a commit group's wait timed out"
        else:
            Emulator(mod.ptx, rec["entry"]).run(rec["grid"][0], rec["block"][0], args, mem, rec.get("dyn_smem", 0))
    return t, _outputs(p, t, mem, addr)


def _run_reference(p, ptx):
    t, mem, addr = _setup(p)
    launches = getattr(p, "launches", None) or [(p.entry, p.grid, p.block, p.zero_outputs, p.arg_order)]
    for entry, grid, block, zero, order in launches:
        _zero(mem, addr, zero)
        Emulator(ptx, entry).run(grid, block, {f"p_{n}": addr[n] for n in order}, mem, p.smem_bytes or 0)
    return t, _outputs(p, t, mem, addr)


def _check(p, t, got, tag):
    want = oracle_outputs(p, t)
    for a in p.outputs:
        compare(got[a.name], want[a.name], a.dtype, rtol_for(p), f"{tag}.{a.name}",
                rms_floor=rms_floor_for(p), atol=atol_for(p))


def _problem(key):
    return irgen.SMALL[key]() if key in irgen.SMALL else corpus.CORPUS[key]()


def _tensor_core(p) -> bool:
    return any(r["kind"] != "generic" for r in compile_graph(Graph.from_dict(p.graph), p.meta()).kernels)


@pytest.mark.parametrize("key", SMALL_KEYS + CORPUS_KEYS)
def test_emitted_ptx_matches_oracle(key):
    p = _problem(key)
    if _tensor_core(p):
        # a corpus kernel the tensor-core lowering takes runs in the tensor-core emulator
        from tests.test_tc_emulated import run_emulated
        t = data.make_inputs(p)
        got, code, _ = run_emulated(p, t, {})
        assert code == 0
        _check(p, t, got, f"tc-emu:{key}")
        return
    t, got = _run_ours(p)
    _check(p, t, got, f"emu:{key}")


@pytest.mark.parametrize("key", CORPUS_KEYS)
def test_emitted_ptx_without_shortcuts_matches_oracle(key):
    # per-level tree barriers, no redux, no unrolling: the CUDA-core emitter's plain forms
    if key in HEAVY_CUDA_CORE:
        pytest.skip("this form runs in the GPU corpus tests (minutes in the scalar emulator)")
    p = _problem(key)
    opts = {"tree_barriers": True, "no_redux": True, "no_unroll": True}
    if _tensor_core(p):
        opts["patterns"] = False             # the CUDA-core form of a tensor-core corpus kernel
    t, got = _run_ours(p, opts)
    _check(p, t, got, f"emu-plain:{key}")


@pytest.mark.parametrize("key", SMALL_KEYS + CORPUS_KEYS)
def test_reference_emitter_ptx_matches_oracle(key):
    path = GOLDEN / "ref_ptx" / f"{key}.ptx"
    if not path.exists():
        pytest.skip("the reference emitter rejects this IR or its PTX fails the def-use check")
    if key in HEAVY_CUDA_CORE:
        pytest.skip("the reference PTX of this case runs in the GPU corpus tests (minutes in the scalar emulator)")
    p = _problem(key)
    t, got = _run_reference(p, path.read_text())
    _check(p, t, got, f"emu-ref:{key}")


def test_small_cuda_core_bmm_and_attention():
    # the CUDA-core forms of configs 4 and 5 (tensor-core lowering off), at sizes the emulator runs
    # in seconds: cp.async double buffering, the online-softmax Accum nest with its causal Select
    for p in (irgen.bmm_ir(1, 64, 64, 64), irgen.attention_ir(1, 1, 32, 32, True)):
        mod_opts = {"patterns": False}
        t, got = _run_ours(p, mod_opts)
        _check(p, t, got, f"emu:{p.name}")


def test_attention_the_tensor_core_lowering_declines():
    # head dim 256 has no tensor-core form (32, 64 and 128 do): the attention pattern declines it, so
    # the CUDA-core form runs (every record generic)
    p = irgen.attention_ir(1, 1, 16, 256, True)
    t, got = _run_ours(p)
    _check(p, t, got, f"emu:{p.name}")


@pytest.mark.parametrize("build,shape", [(corpus.col_sum, (0, 96)), (corpus.mid_sum, (2, 0, 32)),
                                         (corpus.rmsnorm, (0, 512))], ids=["colsum-0rows", "midsum-0mid", "rmsnorm-0rows"])
def test_empty_extents(build, shape):
    # a reduction over an empty axis leaves its identity (0 for a sum, as torch's sum of nothing);
    # a tile with no rows writes nothing
    p = build(*shape)
    t, got = _run_ours(p)
    _check(p, t, got, f"emu:{p.name}")
    for a in p.outputs:
        assert not got[a.name].numel() or not got[a.name].any()


@pytest.mark.parametrize("key", ["c1", "c1w", "k_logsoftmax", "k_mathzoo"])
def test_fast_math_options_match_oracle(key, tmp_path):
    # opt-in approx_ftz (ex2/lg2 flush subnormals) and fast_div (div.full, 2 ulp): within the
    # tolerances on normal data; the PTX must still assemble
    import shutil
    import subprocess
    p = _problem(key)
    opts = {"approx_ftz": True, "fast_div": True}
    t, got = _run_ours(p, opts)
    _check(p, t, got, f"emu-fast:{key}")
    ptx = compile_graph(Graph.from_dict(p.graph), p.meta(), opts).ptx
    assert "ex2.approx.ftz.f32" in ptx or "lg2.approx.ftz.f32" in ptx
    src = tmp_path / "k.ptx"
    src.write_text(ptx)
    ptxas = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
    r = subprocess.run([ptxas, "-arch=sm_100a", str(src), "-o", str(tmp_path / "k.cubin")], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr


def test_softmax_with_one_division_per_row():
    # the warp-per-row softmax with y = e * (1 / s): one IEEE division per row instead of per element
    p = irgen.softmax_ir(64, 1024, "warp", recip=True)
    t, got = _run_ours(p)
    _check(p, t, got, "emu:softmax-recip")
