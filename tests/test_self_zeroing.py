"""Self-zeroing accumulators (compile option ``self_zeroing``).

An output that a kernel only accumulates into with atomic adds (listed in ``zero_outputs``) normally
needs a memset before every launch.  With the option the adds go to a scratch the runtime zeroes once;
the block that finishes last (a ticket in the scratch picks it) takes each accumulator with an atomic
exchange against 0 and stores it to the output, so the output needs no zeroing and the scratch is zero
again for the next launch.  The CPU tests run the emitted PTX in the SIMT emulator, launch after launch,
with the output filled with garbage before each; the GPU test does the same through the runtime.
"""
import numpy as np
import pytest
import torch

from emmy_ptx_b200 import corpus, data, irgen
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from tests.ptxemu import Emulator, Memory


def _compile(p, opts):
    return compile_graph(Graph.from_dict(p.graph), p.meta(), opts)


@pytest.mark.parametrize("dtype", ["f32", "i32"])
def test_sum_without_zeroing_launch_after_launch(dtype):
    p = irgen.sum_ir(1 << 12, dtype, blocks=5, threads=128)
    mod = _compile(p, {"self_zeroing": True})
    rec = mod.kernels[0]
    assert rec["zero_outputs"] == [] and rec["self_zeroing"] == ["out"]
    acc_spec = rec["scratch"][0]
    assert acc_spec["zeroed"] and rec["extra"] == [{"name": acc_spec["name"], "kind": "buffer", "param": "p_acc"}]
    t = data.make_inputs(p)
    npdt = np.float32 if dtype == "f32" else np.int32
    mem = Memory()
    x = mem.alloc(t["x"].numpy().copy())
    acc = mem.alloc(np.zeros(acc_spec["shape"][0], np.int32))
    want = t["x"].double().sum().item() if dtype == "f32" else int(t["x"].long().sum().item())
    for _ in range(3):
        out = mem.alloc(np.full(1, 0x7F7F7F7F, np.uint32).view(npdt))
        Emulator(mod.ptx, rec["entry"]).run(rec["grid"][0], rec["block"][0], {"p_x": x, "p_out": out, "p_acc": acc},
                                            mem, rec.get("dyn_smem", 0))
        got = mem.array(out, npdt, (1,))[0]
        if dtype == "i32":
            assert int(got) == want
        else:
            assert abs(float(got) - want) <= 1e-5 * abs(want)
        assert not mem.array(acc, np.int32, (acc_spec["shape"][0],)).any()


def test_option_leaves_other_kernels_alone():
    # no zeroed output (softmax), or an output the kernel also reads or writes without an atomic:
    # the option changes nothing
    for p in (irgen.softmax_ir(8, 256), corpus.CORPUS["k_hist"](), corpus.CORPUS["k_rmsnorm"]()):
        plain = _compile(p, {})
        opt = _compile(p, {"self_zeroing": True})
        assert plain.ptx == opt.ptx
        assert all("self_zeroing" not in r for r in opt.kernels)


def test_default_compile_keeps_the_reference_abi():
    # without the option the sum keeps its plain parameters and its zeroed output
    p = irgen.sum_ir(1 << 12, "f32", blocks=5, threads=128)
    rec = _compile(p, {}).kernels[0]
    assert rec["zero_outputs"] == ["out"] and "extra" not in rec and "scratch" not in rec


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["f32", "i32"])
def test_sum_without_zeroing_on_the_gpu(dtype):
    from emmy_ptx_b200.runtime import Executable
    p = irgen.FULL["c2" if dtype == "f32" else "c2i"]()
    ex = Executable(_compile(p, {"self_zeroing": True}))
    t = {k: v.cuda() for k, v in data.make_inputs(p).items()}
    want = t["x"].double().sum().item() if dtype == "f32" else int(t["x"].long().sum().item())
    for _ in range(4):
        t["out"].view(torch.int32).fill_(0x7F7F7F7F)
        ex(t)
        torch.cuda.synchronize()
        got = t["out"].item()
        if dtype == "i32":
            assert got == want
        else:
            assert abs(got - want) <= 1e-5 * abs(want) + 1e-3
        acc = next(iter(ex.scratch.values()))
        assert not acc.any().item()
    ex.close()


def test_runtime_refuses_another_grid_for_a_ticket_kernel():
    # the last block is found by counting to the compiled grid: another launch grid would leave the
    # accumulators unread and unzeroed, so the runtime refuses it before touching the device
    from emmy_ptx_b200.runtime import Executable
    p = irgen.sum_ir(1 << 12, "f32", blocks=5, threads=128)
    rec = _compile(p, {"self_zeroing": True}).kernels[0]
    fake = Executable.__new__(Executable)
    fake.compiled = type("M", (), {"kernels": [rec]})()
    fake.scratch = {}
    fake.funcs = [None]
    with pytest.raises(ValueError, match="compiled grid"):
        fake.launch(0, {}, 0, grid=[4, 1, 1], zero=False)


def test_an_output_written_plainly_twice_is_left_alone():
    # two plain Writes of a zeroed output (and a Load of it) disqualify it without tripping the check
    from emmy_ptx_b200.irgen import TensorSpec, Tile, Axis, Load, Write, V, _graph, Problem
    args = [TensorSpec("x", (64,), "f32", ("normal", 1.0)), TensorSpec("y", (64,), "f32", output=True)]
    body = [Tile([Axis("i", 64)], [Load(["a"], "x", [V("i")], "f32"), Write("y", ["a"], [V("i")], "f32"),
                                   Write("y", ["a"], [V("i")], "f32")])]
    p = Problem("twice", "corpus", "twice", _graph("twice", args, body), args, grid=1, block=64,
                zero_outputs=["y"])
    rec = _compile(p, {"self_zeroing": True}).kernels[0]
    assert rec["zero_outputs"] == ["y"] and "self_zeroing" not in rec
