"""GPU parity: this backend's kernels and the reference emitter's PTX against the CPU oracle.

Every launch goes through the C ABI (``libemmy_launch.so``).  Small configurations are compared
with the oracle interpreter element by element; the full benchmark sizes are checked against
float64 / fp32 references of the source expression (exact for the integer sum).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from emmy_ptx_b200 import irgen, data
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.runtime import Executable
from emmy_ptx_b200.launcher import Device
from oracle.run import oracle_outputs
from tests.checks import compare, rtol_for, rms_floor_for

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


def _run_ours(p, t_cpu, **opts):
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), opts)
    ex = Executable(mod)
    t = {k: v.cuda() for k, v in t_cpu.items()}
    ex(t)
    torch.cuda.synchronize()
    return {a.name: t[a.name].cpu() for a in p.outputs}, ex


@pytest.mark.parametrize("key", sorted(irgen.SMALL))
def test_small_config_matches_oracle(key):
    p = irgen.SMALL[key]()
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t)
    assert ex.error_code() == 0
    for a in p.outputs:
        compare(got[a.name], want[a.name], a.dtype, rtol_for(p), f"{key}.{a.name}", rms_floor=rms_floor_for(p))


@pytest.mark.parametrize("key", sorted(irgen.SMALL))
def test_cuda_core_path_matches_oracle(key):
    """The statement-at-a-time path alone (tensor-core patterns off, tree barriers on)."""
    p = irgen.SMALL[key]()
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, _ = _run_ours(p, t, patterns=False, tree_barriers=True, no_redux=True)
    for a in p.outputs:
        compare(got[a.name], want[a.name], a.dtype, rtol_for(p), f"{key}.{a.name}")


@pytest.mark.parametrize("key", sorted(irgen.SMALL))
def test_reference_emitter_ptx_matches_oracle(key):
    """The reference's own PTX for the same IR (committed fixture), JIT-compiled for this GPU,
    on the same seeded inputs: pins the oracle to the reference implementation."""
    p = irgen.SMALL[key]()
    ptx = (GOLDEN / "ref_ptx" / f"{key}.ptx").read_text()
    dev = Device.get(torch.cuda.current_device())
    mod = dev.load_ptx(ptx)
    fn = dev.function(mod, p.entry)
    t_cpu = data.make_inputs(p)
    t = {k: v.cuda() for k, v in t_cpu.items()}
    stream = torch.cuda.current_stream().cuda_stream
    for name in p.zero_outputs:
        t[name].zero_()
    smem = p.smem_bytes
    dev.launch_u64(fn, [p.grid, 1, 1], [p.block, 1, 1], smem, stream, [t[n].data_ptr() for n in p.arg_order])
    torch.cuda.synchronize()
    want = oracle_outputs(p, t_cpu)
    for a in p.outputs:
        compare(t[a.name].cpu(), want[a.name], a.dtype, rtol_for(p), f"ref:{key}.{a.name}")
    dev.unload(mod)


# ---- full benchmark sizes ---------------------------------------------------------------------


def test_full_sum_f32_and_i32():
    for key in ("c2", "c2i"):
        p = irgen.FULL[key]()
        t = data.make_inputs(p)
        got, _ = _run_ours(p, t)
        x = t["x"]
        if p.params["dtype"] == "i32":
            want = x.long().sum()
            assert abs(int(want)) < 2 ** 31
            assert int(got["out"].item()) == int(want)
        else:
            want = float(np.sum(x.numpy().astype(np.float64)))
            assert abs(got["out"].item() - want) <= 1e-5 * abs(want)


def test_full_softmax():
    p = irgen.FULL["c1"]()
    t = data.make_inputs(p)
    got, _ = _run_ours(p, t)
    want = torch.softmax(t["x"].cuda().double(), dim=-1).cpu()
    compare(got["y"], want, "f32", 1e-5, "c1 full")


def test_full_fused_bf16():
    p = irgen.FULL["c3"]()
    t = data.make_inputs(p)
    got, _ = _run_ours(p, t)
    a, b, c, d = (t[k].cuda() for k in "abcd")
    want = (torch.relu(a.double() * b.double() + c.double()) * torch.exp(d.double())).cpu()
    compare(got["y"], want, "bf16", 1e-5, "c3 full")


def test_tensor_core_gemm_many_tiles_per_cta():
    """Two CTAs walk all eight tiles: accumulator ping-pong and ring wrap-around are exercised."""
    p = irgen.SMALL["c4tc"]()
    t = data.make_inputs(p)
    want = oracle_outputs(p, t)
    got, ex = _run_ours(p, t, sms=2, gemm_pair=False)
    assert ex.records[0]["kind"] == "tcgen05_gemm" and ex.records[0]["grid"] == [2, 1, 1]
    assert ex.error_code() == 0
    compare(got["C"], want["C"], "f32", 1e-4, "c4tc sms=2")


def test_full_bmm_tensor_core_sampled():
    p = irgen.FULL["c4"]()
    gen = torch.Generator(device="cuda").manual_seed(7)
    A = (torch.randn(p.spec("A").shape, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    B = (torch.randn(p.spec("B").shape, generator=gen, device="cuda") * 0.02).to(torch.bfloat16)
    C = torch.empty(p.spec("C").shape, dtype=torch.float32, device="cuda")
    mod = compile_graph(Graph.from_dict(p.graph), p.meta())
    assert mod.kernels[0]["kind"] == "tcgen05_gemm_pair"
    ex = Executable(mod)
    ex({"A": A, "B": B, "C": C})
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    for b in (0, 7, 15):
        want = torch.matmul(A[b].double(), B[b].double())
        compare(C[b], want, "f32", 1e-4, f"c4 full batch {b}")


def test_full_attention_tensor_core_sampled():
    """Config 5 at full size through the tcgen05 kernel; sampled heads against float64 attention."""
    full_attention_check({})


def full_attention_check(opts):
    """Config 5 at full size compiled with ``opts``; heads (0,0), (3,17), (7,31) against float64."""
    import math
    p = irgen.FULL["c5"]()
    gen = torch.Generator(device="cuda").manual_seed(11)
    shape = p.spec("Q").shape
    Q, K, V = ((torch.randn(shape, generator=gen, device="cuda")).to(torch.bfloat16) for _ in range(3))
    O = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), opts)
    assert mod.kernels[-1]["kind"] == "tcgen05_attention"
    ex = Executable(mod)
    ex({"Q": Q, "K": K, "V": V, "O": O})
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    scale = 1.0 / math.sqrt(shape[-1])
    for b, h in ((0, 0), (3, 17), (7, 31)):
        q, k, v = Q[b, h].double(), K[b, h].double(), V[b, h].double()
        s_ = (q @ k.T) * scale
        s_ = s_.masked_fill(torch.ones_like(s_, dtype=torch.bool).triu(1), float("-inf"))
        want = torch.softmax(s_, -1) @ v
        compare(O[b, h], want, "bf16", 1e-4, f"c5 full ({b},{h})", rms_floor=True)


@pytest.mark.parametrize("mode", ["mixed", "all_large"])
def test_attention_value_range_fallback(mode):
    """V blocks whose values do not fit f16 stay bf16 (P as bf16 hi + lo) while the other blocks use
    f16: the result still matches the oracle.  ``mixed`` puts 2^20-scaled values in one 64-row kv
    block, ``all_large`` in every row, and one infinity-free extreme (the largest bf16) appears too."""
    p = irgen.SMALL["c5tc"]()
    t_cpu = data.make_inputs(p)
    V = t_cpu["V"].float()
    if mode == "mixed":
        V[:, :, 64:128] *= 2.0 ** 20
    else:
        V *= 2.0 ** 20
        V[0, 0, 5, 3] = 3.3895313892515355e38
    t_cpu["V"] = V.to(torch.bfloat16)
    want = oracle_outputs(p, t_cpu)
    got, ex = _run_ours(p, t_cpu)
    assert ex.error_code() == 0
    compare(got["O"], want["O"], "bf16", rtol_for(p), f"range {mode}", rms_floor=True)


def test_attention_two_stream_schedule():
    """The opt-in overlapped lowering: the second (batch, head) group's value pre-pass runs on the
    runtime's side stream, and that group's attention waits for it through an event.  The f16 copy of
    V and the block flags are poisoned before the call, so an attention that ran before its pre-pass
    would read NaNs or the wrong format; the result must match the oracle."""
    p = irgen.SMALL["c5tc"]()
    t_cpu = data.make_inputs(p)
    want = oracle_outputs(p, t_cpu)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"attn_overlap": True, "attn_overlap_split": 2})
    assert [r.get("stream", 0) for r in mod.kernels] == [0, 0, 1, 0]
    ex = Executable(mod)
    t = {k: v.cuda() for k, v in t_cpu.items()}
    for _ in range(2):
        for v in ex.scratch.values():
            if v.is_floating_point():
                v.fill_(float("nan"))
            else:
                v.fill_(1)
        t["O"].zero_()
        ex(t)
        torch.cuda.synchronize()
        assert ex.error_code() == 0
        compare(t["O"].cpu(), want["O"], "bf16", rtol_for(p), "two-stream attention", rms_floor=True)
    ex.close()
