"""The entry point that allocates nothing, checked against the allocating path.

Some callers cannot allocate device memory when they launch (a host whose own memory pool owns the
GPU, or a latency-critical path where cudaMalloc may synchronise the device).  For them the C ABI has
``emmy_bmm_bf16_noalloc``: the tensor-core batched matmul with its 16-byte scratch (the status word of
its bounded pipeline waits) in a fixed array inside the library instead of a per-call allocation, and
``emmy_bmm_bf16_noalloc_status`` to read that word back.
This file runs last so that a failure here never hides the other tests' results.
"""
import pytest
import torch

from emmy_ptx_b200 import irgen, data
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.runtime import Executable
from tests.checks import compare

pytestmark = pytest.mark.gpu


def _setup():
    p = irgen.SMALL["c4tc"]()
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"gemm_pair": False})   # one CTA per tile
    rec = mod.kernels[0]
    assert rec["kind"] == "tcgen05_gemm"
    ex = Executable(mod)
    t = {k: v.cuda() for k, v in data.make_inputs(p).items()}
    tmaps = [ex._tmap(spec, t[spec["tensor"]]) for spec in rec["tmaps"]]
    return rec, ex, t, tmaps


def test_noalloc_bmm_matches_the_allocating_entry_point_twice():
    rec, ex, t, tmaps = _setup()
    ex(t)                                                   # the allocating path (runtime status word)
    torch.cuda.synchronize()
    assert ex.error_code() == 0
    want = t["C"].clone()

    stream = torch.cuda.current_stream().cuda_stream
    outs = [torch.full_like(want, float("nan")) for _ in range(4)]
    torch.cuda.synchronize()
    for call, out in enumerate(outs):
        free_before = torch.cuda.mem_get_info()[0]
        ex.dev.bmm_noalloc(ex.funcs[0], tmaps[0].addr, tmaps[1].addr, t["A"].data_ptr(), t["B"].data_ptr(),
                           out.data_ptr(), rec["grid"][0], rec["block"][0], rec["dyn_smem"], 16, stream)
        assert ex.dev.bmm_noalloc_status(stream) == 0, f"no-alloc call {call}: a pipeline wait timed out"
        if call > 0:
            # the first call on a device may load the library's device code (the array lives there);
            # every later call must leave the device's free memory exactly as it found it
            assert torch.cuda.mem_get_info()[0] == free_before, f"no-alloc call {call} changed free memory"
        torch.cuda.synchronize()
        compare(out, want, "f32", 1e-4, f"no-alloc call {call}")


def test_noalloc_rejects_scratch_beyond_its_array():
    from emmy_ptx_b200.launcher import EmmyError
    rec, ex, t, tmaps = _setup()
    with pytest.raises(EmmyError, match="scratch"):
        ex.dev.bmm_noalloc(ex.funcs[0], tmaps[0].addr, tmaps[1].addr, t["A"].data_ptr(), t["B"].data_ptr(),
                           t["C"].data_ptr(), rec["grid"][0], rec["block"][0], rec["dyn_smem"], 4096,
                           torch.cuda.current_stream().cuda_stream)
