"""GPU parity for the coverage corpus: this backend's kernels (default, and the plain CUDA-core forms
with the tensor-core lowering off) and the reference emitter's PTX for the same IR, each against the
CPU oracle on the same seeded inputs.

Outputs start filled with a 0x7F byte pattern instead of zeros, so an element a kernel fails to write
(or a ZeroPrologue that does not run first) shows up as a mismatch.
"""
from pathlib import Path

import pytest
import torch

from emmy_ptx_b200 import corpus, data
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.launcher import Device
from emmy_ptx_b200.runtime import Executable
from oracle.run import oracle_outputs
from tests.checks import compare, rtol_for, atol_for, rms_floor_for

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
KEYS = sorted(corpus.CORPUS)


def _device_tensors(p, t_cpu):
    t = {k: v.cuda() for k, v in t_cpu.items()}
    for a in p.outputs:
        t[a.name].view(torch.uint8).fill_(0x7F)
    return t


def _check(p, got, want, tag):
    for a in p.outputs:
        compare(got[a.name].cpu(), want[a.name], a.dtype, rtol_for(p), f"{tag}.{a.name}", atol=atol_for(p),
                rms_floor=rms_floor_for(p))


@pytest.mark.parametrize("opts", [{}, {"tree_barriers": True, "no_redux": True, "no_unroll": True, "patterns": False}],
                         ids=["default", "plain"])
@pytest.mark.parametrize("key", KEYS)
def test_corpus_kernel_matches_oracle(key, opts):
    p = corpus.CORPUS[key]()
    t_cpu = data.make_inputs(p)
    want = oracle_outputs(p, t_cpu)
    ex = Executable(compile_graph(Graph.from_dict(p.graph), p.meta(), opts))
    t = _device_tensors(p, t_cpu)
    ex(t)
    torch.cuda.synchronize()
    _check(p, t, want, key)
    ex.close()


@pytest.mark.parametrize("key", KEYS)
def test_reference_emitter_ptx_on_corpus_matches_oracle(key):
    """The reference's own PTX for each corpus IR, run on the same inputs, pins the oracle to it."""
    path = GOLDEN / "ref_ptx" / f"{key}.ptx"
    if not path.exists():
        pytest.skip("the reference emitter rejects this IR (recorded in the golden manifest)")
    p = corpus.CORPUS[key]()
    dev = Device.get(torch.cuda.current_device())
    mod = dev.load_ptx(path.read_text())
    t_cpu = data.make_inputs(p)
    t = _device_tensors(p, t_cpu)
    stream = torch.cuda.current_stream().cuda_stream
    launches = getattr(p, "launches", None) or [(p.entry, p.grid, p.block, p.zero_outputs, p.arg_order)]
    for entry, grid, block, zero, order in launches:
        for name in zero:
            t[name].zero_()
        fn = dev.function(mod, entry)
        dev.launch_u64(fn, [grid, 1, 1], [block, 1, 1], 0, stream, [t[n].data_ptr() for n in order])
    torch.cuda.synchronize()
    _check(p, t, oracle_outputs(p, t_cpu), f"ref:{key}")
    dev.unload(mod)
