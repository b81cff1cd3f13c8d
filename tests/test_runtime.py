"""The runtime's launch sequence, on the CPU: an Executable driven through a fake device records every
call, so the order of zeroing, launches, stream forks and joins can be checked without a GPU."""
import pytest
import torch

from emmy_ptx_b200 import corpus, data, irgen, launcher
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.runtime import Executable

MAIN, SIDE = 100, 777


class FakeDevice:
    """Stands in for :class:`launcher.Device`: returns handles and logs the calls that order work."""

    def __init__(self):
        self.log = []
        self.events = 0
        self.launches = 0

    def load_ptx(self, ptx):
        return "module"

    def function(self, mod, entry):
        return entry

    def set_max_dyn_smem(self, fn, nbytes):
        pass

    def set_carveout(self, fn, percent):
        self.log.append(("carveout", fn, percent))

    def stream(self):
        return SIDE

    def sync_event(self):
        self.events += 1
        return f"ev{self.events}"

    def record(self, ev, stream):
        self.log.append(("record", ev, stream))

    def wait_event(self, stream, ev):
        self.log.append(("wait", stream, ev))

    def memset_d32(self, ptr, value, count, stream):
        self.log.append(("zero", count, stream))

    def launch_u64(self, fn, grid, block, dyn_smem, stream, params, align=None, pdl=False):
        self.log.append(("launch", fn, stream))

    def launch(self, fn, grid, block, dyn_smem, stream, arg_ptrs, cluster=(1, 1, 1), pdl=False):
        self.log.append(("launch", fn, stream))

    def tmap_encode_tiled(self, *args, **kw):
        pass

    def unload(self, mod):
        pass

    def destroy_event(self, ev):
        pass

    def destroy_stream(self, stream):
        pass


class HostExecutable(Executable):
    def _device_tensor(self, shape, dtype):
        return torch.empty(shape, dtype=dtype)


@pytest.fixture
def fake(monkeypatch):
    dev = FakeDevice()
    monkeypatch.setattr(launcher.Device, "get", classmethod(lambda cls, index=0: dev))
    return dev


def _exe(p, opts=None):
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), opts or {})
    return HostExecutable(mod, device=0), data.make_inputs(p)


def test_two_stream_schedule_orders_the_side_stream(fake):
    # the opt-in overlap: pre-pass 0 and attention 0 on the caller's stream, pre-pass 1 on the side
    # stream after pre-pass 0, attention 1 after pre-pass 1, and the side stream joined at the end
    ex, t = _exe(irgen.attention_ir(1, 16, 512, 128), {"attn_overlap": True})
    names = [r["entry"] for r in ex.records]
    ev = {n: ex._events[n] for n in names}
    fork = ex._fork
    ex.run(t, MAIN)
    launches = [(e[1], e[2]) for e in fake.log if e[0] == "launch"]
    assert launches == [(names[0], MAIN), (names[1], MAIN), (names[2], SIDE), (names[3], MAIN)]
    order = [e for e in fake.log if e[0] in ("record", "wait", "launch")]
    assert order == [
        ("launch", names[0], MAIN), ("record", ev[names[0]], MAIN),
        ("launch", names[1], MAIN), ("record", ev[names[1]], MAIN),
        ("record", fork, MAIN), ("wait", SIDE, fork),             # fork: the side stream follows the main one
        ("wait", SIDE, ev[names[0]]),                            # "after" pre-pass 0, on the other stream
        ("launch", names[2], SIDE), ("record", ev[names[2]], SIDE),
        ("wait", MAIN, ev[names[2]]),                            # attention 1 after pre-pass 1
        ("launch", names[3], MAIN), ("record", ev[names[3]], MAIN),
        ("wait", MAIN, ev[names[2]]),                            # join before returning
    ]
    assert ("carveout", names[2], 100) in fake.log


def test_one_stream_module_launches_in_order(fake):
    ex, t = _exe(irgen.attention_ir(1, 2, 512, 128))
    ex.run(t, MAIN)
    assert [e for e in fake.log if e[0] != "zero"] == [("launch", r["entry"], MAIN) for r in ex.records]


def test_zeroing_precedes_its_launch_and_can_be_skipped(fake):
    p = irgen.SMALL["c2"]()                       # the sum accumulates into a zeroed scalar
    ex, t = _exe(p)
    ex.run(t, MAIN)
    assert fake.log == [("zero", 1, MAIN), ("launch", ex.records[0]["entry"], MAIN)]
    fake.log.clear()
    ex.run(t, MAIN, zero=False)
    assert fake.log == [("launch", ex.records[0]["entry"], MAIN)]


def test_empty_grid_launches_nothing(fake):
    ex, t = _exe(corpus.rmsnorm(0, 512))          # zero rows: a zero-block grid
    assert ex.records[0]["grid"][0] == 0
    ex.run(t, MAIN)
    assert not [e for e in fake.log if e[0] == "launch"]


def test_misaligned_operand_is_refused_before_launch(fake):
    ex, t = _exe(irgen.attention_ir(1, 2, 512, 128))
    o = t["O"]
    shifted = torch.empty(o.numel() + 1, dtype=o.dtype)[1:].view(o.shape)      # 2 bytes past an aligned base
    with pytest.raises(ValueError, match="aligned"):
        ex.run({**t, "O": shifted}, MAIN)
    assert not [e for e in fake.log if e[0] == "launch" and e[1] == ex.records[-1]["entry"]]
