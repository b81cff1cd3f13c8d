"""The multi-GPU sum's peer-exchange kernel (:mod:`emmy_ptx_b200.kernels.peer_sum`) and its host side.

On the CPU the kernel of one rank runs in the PTX emulator against exchange buffers in which the other
ranks' steps have already been published: it must write its partial and flag into every rank's buffer,
read the others' slots of the step's parity, and leave the rank-ordered total; a peer that never arrives
ends the bounded wait with status code 51.  Two gloo ranks check the handle exchange and the agreement
used to pick the exchange path.  On a GPU one rank (world 1) runs the real kernel, and with two GPUs two
processes exchange over NVLink.
"""
import os
import socket
import struct

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from emmy_ptx_b200 import dist as edist
from emmy_ptx_b200.codegen.module import module_text
from emmy_ptx_b200.kernels import peer_sum
from tests.ptxemu import Emulator, Memory


def _publish(buf, world, step, rank, value, dtype):
    off = peer_sum.DATA + 8 * ((step & 1) * world + rank)
    buf[off:off + 4] = np.frombuffer(struct.pack("<f" if dtype == "f32" else "<i", value), np.uint8)
    buf[peer_sum.FLAGS + 4 * rank:peer_sum.FLAGS + 4 * rank + 4] = np.frombuffer(struct.pack("<I", step), np.uint8)


def _emulate(world, rank, vals, dtype, steps=1, missing=()):
    """Run ``steps`` launches of rank ``rank``'s kernel; before launch e every other rank (but those in
    ``missing``) has published step e.  Returns the totals, the status word and the buffers."""
    rec = peer_sum.peer_sum_entry(f"peer_sum_{dtype}", rank, world, dtype)
    ptx = module_text([rec])
    mem = Memory()
    bufs = [mem.alloc(np.zeros(peer_sum.BUF_BYTES, np.uint8)) for _ in range(world)]
    table = mem.alloc(np.array(bufs, np.uint64))
    err = mem.alloc(np.zeros(4, np.int32))
    npdt = np.float32 if dtype == "f32" else np.int32
    totals = []
    for e in range(1, steps + 1):
        own = mem.array(bufs[rank], np.uint8, (-1,))
        for k in range(world):
            if k != rank and k not in missing:
                _publish(own, world, e, k, vals[e - 1][k], dtype)
        out = mem.alloc(np.array([vals[e - 1][rank]], npdt))
        Emulator(ptx, rec["name"]).run(1, 32, {"p_out": out, "p_xch": bufs[rank], "p_peers": table, "p_err": err},
                                       mem, 0)
        totals.append(mem.array(out, npdt, (1,))[0])
    return totals, int(mem.array(err, np.int32, (4,))[0]), [mem.array(b, np.uint8, (-1,)) for b in bufs]


@pytest.mark.parametrize("rank", [0, 1, 2])
def test_exchange_gives_the_rank_ordered_total(rank):
    rng = np.random.default_rng(rank)
    vals = [rng.standard_normal(3).astype(np.float32).tolist() for _ in range(3)]
    totals, code, bufs = _emulate(3, rank, vals, "f32", steps=3)
    assert code == 0
    for e, got in enumerate(totals, start=1):
        want = np.float32(0)
        for k in range(3):                      # the order every rank adds in: 0, 1, ..., N-1
            want = np.float32(want + np.float32(vals[e - 1][k]))
        assert got == want, (e, got, want)
    # the last step (3, parity 1) left this rank's partial and flag in every rank's buffer
    for b in bufs:
        off = peer_sum.DATA + 8 * (1 * 3 + rank)
        assert struct.unpack("<f", bytes(b[off:off + 4]))[0] == np.float32(vals[2][rank])
        assert struct.unpack("<I", bytes(b[peer_sum.FLAGS + 4 * rank:peer_sum.FLAGS + 4 * rank + 4]))[0] == 3
    assert struct.unpack("<I", bytes(bufs[rank][0:4]))[0] == 3       # the step counter


def test_integer_exchange_is_exact():
    vals = [[2 ** 30, -7, 123456789, -(2 ** 30)]]
    totals, code, _ = _emulate(4, 2, vals, "i32")
    assert code == 0 and int(totals[0]) == sum(vals[0])


def test_a_peer_that_never_arrives_ends_the_wait_with_a_status():
    totals, code, _ = _emulate(2, 0, [[1.0, 2.0]], "f32", missing=(1,))
    assert code == peer_sum.ERR_PEER_WAIT


def test_kernel_assembles_for_every_world_size():
    import shutil
    import subprocess
    import tempfile
    from pathlib import Path
    ptxas = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
    for world in (1, 2, 8):
        for dtype in ("f32", "i32"):
            txt = module_text([peer_sum.peer_sum_entry("x", world - 1, world, dtype)])
            assert "multimem" not in txt and "multicast" not in txt
            with tempfile.TemporaryDirectory() as td:
                f = Path(td) / "k.ptx"
                f.write_text(txt)
                r = subprocess.run([ptxas, "-arch=sm_100a", str(f), "-o", str(Path(td) / "k.cubin")],
                                   capture_output=True, text=True)
                assert r.returncode == 0, r.stderr


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker_handles(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    d = edist.init(world, rank, backend="gloo", timeout_s=30.0)
    try:
        hs = edist.exchange_handles(d, rank, world, bytes([rank]) * 64)
        both = edist.agree(d, True)
        one = edist.agree(d, rank == 0)
        q.put((rank, [h[0] for h in hs], both, one))
    finally:
        d.destroy_process_group()


def test_handles_and_agreement_across_two_gloo_ranks():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_handles, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    for rank, firsts, both, one in res:
        assert firsts == [0, 1] and both is True and one is False


@pytest.mark.gpu
def test_one_rank_exchange_on_the_gpu():
    from emmy_ptx_b200.launcher import Device
    dev = Device.get(torch.cuda.current_device())
    ex = edist.PeerAllReduce(dev, None, 0, 1, "f32")
    try:
        out = torch.tensor([3.25], dtype=torch.float32, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        for _ in range(5):
            ex(out, "f32", stream)
        torch.cuda.synchronize()
        assert ex.error_code() == 0 and out.item() == 3.25
    finally:
        ex.close()


def _worker_gpu(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    d = edist.init(world, rank, backend="nccl", timeout_s=60.0)
    from emmy_ptx_b200.launcher import Device
    dev = Device.get(rank)
    ex = edist.PeerAllReduce(dev, d, rank, world, "f32")
    try:
        stream = torch.cuda.current_stream().cuda_stream
        got = []
        for step in range(4):
            out = torch.tensor([0.5 + rank + 10 * step], dtype=torch.float32, device="cuda")
            ex(out, "f32", stream)
            torch.cuda.synchronize()
            got.append(out.item())
        q.put((rank, got, ex.error_code()))
    finally:
        ex.close()
        d.barrier()
        d.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_exchange_over_nvlink():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_gpu, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    want = [np.float32(np.float32(0.5 + 10 * s) + np.float32(1.5 + 10 * s)) for s in range(4)]
    for rank, got, code in res:
        assert code == 0 and got == [float(w) for w in want], (rank, got)


def _emulate_fused(world, rank, dtype, peers_by_step, launches=2):
    """The reduction kernel with the exchange fused as its epilogue, run ``launches`` times for rank
    ``rank``; before launch e the other ranks have published ``peers_by_step[e-1]``."""
    from emmy_ptx_b200 import data, irgen
    from emmy_ptx_b200.compiler import compile_graph
    from emmy_ptx_b200.ir import Graph
    p = irgen.sum_ir(1 << 12, dtype, blocks=4, threads=128)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(),
                        {"exchange": {"rank": rank, "world": world, "partial": "out", "dtype": dtype}})
    rec = mod.kernels[0]
    acc_spec = rec["scratch"][0]
    assert [s["name"] for s in rec["extra"]] == ["__xch", "__peers", acc_spec["name"], "__err"]
    assert rec["zero_outputs"] == [] and rec["self_zeroing"] == ["out"] and acc_spec["zeroed"]
    t = data.make_inputs(p)
    npdt = np.float32 if dtype == "f32" else np.int32
    mem = Memory()
    x = mem.alloc(t["x"].numpy().copy())
    bufs = [mem.alloc(np.zeros(peer_sum.BUF_BYTES, np.uint8)) for _ in range(world)]
    table = mem.alloc(np.array(bufs, np.uint64))
    err = mem.alloc(np.zeros(4, np.int32))
    acc = mem.alloc(np.zeros(acc_spec["shape"][0], np.int32))  # zeroed once, as the runtime does
    own = mem.array(bufs[rank], np.uint8, (-1,))
    got = []
    for e in range(1, launches + 1):
        for k, v in peers_by_step[e - 1].items():
            _publish(own, world, e, k, v, dtype)
        out = mem.alloc(np.full(1, 0x7F7F7F7F, np.uint32).view(npdt))   # not zeroed: the kernel writes it
        Emulator(mod.ptx, rec["entry"]).run(rec["grid"][0], rec["block"][0],
                                            {"p_x": x, "p_out": out, "p_xch": bufs[rank], "p_peers": table,
                                             "p_acc": acc, "p_err": err}, mem, rec.get("dyn_smem", 0))
        got.append(mem.array(out, npdt, (1,))[0])
        # the ticket and the accumulator are zero again for the next launch
        assert not mem.array(acc, np.int32, (acc_spec["shape"][0],)).any()
    return t, got, int(mem.array(err, np.int32, (4,))[0])


def test_fused_reduction_and_exchange_f32():
    peers = [{0: 10.5, 1: -3.25}, {0: 1.0, 1: 2.0}]
    t, got, code = _emulate_fused(3, 2, "f32", peers)
    assert code == 0
    local = t["x"].double().sum().item()
    for g, pe in zip(got, peers):
        assert abs(g - (local + sum(pe.values()))) <= 1e-5 * abs(local + sum(pe.values()))


def test_fused_reduction_and_exchange_i32_is_exact():
    peers = [{1: 123456}, {1: -98765}]
    t, got, code = _emulate_fused(2, 0, "i32", peers)
    assert code == 0
    local = int(t["x"].long().sum().item())
    assert [int(g) for g in got] == [local + 123456, local - 98765]


def test_fused_kernel_assembles():
    import shutil
    import subprocess
    import tempfile
    from pathlib import Path
    from emmy_ptx_b200 import irgen
    from emmy_ptx_b200.codegen.ptxcheck import undefined_uses
    from emmy_ptx_b200.compiler import compile_graph
    from emmy_ptx_b200.ir import Graph
    ptxas = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
    for dtype in ("f32", "i32"):
        p = irgen.FULL["c2" if dtype == "f32" else "c2i"]()
        mod = compile_graph(Graph.from_dict(p.graph), p.meta(),
                            {"exchange": {"rank": 5, "world": 8, "partial": "out", "dtype": dtype}})
        assert not undefined_uses(mod.ptx)
        with tempfile.TemporaryDirectory() as td:
            f = Path(td) / "k.ptx"
            f.write_text(mod.ptx)
            r = subprocess.run([ptxas, "-arch=sm_100a", str(f), "-o", str(Path(td) / "k.cubin")],
                               capture_output=True, text=True)
            assert r.returncode == 0, r.stderr


def _fused_executable(dev, rank, world, dtype, n=1 << 20):
    from emmy_ptx_b200 import irgen
    from emmy_ptx_b200.compiler import compile_graph
    from emmy_ptx_b200.ir import Graph
    from emmy_ptx_b200.runtime import Executable
    p = irgen.sum_ir(n, dtype, blocks=148, threads=256)
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(),
                        {"exchange": {"rank": rank, "world": world, "partial": "out", "dtype": dtype}})
    return p, Executable(mod, device=dev.index)


@pytest.mark.gpu
def test_fused_reduction_and_exchange_one_rank_on_the_gpu():
    """The reduction with its exchange epilogue (world 1): the output is the block sum, launch after
    launch (the ticket counter resets itself), for f32 and i32."""
    from emmy_ptx_b200 import data
    from emmy_ptx_b200.launcher import Device
    dev = Device.get(torch.cuda.current_device())
    for dtype in ("f32", "i32"):
        xr = edist.PeerAllReduce(dev, None, 0, 1, dtype)
        try:
            p, ex = _fused_executable(dev, 0, 1, dtype)
            t = {k: v.cuda() for k, v in data.make_inputs(p).items()}
            t["__xch"], t["__peers"] = xr.xch, xr.table
            want = t["x"].double().sum().item() if dtype == "f32" else int(t["x"].long().sum().item())
            for _ in range(3):
                ex(t)
                torch.cuda.synchronize()
                assert ex.error_code() == 0
                got = t["out"].item()
                assert (got == want) if dtype == "i32" else abs(got - want) <= 1e-5 * abs(want)
            ex.close()
        finally:
            xr.close()


def _worker_fused(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank), NCCL_NVLS_ENABLE="0")
    d = edist.init(world, rank, backend="nccl", timeout_s=60.0)
    from emmy_ptx_b200 import data
    from emmy_ptx_b200.launcher import Device
    dev = Device.get(rank)
    xr = edist.PeerAllReduce(dev, d, rank, world, "i32")
    try:
        p, ex = _fused_executable(dev, rank, world, "i32")
        t = {k: v.cuda() for k, v in data.make_inputs(p, seed_offset=rank).items()}
        t["__xch"], t["__peers"] = xr.xch, xr.table
        local = torch.tensor([int(t["x"].long().sum().item())], dtype=torch.int64, device="cuda")
        total = local.clone()
        d.all_reduce(total)
        got = []
        for _ in range(3):
            ex(t)
            torch.cuda.synchronize()
            got.append(int(t["out"].item()))
        q.put((rank, got, int(total.item()), ex.error_code()))
        ex.close()
    finally:
        d.barrier()
        xr.close()
        d.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_reduction_and_exchange_over_nvlink():
    world, port = 2, _port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_fused, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    for rank, got, total, code in res:
        assert code == 0 and got == [total] * 3, (rank, got, total)
