"""The register allocator with liveness reuse (``emmy_ptx_b200.codegen.regalloc``)."""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from emmy_ptx_b200 import corpus, irgen
from emmy_ptx_b200.codegen.ptxcheck import undefined_uses
from emmy_ptx_b200.codegen.regalloc import allocate
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph

PTXAS = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"


def test_disjoint_live_ranges_share_a_register_and_overlapping_ones_do_not():
    body = [
        "\tmov.f32 %f1, 0f3F800000;",
        "\tadd.f32 %f2, %f1, %f1;",        # %f1 dies here
        "\tmul.f32 %f3, %f2, %f2;",        # %f2 dies here
        "\tadd.f32 %f4, %f3, %f3;",
        "\tst.global.f32 [%rd1], %f4;",
    ]
    out, counts = allocate(body)
    assert counts["f"] == 1                # a chain of single-use values needs one register
    body2 = [
        "\tmov.f32 %f1, 0f3F800000;",
        "\tmov.f32 %f2, 0f40000000;",
        "\tadd.f32 %f3, %f1, %f2;",        # %f1 and %f2 live together
        "\tst.global.f32 [%rd1], %f3;",
    ]
    out2, counts2 = allocate(body2)
    regs = re.findall(r"%f\d+", out2[2])
    assert regs[1] != regs[2] and counts2["f"] == 2


def test_a_guarded_write_keeps_the_old_value_alive():
    body = [
        "\tmov.f32 %f1, 0f3F800000;",
        "\tsetp.gt.f32 %p1, %f1, 0f00000000;",
        "\tmov.f32 %f2, 0f40000000;",
        "\t@%p1 mov.f32 %f2, %f1;",        # %f2 keeps 2.0 where %p1 is false
        "\tst.global.f32 [%rd1], %f2;",
    ]
    out, _ = allocate(body)
    r_old = re.findall(r"%f\d+", out[2])[0]
    r_new = re.findall(r"%f\d+", out[3])[0]
    assert r_old == r_new                  # the guarded write goes to the same register
    assert re.findall(r"%f\d+", out[3])[1] != r_new   # and its source (still live) is another one


def test_loop_carried_values_survive_the_back_edge():
    body = [
        "\tmov.f32 %f1, 0f00000000;",
        "\tmov.u32 %r1, 0;",
        "$L1:",
        "\tmov.f32 %f2, 0f3F800000;",       # a temporary inside the loop
        "\tadd.f32 %f1, %f1, %f2;",        # the accumulator lives around the loop
        "\tadd.u32 %r1, %r1, 1;",
        "\tsetp.lt.u32 %p1, %r1, 4;",
        "\t@%p1 bra $L1;",
        "\tst.global.f32 [%rd1], %f1;",
    ]
    out, counts = allocate(body)
    acc = re.findall(r"%f\d+", out[4])[0]
    tmp = re.findall(r"%f\d+", out[3])[0]
    assert acc != tmp and counts["f"] == 2


def _all():
    return {**irgen.SMALL, **corpus.CORPUS}


@pytest.mark.parametrize("key", sorted(_all()))
def test_allocation_keeps_kernels_valid_and_no_larger(key, tmp_path):
    if not Path(PTXAS).exists():
        pytest.skip("ptxas not available")
    p = _all()[key]()
    used = []
    for ra in (False, True):
        ptx = compile_graph(Graph.from_dict(p.graph), p.meta(), {"regalloc": ra, "patterns": False}).ptx
        assert undefined_uses(ptx) == []
        src = tmp_path / f"k{int(ra)}.ptx"
        src.write_text(ptx)
        r = subprocess.run([PTXAS, "-arch=sm_100a", "-v", str(src), "-o", str(tmp_path / "k.cubin")],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
        used.append([int(x) for x in re.findall(r"Used (\d+) registers", r.stderr)])
        if ra:
            declared = sum(int(n) for n in re.findall(r"\.reg \.\w+ %\w+<(\d+)>", ptx))
    assert used[1] <= used[0] or all(b <= a + 2 for a, b in zip(used[0], used[1]))
    assert declared <= 200
