"""The static def-use check of PTX (``emmy_ptx_b200.codegen.ptxcheck``), on hand-written snippets and
on every kernel this backend emits and every reference PTX fixture that a GPU test launches."""
from pathlib import Path

import pytest

from emmy_ptx_b200 import corpus, irgen
from emmy_ptx_b200.codegen.ptxcheck import undefined_uses
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph

GOLDEN = Path(__file__).resolve().parent / "golden"


def _kernel(body: str, decls: str = ".reg .pred %p<4>;\n.reg .b32 %r<16>;\n.reg .f32 %f<8>;\n.reg .b64 %rd<8>;") -> str:
    return f""".version 8.8
.target sm_100a
.address_size 64
.visible .entry k(
\t.param .u64 p_x
)
{{
{decls}
{body}
}}
"""


def test_value_from_the_then_branch_read_in_the_else_branch_is_reported():
    ptx = _kernel("""
    ld.param.u64 %rd1, [p_x];
    mov.u32 %r1, %tid.x;
    setp.lt.s32 %p1, %r1, 7;
    @!%p1 bra ELSE;
    mad.wide.s32 %rd4, %r1, 4, %rd1;
    st.global.u32 [%rd4], %r1;
    bra END;
ELSE:
    st.global.u32 [%rd4], %r1;
END:
    ret;
""")
    got = undefined_uses(ptx)
    assert [(r, t.strip()) for _, _, r, t in got] == [("%rd4", "st.global.u32 [%rd4], %r1;")]


def test_nested_integer_guards_are_not_reported():
    ptx = _kernel("""
    mov.u32 %r1, %tid.x;
    setp.lt.s32 %p1, %r1, 4;
    @!%p1 bra S1;
    mad.lo.s32 %r2, %r1, 4, 0;
    ld.shared.f32 %f1, [%r2];
S1:
    bar.sync 0;
    setp.lt.s32 %p2, %r1, 2;
    @!%p2 bra S2;
    ld.shared.f32 %f2, [%r2];
S2:
    ret;
""")
    assert undefined_uses(ptx) == []


def test_the_widening_guard_is_reported():
    """The same shape with the second guard wider than the first leaves %r2 undefined for 4 <= t < 8."""
    ptx = _kernel("""
    mov.u32 %r1, %tid.x;
    setp.lt.s32 %p1, %r1, 4;
    @!%p1 bra S1;
    mad.lo.s32 %r2, %r1, 4, 0;
S1:
    setp.lt.s32 %p2, %r1, 8;
    @!%p2 bra S2;
    ld.shared.f32 %f2, [%r2];
S2:
    ret;
""")
    assert [r for _, _, r, _ in undefined_uses(ptx)] == ["%r2"]


def test_a_predicate_tested_twice_is_correlated():
    ptx = _kernel("""
    mov.u32 %r1, %tid.x;
    setp.ne.s32 %p1, %r1, 0;
    @!%p1 bra A;
    add.f32 %f1, %f2, 0f3F800000;
A:
    mov.u32 %r3, 5;
    @!%p1 bra B;
    mul.f32 %f3, %f1, %f1;
B:
    ret;
""", ".reg .pred %p<4>;\n.reg .b32 %r<8>;\n.reg .f32 %f<8>;")
    # %f2 is read before any write (a genuine finding); %f1's use follows its definition's guard
    assert sorted(r for _, _, r, _ in undefined_uses(ptx)) == ["%f2"]


def test_a_loop_skipped_at_run_time_leaves_its_values_undefined_after_it():
    ptx = _kernel("""
    mov.u32 %r1, %tid.x;
    ld.param.u64 %rd1, [p_x];
    ld.global.u32 %r2, [%rd1];
    mov.b32 %r3, 0;
    setp.ge.s32 %p1, %r3, %r2;
    @%p1 bra EXIT;
    shr.u32 %r4, %r1, 4;
TOP:
    add.s32 %r3, %r3, 1;
    setp.lt.s32 %p2, %r3, %r2;
    @%p2 bra TOP;
EXIT:
    st.global.u32 [%rd1], %r4;
    ret;
""")
    assert [r for _, _, r, _ in undefined_uses(ptx)] == ["%r4"]


def test_vector_and_pair_destinations_count_as_writes():
    ptx = _kernel("""
    ld.param.u64 %rd1, [p_x];
    ld.global.v4.f32 {%f1, %f2, %f3, %f4}, [%rd1];
    mov.u32 %r1, %laneid;
    shfl.sync.bfly.b32 %r2|%p1, %r1, 1, 31, -1;
    @%p1 add.f32 %f5, %f1, %f4;
    st.global.v2.f32 [%rd1], {%f2, %f3};
    ret;
""")
    assert undefined_uses(ptx) == []


def _all_problems():
    return {**irgen.SMALL, **corpus.CORPUS, **{f"full_{k}": v for k, v in irgen.FULL.items()}}


@pytest.mark.parametrize("key", sorted(_all_problems()))
def test_every_emitted_kernel_reads_only_written_registers(key):
    p = _all_problems()[key]()
    for opts in ({}, {"patterns": False, "tree_barriers": True, "no_redux": True}):
        ptx = compile_graph(Graph.from_dict(p.graph), p.meta(), opts).ptx
        assert undefined_uses(ptx) == [], (key, opts)


def test_every_reference_fixture_that_runs_on_a_gpu_passes_the_check():
    for path in sorted((GOLDEN / "ref_ptx").glob("*.ptx")):
        assert undefined_uses(path.read_text()) == [], path.name
