"""The tensor-core kernels' synchronisation, simulated on the CPU for every CTA of small launches.

:mod:`tests.ctasim` runs one thread per warp of the emitted PTX with shared mbarriers (counts,
transaction bytes, parity), named barriers and randomly delayed TMA / ``tcgen05.commit`` completions.
A kernel passes when every CTA runs to its end under several interleavings with no time-out code
written and no deadlock.  The planted-mistake tests show the simulation notices a missing hand-over.
"""
import math
import re

import pytest

from emmy_ptx_b200 import irgen
from emmy_ptx_b200.codegen.module import module_text, parse_records
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.kernels import tc_attention as ta

from tests.ctasim import CtaSim, Deadlock


def _attention(**kw):
    causal = kw.pop("causal", True)
    seq = kw.pop("seq", 1024)
    b = ta.attention_entry("attn", 1, 1, seq, causal, 1 / math.sqrt(128), **kw)
    txt = module_text([b])
    return txt, parse_records(txt)[0]


def _run_all(txt, rec, seeds=(0, 1), **kw):
    sim = CtaSim(txt, rec)
    for cta in range(rec["grid"][0]):
        for seed in seeds:
            r = sim.run(ctaid=cta, seed=1000 * cta + seed, **kw)
            assert r["errors"] == [], (cta, seed, r["errors"])


@pytest.mark.parametrize("variant", [
    {}, {"pingpong": False}, {"half": False}, {"causal": False}, {"precise": False},
    {"pack_after_turn": True, "defer_sum": True}, {"prefetch_next": 2}, {"pack_in_turn": True},
])
def test_attention_pipeline_completes(variant):
    txt, rec = _attention(**variant)
    _run_all(txt, rec)


def test_attention_head_dim_64_pipeline_completes():
    txt, rec = _attention(dim=64)
    _run_all(txt, rec)


@pytest.mark.parametrize("seq,causal", [(320, True), (200, True), (200, False), (700, False)])
def test_attention_ragged_sequence_pipeline_completes(seq, causal):
    # S no multiple of 256 (or 64): the same hand-overs, with the key-limit mask and the rows past S
    # skipped at the store
    txt, rec = _attention(seq=seq, causal=causal)
    _run_all(txt, rec)


def test_attention_flagged_blocks_take_the_bf16_path():
    # every value block flagged as not fitting f16: the producer loads V itself and the MMA issuers
    # and softmax take the two-part P path; the hand-overs are the same
    txt, rec = _attention()
    _run_all(txt, rec, seeds=(0,), global_load=lambda ins, regs: 1)


def test_attention_long_delays():
    # completions far slower than the threads: every wait really sleeps
    txt, rec = _attention(seq=512)
    _run_all(txt, rec, seeds=(3,), delay=(200, 2000))


def test_gemm_pipeline_completes():
    p = irgen.SMALL["c4tc"]()
    for sms in (1, 3, 4):
        mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"sms": sms, "gemm_pair": False})
        rec = mod.kernels[0]
        assert rec["kind"] == "tcgen05_gemm"
        _run_all(mod.ptx, rec, seeds=(0, 1))


def test_gemm_edge_tiles_pipeline_completes():
    # edge tiles in M, N and K: the same hand-overs as full tiles (the masking is in the stores only)
    p = irgen.bmm_naive_ir(1, 200, 264, 72)
    for sms in (1, 3):
        mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"sms": sms, "gemm_pair": False})
        rec = mod.kernels[0]
        assert rec["kind"] == "tcgen05_gemm"
        _run_all(mod.ptx, rec, seeds=(0,))


def _expect_deadlock(txt, rec):
    sim = CtaSim(txt, rec)
    with pytest.raises(Deadlock):
        for cta in range(rec["grid"][0]):
            sim.run(ctaid=cta, seed=cta)


def test_planted_missing_turn_hand_over_deadlocks():
    txt, rec = _attention()
    lines = txt.splitlines()
    k = next(i for i, ln in enumerate(lines) if "bar.arrive 2, 256" in ln)
    _expect_deadlock("\n".join(lines[:k] + lines[k + 1:]), rec)


def test_planted_wrong_arrival_count_deadlocks():
    # the P-full barriers expect one arrival per softmax warp (4); asking for 5 stalls the issuers
    txt, rec = _attention()
    bad = re.sub(r"(mbarrier\.init\.shared::cta\.b64 \[[^\]]+\]), 4;", r"\1, 5;", txt)
    assert bad != txt
    _expect_deadlock(bad, rec)


def test_planted_missing_commit_deadlocks():
    p = irgen.SMALL["c4tc"]()
    mod = compile_graph(Graph.from_dict(p.graph), p.meta(), {"sms": 2, "gemm_pair": False})
    lines = mod.ptx.splitlines()
    k = next(i for i, ln in enumerate(lines) if "tcgen05.commit" in ln)
    _expect_deadlock("\n".join(lines[:k] + lines[k + 1:]), mod.kernels[0])


def test_attention_writes_every_row_once():
    # one CTA per 256 query rows: every output row (the simulated lane 0 of each warp covers rows
    # 0, 32, 64, 96 of each tile) is written by exactly one thread, in 8 pieces of 32 bytes
    import collections
    txt, rec = _attention(seq=1024)
    sim = CtaSim(txt, rec)
    rows = collections.Counter()
    for cta in range(rec["grid"][0]):
        for _, addr in sim.run(ctaid=cta, seed=cta)["stores"]:
            rows[addr // 256] += 1
    assert set(rows) == set(range(0, 1024, 32)) and set(rows.values()) == {8}


@pytest.mark.parametrize("causal", [True, False])
def test_attention_with_mask_pipeline_completes(causal):
    # the mask adds global loads and per-column selects to the softmax threads, no hand-over
    txt, rec = _attention(seq=512, causal=causal, mask_name="M")
    _run_all(txt, rec)
