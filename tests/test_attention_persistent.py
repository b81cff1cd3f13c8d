"""The persistent attention schedule (``attn_persistent``), checked on the CPU.

The CTA simulation (:mod:`tests.ctasim`) runs every CTA of small launches in which each CTA walks
several work units (including the shortest causal ones, whose lower rows need two key/value blocks),
and checks that every barrier hand-over completes, that every output row is written by exactly one
warp, every Q tile is loaded exactly once, and every K / V block as often as the units that need it.
The one-thread walk (:mod:`tests.ptxsim`) checks the softmax warpgroups' MUFU turns across unit
boundaries, with and without an injected time-out.
"""
import collections
import math

import pytest

from emmy_ptx_b200 import irgen
from emmy_ptx_b200.codegen.module import module_text, parse_records
from emmy_ptx_b200.compiler import compile_graph
from emmy_ptx_b200.ir import Graph
from emmy_ptx_b200.kernels import tc_attention_persistent as tap

from tests.ctasim import CtaSim
from tests.ptxsim import Walk, barrier_protocol_ok

B, H, S, CTAS = 1, 3, 1024, 5            # 12 units over 5 CTAs: 2 or 3 units each


def _kernel(causal=True, half=True, ctas=CTAS, heads=H, seq=S):
    b = tap.persistent_attention_entry("attn", B, heads, seq, causal, 1 / math.sqrt(128), half=half, ctas=ctas)
    txt = module_text([b])
    return txt, parse_records(txt)[0]


@pytest.mark.parametrize("causal,half", [(True, True), (True, False), (False, True), (False, False)])
def test_every_cta_completes(causal, half):
    txt, rec = _kernel(causal, half)
    sim = CtaSim(txt, rec)
    for cta in range(rec["grid"][0]):
        for seed in (0, 1):
            r = sim.run(ctaid=cta, seed=100 * cta + seed)
            assert r["errors"] == [], (cta, seed, r["errors"])


def test_flagged_blocks_and_slow_completions():
    txt, rec = _kernel()
    sim = CtaSim(txt, rec)
    for cta in range(rec["grid"][0]):
        assert sim.run(ctaid=cta, seed=7, global_load=lambda ins, regs: 1)["errors"] == []
        assert sim.run(ctaid=cta, seed=8, delay=(200, 2000))["errors"] == []


@pytest.mark.parametrize("causal", [True, False])
def test_units_cover_the_problem_once(causal):
    txt, rec = _kernel(causal)
    sim = CtaSim(txt, rec)
    rows, qs, kv = collections.Counter(), collections.Counter(), collections.Counter()
    for cta in range(rec["grid"][0]):
        r = sim.run(ctaid=cta, seed=cta, log_tma=True)
        for _, addr in r["stores"]:
            rows[addr // 256] += 1                      # one O row: 128 bf16
        for _, name, cs, _ in r["tma"]:
            if name == "tmQ":
                qs[cs] += 1
            else:
                kv[(name,) + cs] += 1
    # the simulated thread of each warp is lane 0: rows 0, 32, 64, 96 of each 128-row tile, each
    # stored as 8 pieces of 32 bytes by one thread
    assert set(rows) == {(bh * S + r) for bh in range(B * H) for r in range(0, S, 32)}
    assert set(rows.values()) == {8}
    assert len(qs) == B * H * (S // 128) * 2 and set(qs.values()) == {1}
    nblk, nt = S // 64, S // 256
    for j in range(nblk):
        want = (nt - j // 4) if causal else nt          # units whose rows reach kv block j
        for name in ("tmK", "tmV16"):
            for hh in range(H):
                for col in (0, 64):
                    assert kv[(name, col, 64 * j, hh, 0)] == want, (name, j, hh, col)


def test_turns_pair_across_units():
    txt, rec = _kernel()
    w = Walk(txt)
    for cta in range(rec["grid"][0]):
        seqs = {}
        for first in (4, 8):
            per_warp = [w.run(tid=32 * (first + q), ctaid=cta) for q in range(4)]
            assert all(s_ == per_warp[0] for s_ in per_warp)
            seqs[first] = [e for e in per_warp[0] if e[1] in (1, 2)]
        assert barrier_protocol_ok(seqs, 256) is None, cta


@pytest.mark.parametrize("warp", [4, 8])
def test_timeouts_keep_the_turns(warp):
    txt, rec = _kernel()
    w = Walk(txt)
    cta = 0
    base = w.run(tid=32 * warp, ctaid=cta)
    n = [0]

    def count(k):
        n[0] += 1
        return True
    w.run(tid=32 * warp, ctaid=cta, wait=count)
    for k in sorted({0, 1, n[0] // 2, n[0] - 1}):
        ev = w.run(tid=32 * warp, ctaid=cta, wait=lambda i, k=k: i < k)
        assert [e for e in ev if e[0] != "store_err"] == base, k
        assert ("store_err", tap.ERR_SOFTMAX) in ev or ("store_err", tap.ERR_EPILOGUE) in ev


def test_lowering_option():
    full = irgen.FULL["c5"]()
    recs = compile_graph(Graph.from_dict(full.graph), full.meta(), {"attn_persistent": True}).kernels
    assert [r["kind"] for r in recs] == ["value_prepass", "tcgen05_attention"]
    assert recs[1]["grid"] == [148, 1, 1] and recs[1]["block"] == [384, 1, 1]


def _schedule(P, batch, heads, seq):
    """Each CTA's units in order, as (batch, head, 256-row tile): unit k*P + c on even rounds and
    k*P + (P-1-c) on odd ones, the longest causal tiles first; a CTA stops at its first missing unit."""
    nbh, nt = batch * heads, seq // 256
    out = []
    for c in range(P):
        units, k = [], 0
        while True:
            u = k * P + (P - 1 - c if k & 1 else c)
            if u >= nbh * nt:
                break
            bh = u % nbh
            units.append((bh // heads, bh % heads, nt - 1 - u // nbh))
            k += 1
        out.append(units)
    return out


def test_schedule_model_matches_the_kernel():
    # the units each simulated CTA loads Q for, in order, are the model's
    txt, rec = _kernel()
    sim = CtaSim(txt, rec)
    model = _schedule(CTAS, B, H, S)
    for cta in range(rec["grid"][0]):
        seen = []
        for _, name, cs, _ in sim.run(ctaid=cta, seed=cta, log_tma=True)["tma"]:
            if name == "tmQ":
                u = (cs[3], cs[2], cs[1] // 256)
                if u not in seen:
                    seen.append(u)
        assert seen == model[cta], cta


def test_config5_schedule_is_balanced():
    # config 5 (8 x 32 x 4096, causal) over 148 CTAs: a unit's work is its 64-row key/value blocks over
    # both row halves, 8t + 6 for tile t; the busiest CTA is within 1 % of the mean
    sched = _schedule(148, 8, 32, 4096)
    work = [sum(8 * t + 6 for _, _, t in units) for units in sched]
    assert sum(len(u) for u in sched) == 8 * 32 * 16
    assert max(work) <= 1.01 * (sum(work) / len(work))
