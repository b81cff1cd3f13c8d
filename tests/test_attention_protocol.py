"""The attention kernel's named-barrier protocol, checked on the CPU by walking its PTX.

With ``pingpong`` the two query tiles' softmax warpgroups hand the MUFU turn to each other through
named barriers 1 and 2.  A ``bar.sync`` has no time-out, so a warp that skipped a hand-over (say
after an mbarrier time-out) would leave the other warpgroup waiting for good.  These tests walk the
emitted PTX one softmax thread at a time (:mod:`ptxsim`) and check that

* the two warpgroups' barrier sequences complete against each other for every CTA (no deadlock, no
  double arrival in one phase, nothing left over), and all four warps of a warpgroup agree;
* a time-out at any mbarrier wait of a softmax warp, with or without an O rescale, leaves that
  warp's barrier sequence unchanged and writes the softmax error code.
"""
import math

import pytest

from emmy_ptx_b200.codegen.module import module_text
from emmy_ptx_b200.kernels import tc_attention as ta

from tests.ptxsim import Walk, barrier_protocol_ok

SOFT0, SOFT1 = 4, 8          # first warp of each tile's softmax warpgroup


def _walk(causal=True, half=True, seq=1024, heads=1):
    b = ta.attention_entry("attn", 1, heads, seq, causal, 1 / math.sqrt(128), pingpong=True, half=half)
    return Walk(module_text([b])), b["grid"][0]


def _bars(events):
    return [e for e in events if e[0] != "store_err"]


def _count_waits(w, tid, cta, fcmp=None):
    n = [0]

    def wait(k):
        n[0] += 1
        return True
    w.run(tid=tid, ctaid=cta, wait=wait, fcmp=fcmp)
    return n[0]


@pytest.mark.parametrize("causal,half", [(True, True), (True, False), (False, True)])
def test_turns_complete_for_every_cta(causal, half):
    w, grid = _walk(causal, half)
    for cta in range(grid):
        seqs = {}
        for first in (SOFT0, SOFT1):
            per_warp = [w.run(tid=32 * (first + q) + 5, ctaid=cta) for q in range(4)]
            assert all(s == per_warp[0] for s in per_warp), (cta, first)
            assert not [e for e in per_warp[0] if e[0] == "store_err"]
            seqs[first] = [e for e in per_warp[0] if e[1] in (1, 2)]
        assert seqs[SOFT0] and seqs[SOFT1]
        assert barrier_protocol_ok(seqs, 256) is None, (cta, barrier_protocol_ok(seqs, 256))


def test_protocol_checker_catches_a_missing_hand_over():
    w, _ = _walk()
    s0 = [e for e in w.run(tid=32 * SOFT0, ctaid=0) if e[1] in (1, 2)]
    s1 = [e for e in w.run(tid=32 * SOFT1, ctaid=0) if e[1] in (1, 2)]
    assert barrier_protocol_ok({0: s0, 1: s1}, 256) is None
    assert "deadlock" in barrier_protocol_ok({0: s0[:-1], 1: s1}, 256)
    dup = s1[:3] + [s1[2]] + s1[3:]
    assert barrier_protocol_ok({0: s0, 1: dup}, 256) is not None


@pytest.mark.parametrize("warp", [SOFT0, SOFT1])
@pytest.mark.parametrize("cta", [0, 3])          # the longest (16 / 14 kv blocks) and shortest CTA
def test_timeout_keeps_the_hand_overs(warp, cta):
    w, _ = _walk()
    tid = 32 * warp
    base = w.run(tid=tid, ctaid=cta)
    n = _count_waits(w, tid, cta)
    picks = sorted({0, 1, 2, n // 2, n - 2, n - 1}) if n > 6 else range(n)
    for k in picks:
        ev = w.run(tid=tid, ctaid=cta, wait=lambda i, k=k: i < k)
        assert _bars(ev) == base, (k, _bars(ev)[:8])
        assert ("store_err", ta.ERR_SOFTMAX) in ev or ("store_err", ta.ERR_EPILOGUE) in ev, k


@pytest.mark.parametrize("warp", [SOFT0, SOFT1])
def test_timeout_in_the_rescale_wait(warp):
    # the shortest CTA (4 / 2 kv blocks); its second block raises the running max, so the softmax
    # waits for the previous PV before rescaling O; a time-out there keeps the hand-overs too
    w, _ = _walk()
    tid, cta = 32 * warp, 3

    def fcmp(k):
        return k == 0
    base = w.run(tid=tid, ctaid=cta)
    assert _bars(w.run(tid=tid, ctaid=cta, fcmp=fcmp)) == base
    n = _count_waits(w, tid, cta, fcmp)
    assert n > _count_waits(w, tid, cta)          # the rescale added a wait
    for k in range(n):
        ev = w.run(tid=tid, ctaid=cta, wait=lambda i, k=k: i < k, fcmp=fcmp)
        assert _bars(ev) == base, k


def test_turns_are_off_without_pingpong():
    b = ta.attention_entry("attn", 1, 1, 1024, True, 1 / math.sqrt(128), pingpong=False)
    w = Walk(module_text([b]))
    ev = w.run(tid=32 * SOFT0, ctaid=0)
    assert [e for e in ev if e[1] in (1, 2)] == []
