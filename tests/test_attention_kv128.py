"""CPU checks of the attention kernel with 128-row key/value blocks (option ``attn_kv128``).

* its emitted PTX run by the tensor-core emulator against the oracle: causal and full, f16 P with the
  pre-pass's copy of V and bf16 P_hi + P_lo, the issue order that relies on in-order MMAs, the
  packing kept in the MUFU turn, a value block outside the f16 range, and late completions;
* every CTA of small launches through the CTA simulation with randomly delayed completions (no
  deadlock, no time-out code), also with every value block flagged;
* the softmax warpgroups' named-barrier hand-overs walked one thread at a time, with a time-out
  injected at each wait;
* the register split that ``setmaxnreg`` makes fits the registers the block is launched with.
"""
import math
import re

import pytest
import torch

from emmy_ptx_b200 import data, irgen
from emmy_ptx_b200.codegen.module import module_text, parse_records
from emmy_ptx_b200.kernels import tc_attention_kv128 as t128

from tests.ctasim import CtaSim
from tests.ptxsim import Walk, barrier_protocol_ok
from tests.test_tc_emulated import _check

SOFT0, SOFT1 = 4, 8


@pytest.mark.parametrize("key,opts", [
    ("c5tc", {}),
    ("c5tcnc", {}),
    ("c5tcnc", {"attn_half": False}),
    ("c5tcnc", {"attn_ordered": True}),
    ("c5tcnc", {"attn_pack_in_turn": True}),
    ("c5tcnc", {"attn_pingpong": False}),
])
def test_kv128_emulated_matches_oracle(key, opts):
    p = irgen.SMALL[key]()
    _check(p, data.make_inputs(p), {"attn_kv128": True, **opts}, "tcgen05_attention")


def test_kv128_value_range_fallback_emulated():
    # one 128-row value block holds a value above the f16 range: that block takes bf16 P_hi + P_lo
    # with V itself, the others f16 P with the copy
    p = irgen.attention_ir(1, 1, 512, 128, True)
    t = data.make_inputs(p)
    v = t["V"].float()
    v[0, 0, 130, 5] = 2.0 ** 20
    t["V"] = v.to(torch.bfloat16)
    _check(p, t, {"attn_kv128": True}, "tcgen05_attention")


@pytest.mark.parametrize("opts", [{}, {"attn_ordered": True}])
def test_kv128_with_late_completions(opts):
    p = irgen.attention_ir(1, 1, 512, 128, True)
    _check(p, data.make_inputs(p), {"attn_kv128": True, **opts}, "tcgen05_attention", defer=True)


def _entry(**kw):
    causal = kw.pop("causal", True)
    seq = kw.pop("seq", 1024)
    b = t128.attention_kv128_entry("attn", 1, 1, seq, causal, 1 / math.sqrt(128), **kw)
    txt = module_text([b])
    return txt, parse_records(txt)[0]


def _run_all(txt, rec, seeds=(0, 1), **kw):
    sim = CtaSim(txt, rec)
    for cta in range(rec["grid"][0]):
        for seed in seeds:
            r = sim.run(ctaid=cta, seed=1000 * cta + seed, **kw)
            assert r["errors"] == [], (cta, seed, r["errors"])


@pytest.mark.parametrize("variant", [
    {}, {"pingpong": False}, {"half": False}, {"causal": False}, {"ordered": True}, {"pack_in_turn": True},
])
def test_kv128_pipeline_completes(variant):
    txt, rec = _entry(**variant)
    _run_all(txt, rec)


def test_kv128_flagged_blocks_take_the_bf16_path():
    txt, rec = _entry()
    _run_all(txt, rec, seeds=(0,), global_load=lambda ins, regs: 1)


def test_kv128_long_delays():
    txt, rec = _entry(seq=512)
    _run_all(txt, rec, seeds=(3,), delay=(200, 2000))


def _walk(causal=True, half=True, seq=1024):
    b = t128.attention_kv128_entry("attn", 1, 1, seq, causal, 1 / math.sqrt(128), half=half)
    return Walk(module_text([b])), b["grid"][0]


@pytest.mark.parametrize("causal,half", [(True, True), (True, False), (False, True)])
def test_kv128_turns_complete_for_every_cta(causal, half):
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


@pytest.mark.parametrize("warp", [SOFT0, SOFT1])
@pytest.mark.parametrize("cta", [0, 1])           # the longest (8 / 7 kv blocks) and shortest CTA
def test_kv128_timeout_keeps_the_hand_overs(warp, cta):
    w, _ = _walk()
    tid = 32 * warp
    base = w.run(tid=tid, ctaid=cta)
    n = [0]

    def count(k):
        n[0] += 1
        return True
    w.run(tid=tid, ctaid=cta, wait=count)
    picks = sorted({0, 1, 2, n[0] // 2, n[0] - 2, n[0] - 1}) if n[0] > 6 else range(n[0])
    for k in picks:
        ev = w.run(tid=tid, ctaid=cta, wait=lambda i, k=k: i < k)
        assert [e for e in ev if e[0] != "store_err"] == base, k
        assert ("store_err", t128.ERR_SOFTMAX) in ev or ("store_err", t128.ERR_EPILOGUE) in ev, k


def test_kv128_register_split_fits_the_launch():
    txt, rec = _entry()
    launch = int(re.search(r"\.maxnreg (\d+)", txt).group(1))
    dec = [int(x) for x in re.findall(r"setmaxnreg\.dec\.sync\.aligned\.u32 (\d+);", txt)]
    inc = [int(x) for x in re.findall(r"setmaxnreg\.inc\.sync\.aligned\.u32 (\d+);", txt)]
    assert dec == [t128.REGS_CONTROL] and inc == [t128.REGS_SOFTMAX]
    # warpgroup 0 (warps 0-3) gives registers up, warpgroups 1 and 2 (the softmax) take them
    assert 128 * dec[0] + 256 * inc[0] <= rec["block"][0] * launch
    assert all(v % 8 == 0 and 24 <= v <= 256 for v in dec + inc)
