"""Planted mistakes in the oracle must be caught by the golden source-expression vectors.

Each test changes one rule of the oracle's restatement of the reference semantics (on the CPU, for
the duration of the test) and checks that the comparison against the committed float64 vectors
fails: the vectors pin those rules, not just the kernels that happen to agree with them.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from emmy_ptx_b200 import corpus, data
from oracle import interp
from oracle.run import oracle_outputs
from tests.checks import compare

GOLDEN = Path(__file__).resolve().parent / "golden"


def _matches_vectors(key) -> bool:
    p = corpus.CORPUS[key]()
    got = oracle_outputs(p, data.make_inputs(p))
    vec = np.load(GOLDEN / "vectors" / f"{key}.npz")
    try:
        for a in p.outputs:
            compare(got[a.name], torch.from_numpy(vec[a.name]).reshape(a.shape), a.dtype, 1e-4, a.name)
    except AssertionError:
        return False
    return True


def test_unplanted_oracle_matches():
    assert _matches_vectors("k_special") and _matches_vectors("k_intops")


def test_unordered_not_equal_is_caught(monkeypatch):
    # setp.ne is ordered (NaN != NaN is false); numpy's != is not
    monkeypatch.setitem(interp.COMPARE, "not_equal", np.not_equal)
    assert not _matches_vectors("k_special")


def test_floor_division_is_caught(monkeypatch):
    # integer division truncates toward zero (div.s32); floor division differs for negative operands
    monkeypatch.setattr(interp, "_trunc_div", lambda a, b: np.asarray(a, np.int64) // np.asarray(b, np.int64))
    assert not _matches_vectors("k_intops")


def test_last_true_select_branch_is_caught(monkeypatch):
    # Select: the first true branch wins; taking the last true one changes x > 10 (both predicates hold)
    def last_wins(self, st, mask):
        brs = list(st.branches)
        vals = [self.value(b.value) for b in brs]
        L = len(mask)
        out = np.broadcast_to(np.asarray(interp._cast(vals[-1], "i32").v), (L,)).copy()
        for b, v in zip(brs[:-1], vals[:-1]):
            p = np.broadcast_to(interp._cast(self.expr(b.select), "pred").v, (L,))
            out = np.where(p, np.broadcast_to(np.asarray(v.v), (L,)), out)
        self.env[st.name] = interp.Val(out.astype(np.int32), "i")
    monkeypatch.setattr(interp.Interpreter, "st_Select", last_wins)
    assert not _matches_vectors("k_intops")


def test_nan_keeping_max_is_caught(monkeypatch):
    # max.f32 returns the non-NaN operand (relu of NaN is 0); a NaN-propagating max differs
    monkeypatch.setitem(interp.BINARY_F, "maximum", np.maximum)
    assert not _matches_vectors("k_special")
