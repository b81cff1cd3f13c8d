"""The attention timeline summary (``python -m emmy_ptx_b200.timeline``) on a synthetic trace."""
import numpy as np

from emmy_ptx_b200.kernels import tc_attention as ta
from emmy_ptx_b200.timeline import summarise


def test_summary_intervals_of_a_synthetic_trace():
    ctas = 4
    tr = np.zeros((ctas, ta.TRACE_SLOTS, ta.TRACE_EVENTS), dtype=np.int64)
    for c in range(ctas):
        for j in range(64):
            base = 10_000 + 1_600 * j
            tr[c, j, :8] = base + np.arange(8) * 100          # issuer events 100 cycles apart
            for b in (8, 16):
                tr[c, j, b:b + 8] = base + np.array([0, 30, 230, 320, 1100, 1160, 1320, 350])
        tr[c, 65, 0], tr[c, 65, 1] = 0, 64 * 1_600
    s = summarise(tr, np.full(ctas, 15))
    iv = s["intervals"]
    assert iv["issuer 0 iteration"]["median"] == 1600
    assert iv["issuer: K(j+1) arrived -> S(j+1) issued"]["median"] == 100
    assert iv["softmax 0: turn taken -> exps done"]["median"] == 1100 - 350
    assert iv["softmax 1: P written -> next S ready"]["median"] == 1600 - 1320
    assert s["per_cta"]["t=15 (64 blocks)"]["clk_per_block"] == 1600
