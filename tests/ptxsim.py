"""A single-thread walk of an emitted PTX entry, for checking control flow on the CPU.

The walk executes the integer, predicate and branch instructions of one thread exactly (32- and 64-bit
wraparound, C-style unsigned division) and treats the rest as opaque: floating-point results are
unknown, loads return 0 unless a callback says otherwise, and stores, fences, tensor-core and TMA
instructions do nothing.  ``mbarrier.try_wait`` asks a callback whether the wait succeeds, so a test
can make any particular wait time out, and every named-barrier operation (``bar.sync``,
``bar.arrive``, ``barrier.sync``) is recorded in order.  A floating-point comparison asks another
callback.  ``vote`` returns the thread's own predicate: the walk stands for a warp whose lanes agree.

It is test infrastructure: it proves properties of the emitted control flow (which barrier
operations a warp performs on every path) that a GPU run can only show by hanging.
"""
from __future__ import annotations

import re

from emmy_ptx_b200.codegen.ptxcheck import _entries, _instructions

from tests.ctasim import alu

_M32 = (1 << 32) - 1
_IMM = re.compile(r"^-?(?:0[xX][0-9a-fA-F]+|\d+)$")


class StepLimit(RuntimeError):
    pass


class Walk:
    """Run entry ``name`` of ``ptx`` as the thread ``tid`` of CTA ``ctaid``."""

    def __init__(self, ptx: str, name: str | None = None):
        for ename, body in _entries(ptx):
            if name is None or ename == name:
                self.ins = _instructions(body)
                break
        else:
            raise KeyError(name)
        self.labels = {x.label: k for k, x in enumerate(self.ins) if x.label}

    def run(self, tid: int, ctaid: int = 0, wait=None, fcmp=None, load=None, max_steps: int = 5_000_000):
        """Returns the recorded events: ``("bar.sync" | "bar.arrive" | "barrier.sync", id, count)``
        and ``("store_err", value)`` for stores of immediates to global memory.  ``wait(k)`` decides
        the k-th ``try_wait`` (default: succeeds), ``fcmp(k)`` the k-th floating-point ``setp``
        (default: false), ``load(k, op)`` the k-th load's value (default: 0)."""
        regs: dict[str, object] = {"%tid.x": tid, "%ctaid.x": ctaid, "%ntid.x": 0, "%smid": 0,
                                   "%laneid": tid & 31}
        events = []
        nwait = nf = nld = 0
        pc, steps = 0, 0

        def val(o: str):
            o = o.strip()
            if _IMM.match(o):
                return int(o, 0)
            if o.startswith("0f") or o.startswith("0d"):
                return None
            if re.match(r"^[A-Za-z_$]", o):
                return 0                      # a symbol: shared-memory offsets are taken from 0
            return regs.get(o)

        while pc < len(self.ins):
            steps += 1
            if steps > max_steps:
                raise StepLimit(f"more than {max_steps} steps (pc {pc})")
            x = self.ins[pc]
            pc += 1
            if x.label:
                continue
            if x.guard is not None:
                g = regs.get(x.guard)
                if g is None:
                    raise ValueError(f"guard {x.guard} unknown at line {x.line}: {x.op}")
                if bool(g) == x.neg:
                    continue
            op, ops = x.op, x.ops
            head = op.split(".")[0]
            if op == "bra" or op.startswith("bra."):
                pc = self.labels[ops[-1]]
                continue
            if op in ("ret", "exit"):
                break
            if op.startswith(("bar.sync", "bar.arrive", "barrier.sync", "barrier.arrive")) \
                    and not op.startswith("bar.warp"):
                bid = val(ops[0])
                cnt = val(ops[1]) if len(ops) > 1 else None
                events.append((op.split(".")[0] + "." + op.split(".")[1], bid, cnt))
                continue
            if op.startswith("mbarrier.try_wait"):
                ok = True if wait is None else bool(wait(nwait))
                nwait += 1
                regs[ops[0]] = ok
                continue
            if op.startswith("vote.sync"):
                regs[ops[0]] = bool(regs.get(ops[1]))
                continue
            if op.startswith("setp.") and op.split(".")[-1].startswith("f"):
                regs[ops[0]] = False if fcmp is None else bool(fcmp(nf))
                nf += 1
                continue
            if op.startswith(("ld.", "ldu.")):
                if op.startswith("ld.param") or load is None:
                    v = 0
                else:
                    v = load(nld, op)
                    nld += 1
                if ops[0].startswith("{"):
                    for r in ops[0].strip("{}").split(","):
                        regs[r.strip()] = v
                else:
                    regs[ops[0]] = v
                continue
            if op.startswith("st.global") and len(ops) == 2 and _IMM.match(ops[1].strip()):
                events.append(("store_err", int(ops[1], 0)))
                continue
            if op.startswith("vote.sync.ballot"):
                regs[ops[0]] = _M32 if regs.get(ops[1]) else 0
                continue
            try:
                if alu(op, ops, regs, val):
                    continue
            except ValueError as e:
                raise ValueError(f"line {x.line}: {e}") from None
            # anything else: its register results are unknown
            if ops and not op.startswith(("st.", "tcgen05.st", "tcgen05.mma", "tcgen05.commit", "cp.",
                                          "fence", "mbarrier.init", "mbarrier.arrive", "red.", "bar.warp")):
                d = ops[0]
                if d.startswith("{"):
                    for r in d.strip("{}").split(","):
                        regs[r.strip()] = None
                elif d.startswith("%"):
                    regs[d] = None
        return events


def barrier_protocol_ok(seqs: dict[int, list], count: int) -> str | None:
    """Replay the named-barrier operations of several thread groups (``seqs``: group -> list of
    ``(op, id, count)``; each group is ``count // len(seqs)`` threads that all perform its sequence)
    and report the first problem: a deadlock, a group arriving twice in one phase of a barrier (its
    second arrival would complete the phase without the other group), or arrivals left over at the
    end.  None when every sequence runs to its end."""
    per = count // len(seqs)
    pos = {g: 0 for g in seqs}
    waiting: dict[int, int] = {}            # group -> barrier it waits on
    pending: dict[int, set] = {}            # barrier id -> groups arrived in the current phase
    progress = True
    while progress:
        progress = False
        for g, seq in seqs.items():
            if g in waiting or pos[g] >= len(seq):
                continue
            op, bid, cnt = seq[pos[g]]
            if cnt != count:
                return f"group {g} op {pos[g]}: count {cnt}, expected {count}"
            arrived = pending.setdefault(bid, set())
            if g in arrived:
                return f"group {g} arrives twice in one phase of barrier {bid} (op {pos[g]})"
            arrived.add(g)
            if len(arrived) * per == count:
                arrived.clear()
                for w, b in list(waiting.items()):
                    if b == bid:
                        del waiting[w]
                        pos[w] += 1
                pos[g] += 1
            elif op.endswith("sync"):
                waiting[g] = bid
            else:
                pos[g] += 1
            progress = True
    if waiting:
        return "deadlock: " + ", ".join(f"group {g} waits on barrier {b} at op {pos[g]}" for g, b in waiting.items())
    left = [g for g, seq in seqs.items() if pos[g] < len(seq)]
    if left:
        return f"groups {left} did not finish"
    if any(pending.values()):
        return f"arrivals left over: {pending}"
    return None
