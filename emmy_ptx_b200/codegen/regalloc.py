"""Typed register allocation with liveness reuse for emitted PTX bodies.

The emitter hands out a fresh virtual register for every value (as the reference's counters do,
compile.py:330-360).  This pass renames them so that registers whose values are dead are reused, per
register class: liveness by backward dataflow over the instruction-level control-flow graph, an
interference graph (a register written at a point interferes with every register live after it,
and the registers one instruction writes interfere with each other), then greedy colouring in order of
first definition.  The declared register counts shrink accordingly (``.reg .f32 %f<N>``).

A write under a guard (``@%p mov ...``) does not end the register's previous value, so the pass
treats it as a read and a write.  The renamed body reads exactly the values the original read on every
path; the test suite checks it with the def-use check, ptxas, and the GPU parity tests.
"""
from __future__ import annotations

import re

from .ptxcheck import _instructions, _NO_DEST

_REG = re.compile(r"%(rd|r|f|p|h)(\d+)\b")
# register-class prefixes as the PTX builder names them, longest first
_CLASSES = ("rd", "r", "f", "p", "h")


def _regs_in(text: str) -> list[str]:
    return [m.group(0) for m in _REG.finditer(text)]


def allocate(lines: list[str]) -> tuple[list[str], dict[str, int]]:
    """Rename the virtual registers of a kernel body (``lines``, one instruction or label each) with
    liveness reuse.  Returns the new lines and the number of registers per class prefix."""
    ins = _instructions(lines)
    n = len(ins)
    if not n:
        return list(lines), {}
    labels = {x.label: k for k, x in enumerate(ins) if x.label}
    uses, defs, kills = [], [], []
    for x in ins:
        if x.label:
            uses.append(set())
            defs.append(set())
            kills.append(set())
            continue
        u, d = set(), set()
        if x.guard:
            u.add(x.guard)
        no_dest = x.op.startswith(_NO_DEST) and not x.op.startswith("bar.red")
        first_is_dest = bool(x.ops) and not no_dest and not x.ops[0].startswith("[")
        for j, o in enumerate(x.ops):
            toks = set(_regs_in(o))
            if j == 0 and first_is_dest:
                d |= toks
            else:
                u |= toks
        if x.guard:
            u |= d                     # a guarded write keeps the old value where the guard is false
            kills.append(set())
        else:
            kills.append(set(d))
        uses.append(u)
        defs.append(d)
    succ = [[] for _ in range(n)]
    for k, x in enumerate(ins):
        if x.label:
            if k + 1 < n:
                succ[k].append(k + 1)
            continue
        if x.op.startswith("bra"):
            tgt = labels.get(x.ops[-1]) if x.ops else None
            if tgt is not None:
                succ[k].append(tgt)
            if x.guard is not None and k + 1 < n:
                succ[k].append(k + 1)
        elif x.op in ("ret", "exit") or x.op.startswith(("ret.", "exit.")):
            if x.guard is not None and k + 1 < n:
                succ[k].append(k + 1)
        elif k + 1 < n:
            succ[k].append(k + 1)
    live_in = [set() for _ in range(n)]
    live_out = [set() for _ in range(n)]
    changed = True
    while changed:
        changed = False
        for k in range(n - 1, -1, -1):
            out = set()
            for s_ in succ[k]:
                out |= live_in[s_]
            inn = uses[k] | (out - kills[k])
            if out != live_out[k] or inn != live_in[k]:
                live_out[k], live_in[k] = out, inn
                changed = True
    # interference
    adj: dict[str, set] = {}
    order: list[str] = []
    seen = set()
    for k, x in enumerate(ins):
        for r in sorted(defs[k] | uses[k]):
            if r not in seen:
                seen.add(r)
                order.append(r)
                adj.setdefault(r, set())
        for d_ in defs[k]:
            for r in live_out[k]:
                if r != d_:
                    adj[d_].add(r)
                    adj.setdefault(r, set()).add(d_)
            for d2 in defs[k]:
                if d2 != d_:
                    adj[d_].add(d2)
    for r in live_in[0] if n else ():
        for r2 in live_in[0]:
            if r2 != r:
                adj.setdefault(r, set()).add(r2)
    # greedy colouring per class, in order of first appearance
    cls_of = lambda r: _REG.match(r).group(1)        # noqa: E731
    color: dict[str, int] = {}
    counts: dict[str, int] = {}
    for r in order:
        taken = {color[q] for q in adj.get(r, ()) if q in color and cls_of(q) == cls_of(r)}
        c = 1
        while c in taken:
            c += 1
        color[r] = c
        counts[cls_of(r)] = max(counts.get(cls_of(r), 0), c)
    mapping = {r: f"%{cls_of(r)}{c}" for r, c in color.items()}
    out_lines = [_REG.sub(lambda m: mapping.get(m.group(0), m.group(0)), ln) for ln in lines]
    return out_lines, counts
