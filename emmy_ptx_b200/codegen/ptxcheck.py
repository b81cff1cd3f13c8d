"""A static check of PTX text: every register read has been written on every feasible path.

PTX gives no such guarantee.  A register read before any write holds whatever was left there, and a
garbage address faults the GPU.  :func:`undefined_uses` walks each ``.entry`` instruction by
instruction and computes the set of registers written on all paths that reach each point.

The analysis is a must-analysis with light path sensitivity, so the two usual correlated-branch
forms are not reported:

* a predicate tested twice, with no write to it in between (``@!%p bra A ... @!%p bra B``): the
  second branch follows the first;
* nested integer guards on one register, e.g. ``setp.lt.s32 %p, %r1, 4`` and later ``%r1 < 2``.
  An interval per register, learned from branches on ``setp.<cmp>.s32 %p, %rX, imm``, decides a
  later guard that the interval already settles.

Each program point keeps a few (facts, written registers) states, merged by facts.  Past a small
bound they collapse into one state without facts; the analysis loses precision but stays sound.
A write under a guard (``@%p mov ...``) counts as a write.

The test suite runs this on every kernel this backend emits.  It also runs on the reference
emitter's PTX before that PTX is kept as a fixture that runs on a GPU.
"""
from __future__ import annotations

import re

_DECL = re.compile(r"\.reg\s+\.\w+\s+(.+?);")
_TOKEN = re.compile(r"%?[A-Za-z_$][\w$]*")
_LABEL = re.compile(r"^([A-Za-z_$][\w$]*):$")
_IMM = re.compile(r"^-?(?:0[xX][0-9a-fA-F]+|\d+)$")
_MAX_STATES = 16
_INF = float("inf")

# opcodes whose first operand is read, not written
_NO_DEST = ("st.", "red.", "bar.", "bar ", "barrier.", "bra", "ret", "exit", "membar", "fence", "griddepcontrol",
            "setmaxnreg", "trap", "prefetch", "nanosleep", "cp.async", "tcgen05.dealloc", "tcgen05.relinquish",
            "tcgen05.fence", "tcgen05.wait", "tcgen05.st", "tcgen05.mma", "tcgen05.commit", "tcgen05.alloc",
            "tcgen05.cp", "tcgen05.shift", "mbarrier.init", "mbarrier.expect_tx", "mbarrier.inval", "stmatrix",
            "multimem.st", "multimem.red", "pmevent", "call")


def _split_operands(s: str) -> list[str]:
    out, depth, cur = [], 0, []
    for ch in s:
        if ch in "{[":
            depth += 1
        elif ch in "}]":
            depth -= 1
        if ch == "," and depth == 0:
            out.append("".join(cur).strip())
            cur = []
        else:
            cur.append(ch)
    tail = "".join(cur).strip()
    if tail:
        out.append(tail)
    return out


def _declared(lines) -> set[str]:
    names = set()
    for ln in lines:
        for m in _DECL.finditer(ln):
            for part in m.group(1).split(","):
                part = part.strip()
                r = re.fullmatch(r"(%?[A-Za-z_$][\w$]*)<(\d+)>", part)
                if r:
                    names.update(f"{r.group(1)}{i}" for i in range(int(r.group(2))))
                elif part:
                    names.add(part)
    return names


def _entries(ptx: str):
    """(entry name, body lines) for every ``.entry`` / ``.func`` of the module."""
    lines = [ln.split("//", 1)[0].strip() for ln in ptx.splitlines()]
    i = 0
    while i < len(lines):
        ln = lines[i]
        m = re.match(r"^(?:\.visible\s+|\.weak\s+)?\.(?:entry|func)\s+(?:\([^)]*\)\s*)?([\w$]+)", ln)
        if not m:
            i += 1
            continue
        j = i
        while j < len(lines) and lines[j] != "{":
            j += 1
        depth, k, body = 0, j, []
        while k < len(lines):
            depth += lines[k].count("{") - lines[k].count("}")
            body.append(lines[k])
            k += 1
            if depth == 0:
                break
        yield m.group(1), body
        i = k


class _Ins:
    __slots__ = ("line", "label", "guard", "neg", "op", "ops", "uses", "defs")

    def __init__(self, line, label=None, guard=None, neg=False, op="", ops=()):
        self.line, self.label, self.guard, self.neg, self.op, self.ops = line, label, guard, neg, op, list(ops)
        self.uses, self.defs = set(), set()


def _instructions(body) -> list[_Ins]:
    out = []
    for idx, ln in enumerate(body):
        s = ln.strip()
        if not s or s.startswith("."):
            continue
        for stmt in (x.strip() for x in s.split(";")):
            # scope braces of inline blocks ("{ .reg ...; ... }") are not instructions
            while stmt.startswith("{") and not stmt.startswith(("{%", "{ %")):
                stmt = stmt[1:].strip()
            while stmt.endswith("}") and stmt.count("{") < stmt.count("}"):
                stmt = stmt[:-1].strip()
            if not stmt or stmt.startswith("."):
                continue
            lm = _LABEL.match(stmt)
            if lm:
                out.append(_Ins(idx, label=lm.group(1)))
                continue
            guard, neg = None, False
            if stmt.startswith("@"):
                g, stmt = stmt.split(None, 1)
                neg = g.startswith("@!")
                guard = g[2:] if neg else g[1:]
            parts = stmt.split(None, 1)
            out.append(_Ins(idx, guard=guard, neg=neg, op=parts[0],
                            ops=_split_operands(parts[1]) if len(parts) > 1 else []))
    return out


def _cmp_holds(cmp: str, lo: float, hi: float, k: int):
    """Whether ``x <cmp> k`` is settled for every x in [lo, hi]: True, False or None."""
    if cmp == "lt":
        return True if hi < k else (False if lo >= k else None)
    if cmp == "le":
        return True if hi <= k else (False if lo > k else None)
    if cmp == "gt":
        return True if lo > k else (False if hi <= k else None)
    if cmp == "ge":
        return True if lo >= k else (False if hi < k else None)
    if cmp == "eq":
        return True if lo == hi == k else (False if k < lo or k > hi else None)
    if cmp == "ne":
        return False if lo == hi == k else (True if k < lo or k > hi else None)
    return None


def _refine(cmp: str, truth: bool, lo: float, hi: float, k: int):
    """The interval of x after learning ``(x <cmp> k) == truth``; None when that is impossible."""
    if not truth:
        cmp = {"lt": "ge", "le": "gt", "gt": "le", "ge": "lt", "eq": "ne", "ne": "eq"}[cmp]
    if cmp == "lt":
        hi = min(hi, k - 1)
    elif cmp == "le":
        hi = min(hi, k)
    elif cmp == "gt":
        lo = max(lo, k + 1)
    elif cmp == "ge":
        lo = max(lo, k)
    elif cmp == "eq":
        lo, hi = max(lo, k), min(hi, k)
    elif cmp == "ne":
        if lo == hi == k:
            return None
        return lo, hi
    return (lo, hi) if lo <= hi else None


class _Facts:
    """Immutable path facts: predicate truths, predicate definitions ``p := (x cmp k)``, intervals."""

    __slots__ = ("pv", "pd", "iv", "_key")

    def __init__(self, pv=None, pd=None, iv=None):
        self.pv = pv or {}
        self.pd = pd or {}
        self.iv = iv or {}
        self._key = None

    def key(self):
        if self._key is None:
            self._key = (frozenset(self.pv.items()), frozenset(self.pd.items()), frozenset(self.iv.items()))
        return self._key

    def kill(self, regs) -> "_Facts":
        if not regs:
            return self
        pv = {p: v for p, v in self.pv.items() if p not in regs}
        pd = {p: d for p, d in self.pd.items() if p not in regs and d[0] not in regs}
        iv = {r: v for r, v in self.iv.items() if r not in regs}
        if len(pv) == len(self.pv) and len(pd) == len(self.pd) and len(iv) == len(self.iv):
            return self
        return _Facts(pv, pd, iv)

    def with_def(self, p, d) -> "_Facts":
        pd = dict(self.pd)
        pd[p] = d
        return _Facts(dict(self.pv), pd, dict(self.iv))

    def decide(self, p):
        if p in self.pv:
            return self.pv[p]
        d = self.pd.get(p)
        if d is not None:
            x, cmp, k = d
            lo, hi = self.iv.get(x, (-_INF, _INF))
            return _cmp_holds(cmp, lo, hi, k)
        return None

    def learn(self, p, truth) -> "_Facts | None":
        pv = dict(self.pv)
        pv[p] = truth
        iv = dict(self.iv)
        d = self.pd.get(p)
        if d is not None:
            x, cmp, k = d
            lo, hi = iv.get(x, (-_INF, _INF))
            r = _refine(cmp, truth, lo, hi, k)
            if r is None:
                return None
            iv[x] = r
        return _Facts(pv, dict(self.pd), iv)


_SETP = re.compile(r"^setp\.(lt|le|gt|ge|eq|ne)\.s32$")


def _merge(states: dict) -> dict:
    if len(states) <= _MAX_STATES:
        return states
    allw = frozenset.intersection(*states.values())
    return {_Facts().key(): allw}


def undefined_uses(ptx: str) -> list[tuple[str, int, str, str]]:
    """Every (entry, body line, register, source line) where a register may be read before any
    write on some feasible path from the entry."""
    problems = []
    for name, body in _entries(ptx):
        regs = _declared(body)
        ins = _instructions(body)
        n = len(ins)
        labels = {x.label: k for k, x in enumerate(ins) if x.label}
        for x in ins:
            if x.label:
                continue
            if x.guard in regs:
                x.uses.add(x.guard)
            no_dest = x.op.startswith(_NO_DEST) and not x.op.startswith("bar.red")   # bar.red writes a result
            first_is_dest = bool(x.ops) and not no_dest and not x.ops[0].startswith("[")
            for j, o in enumerate(x.ops):
                toks = {t for t in _TOKEN.findall(o) if t in regs}
                if j == 0 and first_is_dest:
                    x.defs |= toks
                else:
                    x.uses |= toks
        facts_of = {}            # facts key -> _Facts
        state = [dict() for _ in range(n)]   # per instruction: facts key -> written set (on entry)
        if n:
            f0 = _Facts()
            facts_of[f0.key()] = f0
            state[0] = {f0.key(): frozenset()}
        work = [0] if n else []
        inwork = set(work)

        def push(k, fk, written):
            cur = state[k]
            old = cur.get(fk)
            new = written if old is None else (old & written)
            if old is not None and new == old:
                return
            cur[fk] = new
            state[k] = _merge(cur)
            if k not in inwork:
                inwork.add(k)
                work.append(k)

        def transfer(f: _Facts, x: _Ins) -> _Facts:
            """Facts after ``x`` executes: what it writes is forgotten; a compare of a register
            with an immediate (or of a register with itself) defines its predicate."""
            f2 = f.kill(x.defs)
            m = _SETP.match(x.op)
            if m and len(x.ops) == 3 and x.ops[0] in regs:
                a, b = x.ops[1], x.ops[2]
                if a in regs and _IMM.match(b):
                    f2 = f2.with_def(x.ops[0], (a, m.group(1), int(b, 0)))
                elif a == b and a in regs and m.group(1) in ("eq", "ne"):
                    f2 = f2.learn(x.ops[0], m.group(1) == "eq")
            return f2

        def follow(k, x, f, written):
            """Propagate one executed instruction's outgoing state to its successors."""
            if x.op.startswith("bra"):
                tgt = labels.get(x.ops[-1]) if x.ops else None
                if tgt is not None:
                    facts_of[f.key()] = f
                    push(tgt, f.key(), written)
                return
            if x.op in ("ret", "exit") or x.op.startswith(("ret.", "exit.")):
                return
            if k + 1 < n:
                facts_of[f.key()] = f
                push(k + 1, f.key(), written)

        while work:
            k = work.pop()
            inwork.discard(k)
            x = ins[k]
            for fk, written in list(state[k].items()):
                f = facts_of.get(fk) or _Facts()
                if x.label:
                    if k + 1 < n:
                        push(k + 1, fk, written)
                    continue
                if x.guard is None:
                    follow(k, x, transfer(f, x), written | x.defs)
                    continue
                # guarded: the instruction runs when the guard equals ``not neg``
                truth = f.decide(x.guard)
                for g in ((truth,) if truth is not None else (True, False)):
                    base = f if truth is not None else f.learn(x.guard, g)
                    if base is None:
                        continue
                    if g != x.neg:
                        follow(k, x, transfer(base, x), written | x.defs)
                    elif k + 1 < n:
                        facts_of[base.key()] = base
                        push(k + 1, base.key(), written)
        for k in range(n):
            x = ins[k]
            if x.label or not state[k] or not x.uses:
                continue
            have = frozenset.intersection(*state[k].values())
            for r in sorted(x.uses - have):
                problems.append((name, x.line, r, body[x.line]))
    return problems
