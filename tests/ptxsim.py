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

_M32, _M64 = (1 << 32) - 1, (1 << 64) - 1
_IMM = re.compile(r"^-?(?:0[xX][0-9a-fA-F]+|\d+)$")


class StepLimit(RuntimeError):
    pass


def _bits(op: str) -> int:
    m = re.search(r"\.[usb](8|16|32|64)\b", op)
    return int(m.group(1)) if m else 32


def _signed(v: int, bits: int) -> int:
    v &= (1 << bits) - 1
    return v - (1 << bits) if v >> (bits - 1) else v


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
            if op.startswith("setp."):
                parts = op.split(".")
                cmp, ty = parts[1], parts[-1]
                if ty.startswith("f"):
                    r = False if fcmp is None else bool(fcmp(nf))
                    nf += 1
                else:
                    a_, b_ = val(ops[1]), val(ops[2])
                    if a_ is None or b_ is None:
                        raise ValueError(f"unknown operand at line {x.line}: {op} {ops}")
                    bits = int(ty[1:])
                    if ty[0] == "s":
                        a_, b_ = _signed(a_, bits), _signed(b_, bits)
                    else:
                        a_, b_ = a_ & ((1 << bits) - 1), b_ & ((1 << bits) - 1)
                    r = {"eq": a_ == b_, "ne": a_ != b_, "lt": a_ < b_, "le": a_ <= b_,
                         "gt": a_ > b_, "ge": a_ >= b_}[cmp]
                regs[ops[0]] = r
                continue
            if op in ("and.pred", "or.pred", "xor.pred", "not.pred"):
                if op == "not.pred":
                    regs[ops[0]] = not regs.get(ops[1])
                else:
                    a_, b_ = bool(regs.get(ops[1])), bool(regs.get(ops[2]))
                    regs[ops[0]] = {"and": a_ and b_, "or": a_ or b_, "xor": a_ != b_}[head]
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
            if op.startswith(("mov.u32", "mov.b32", "mov.u64", "mov.b64", "mov.s32")) and not ops[0].startswith("{"):
                src = ops[1].strip()
                if src.startswith("{"):
                    regs[ops[0]] = None
                elif src.startswith("%") and src not in regs and not src[1:].replace("_", "").isalnum():
                    regs[ops[0]] = None
                else:
                    regs[ops[0]] = val(src) if not re.match(r"^[A-Za-z_]", src) else 0
                continue
            if head in ("add", "sub", "mul", "mad", "shl", "shr", "and", "or", "xor", "div", "rem", "min",
                        "max", "neg", "not", "cvt", "cvta", "selp") and not ops[0].startswith("{"):
                ty = op.split(".")[-1]
                if ty.startswith("f") or ".f32" in op or ".f64" in op or "x2" in op:
                    regs[ops[0]] = None
                    continue
                srcs = [val(o) for o in ops[1:]]
                if head == "selp":
                    p = regs.get(ops[3])
                    regs[ops[0]] = srcs[0] if p else srcs[1]
                    continue
                if head in ("cvt", "cvta"):
                    regs[ops[0]] = srcs[0]
                    continue
                if any(s is None for s in srcs):
                    regs[ops[0]] = None
                    continue
                bits = 64 if (".wide" in op or _bits(op) == 64) else _bits(op)
                m = (1 << bits) - 1
                a_ = srcs[0]
                b_ = srcs[1] if len(srcs) > 1 else 0
                if head == "add":
                    r = a_ + b_
                elif head == "sub":
                    r = a_ - b_
                elif head == "mul":
                    r = (a_ & _M32) * (b_ & _M32) if ".wide" in op else a_ * b_
                elif head == "mad":
                    r = ((a_ & _M32) * (b_ & _M32) if ".wide" in op else a_ * b_) + srcs[2]
                elif head == "shl":
                    r = a_ << (b_ & 63)
                elif head == "shr":
                    r = ((_signed(a_, bits) if ".s" in op else a_ & m) >> b_)
                elif head == "and":
                    r = a_ & b_
                elif head == "or":
                    r = a_ | b_
                elif head == "xor":
                    r = a_ ^ b_
                elif head in ("div", "rem"):
                    if ".s" in op:
                        sa, sb = _signed(a_, bits), _signed(b_, bits)
                        q = abs(sa) // abs(sb) * (1 if (sa >= 0) == (sb >= 0) else -1)
                        r = q if head == "div" else sa - q * sb
                    else:
                        r = (a_ & m) // (b_ & m) if head == "div" else (a_ & m) % (b_ & m)
                elif head == "min":
                    r = min(a_, b_)
                elif head == "max":
                    r = max(a_, b_)
                elif head == "neg":
                    r = -a_
                else:
                    r = ~a_
                regs[ops[0]] = r & m
                continue
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
