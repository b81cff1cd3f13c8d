"""A CTA-level simulation of an emitted tensor-core kernel's synchronisation, on the CPU.

One thread stands for each warp (lane 0: the lane every elected role in these kernels uses; the other
roles are warp-uniform).  The threads execute the integer, predicate and branch instructions of the
PTX exactly and share

* shared memory words (``st.shared`` / ``ld.shared``: the TMEM address slot, the per-block flags),
* mbarriers with their arrival counts, transaction bytes and phase parity (``mbarrier.init``,
  ``arrive``, ``arrive.expect_tx``, ``try_wait.parity``),
* named barriers (``bar.sync`` / ``bar.arrive`` / ``barrier.sync``, 32 threads per warp),
* asynchronous completions: a ``cp.async.bulk.tensor`` delivers its box's bytes to its mbarrier, and a
  ``tcgen05.commit`` arrives on its mbarrier, each after a random delay (a thread's commits complete in
  issue order, as the tensor core runs one thread's MMAs in order).

Data (floating-point values, TMA contents, MMA results) is not modelled.  A thread whose
``try_wait`` fails sleeps until that mbarrier changes phase, so a protocol error shows as a deadlock
(no runnable thread and nothing in flight) instead of a time-out.  The scheduler interleaves threads
at random from a seed, so repeated runs explore different orders.

This is test infrastructure: it checks, for every CTA of a small launch, that the producer, MMA and
softmax / epilogue roles hand every barrier phase over and reach the end, which on a GPU could only
be learnt by hanging it.
"""
from __future__ import annotations

import heapq
import random
import re

from emmy_ptx_b200.codegen.ptxcheck import _entries, _instructions

_IMM = re.compile(r"^-?(?:0[xX][0-9a-fA-F]+|\d+)$")
_M32 = (1 << 32) - 1
_DTYPE_BYTES = {"bf16": 2, "f16": 2, "f32": 4, "u8": 1, "i32": 4}


def _signed(v: int, bits: int) -> int:
    v &= (1 << bits) - 1
    return v - (1 << bits) if v >> (bits - 1) else v


def _bits(op: str) -> int:
    m = re.search(r"\.[usb](8|16|32|64)\b", op)
    return int(m.group(1)) if m else 32


def alu(op: str, ops: list, regs: dict, val) -> bool:
    """Execute an integer / predicate / move instruction on ``regs``; False when ``op`` is not one.
    Floating-point results become None (unknown)."""
    head = op.split(".")[0]
    if op.startswith("setp.") and not op.split(".")[-1].startswith("f"):
        parts = op.split(".")
        cmp, ty = parts[1], parts[-1]
        a_, b_ = val(ops[1]), val(ops[2])
        if a_ is None or b_ is None:
            raise ValueError(f"unknown operand: {op} {ops}")
        bits = int(ty[1:])
        if ty[0] == "s":
            a_, b_ = _signed(a_, bits), _signed(b_, bits)
        else:
            a_, b_ = a_ & ((1 << bits) - 1), b_ & ((1 << bits) - 1)
        regs[ops[0]] = {"eq": a_ == b_, "ne": a_ != b_, "lt": a_ < b_, "le": a_ <= b_,
                        "gt": a_ > b_, "ge": a_ >= b_}[cmp]
        return True
    if op in ("and.pred", "or.pred", "xor.pred", "not.pred"):
        if op == "not.pred":
            regs[ops[0]] = not regs.get(ops[1])
        else:
            a_, b_ = bool(regs.get(ops[1])), bool(regs.get(ops[2]))
            regs[ops[0]] = {"and": a_ and b_, "or": a_ or b_, "xor": a_ != b_}[head]
        return True
    if op.startswith(("mov.u32", "mov.b32", "mov.u64", "mov.b64", "mov.s32")) and not ops[0].startswith("{"):
        src = ops[1].strip()
        if src.startswith("{"):
            parts = [val(x) for x in src.strip("{}").split(",")]
            if op.startswith("mov.b64") and len(parts) == 2 and all(isinstance(x, int) for x in parts):
                regs[ops[0]] = (parts[0] & _M32) | ((parts[1] & _M32) << 32)
            else:
                regs[ops[0]] = None
        elif src.startswith(("0f", "0d")):
            regs[ops[0]] = None
        elif re.match(r"^[A-Za-z_$]", src):
            regs[ops[0]] = val(src)
        else:
            regs[ops[0]] = val(src)
        return True
    if head in ("add", "sub", "mul", "mad", "shl", "shr", "and", "or", "xor", "div", "rem", "min",
                "max", "neg", "not", "cvt", "cvta", "selp") and not ops[0].startswith("{"):
        ty = op.split(".")[-1]
        if ty.startswith("f") or ".f32" in op or ".f64" in op or "x2" in op:
            regs[ops[0]] = None
            return True
        srcs = [val(o) for o in ops[1:]]
        if head == "selp":
            regs[ops[0]] = srcs[0] if regs.get(ops[3]) else srcs[1]
            return True
        if head in ("cvt", "cvta"):
            regs[ops[0]] = srcs[0]
            return True
        if any(x is None for x in srcs):
            regs[ops[0]] = None
            return True
        bits = 64 if (".wide" in op or _bits(op) == 64) else _bits(op)
        m = (1 << bits) - 1
        a_, b_ = srcs[0], (srcs[1] if len(srcs) > 1 else 0)
        signed = bool(re.search(r"\.s(8|16|32|64)\b", op))
        if ".wide" in op:
            w = (lambda v: _signed(v, 32)) if signed else (lambda v: v & _M32)
        if head == "add":
            r = a_ + b_
        elif head == "sub":
            r = a_ - b_
        elif head == "mul":
            r = w(a_) * w(b_) if ".wide" in op else a_ * b_
        elif head == "mad":
            r = (w(a_) * w(b_) if ".wide" in op else a_ * b_) + srcs[2]
        elif head == "shl":
            r = a_ << (b_ & 63)
        elif head == "shr":
            r = (_signed(a_, bits) if ".s" in op else a_ & m) >> b_
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
        elif head in ("min", "max"):
            x_, y_ = (_signed(a_, bits), _signed(b_, bits)) if signed else (a_ & m, b_ & m)
            r = min(x_, y_) if head == "min" else max(x_, y_)
        elif head == "neg":
            r = -a_
        else:
            r = ~a_
        regs[ops[0]] = r & m
        return True
    return False


class _MBar:
    __slots__ = ("count", "pending", "tx", "phase")

    def __init__(self, count):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0

    def settle(self) -> bool:
        """Complete the phase when every arrival and transaction byte is in; True if it completed."""
        if self.pending == 0 and self.tx == 0:
            self.phase += 1
            self.pending = self.count
            return True
        return False


class Deadlock(AssertionError):
    pass


class CtaSim:
    """Entry ``name`` of ``ptx`` with its launch record ``rec`` (params, tmaps, block)."""

    def __init__(self, ptx: str, rec: dict, name: str | None = None):
        name = name or rec["entry"]
        for ename, body in _entries(ptx):
            if ename == name:
                self.ins = _instructions(body)
                break
        else:
            raise KeyError(name)
        self.labels = {x.label: k for k, x in enumerate(self.ins) if x.label}
        self.rec = rec
        # every parameter symbol gets a distinct fake address, so a tensor-map operand names its map
        self.symbols: dict[str, int] = {}
        self.tmap_bytes: dict[int, int] = {}
        self.tmap_name: dict[int, str] = {}
        for k, spec in enumerate(rec.get("tmaps", [])):
            addr = 0x7000_0000 + 0x1000 * k
            self.symbols[f"p_{spec['name']}"] = addr
            self.tmap_name[addr] = spec["name"]
            nbytes = _DTYPE_BYTES[spec["dtype"]]
            for b in spec["box"]:
                nbytes *= int(b)
            self.tmap_bytes[addr] = nbytes
        self.warps = int(rec["block"][0]) // 32

    def _addr(self, regs, operand: str) -> int:
        inner = operand.strip()[1:-1]
        m = re.match(r"^(%?[\w$]+)(?:\+(-?\w+))?$", inner.replace(" ", ""))
        if not m:
            raise ValueError(f"address {operand}")
        base = m.group(1)
        b = regs.get(base) if base.startswith("%") else (int(base, 0) if _IMM.match(base) else self.symbols.get(base, 0))
        if b is None:
            raise ValueError(f"unknown address register in {operand}")
        off = int(m.group(2), 0) if m.group(2) else 0
        return b + off

    def run(self, ctaid: int = 0, seed: int = 0, delay=(1, 60), max_steps: int = 20_000_000,
            global_load=None, log_tma: bool = False) -> dict:
        """Simulate one CTA.  Returns ``{"errors": [...], "steps": n, "stores": [(warp, address)],
        "tma": [(warp, map name, coordinates)] or None}``: error codes written, global stores (from
        address 0 for every pointer parameter) and, with ``log_tma``, every TMA load issued.  Raises
        :class:`Deadlock` with each waiting thread's position when nothing can run."""
        rng = random.Random(seed)
        smem: dict[int, int] = {}
        mbars: dict[int, _MBar] = {}
        named: dict[int, list] = {}          # id -> [arrived threads, [waiting warp ids], count]
        inflight: list = []                  # (time, seq, kind, addr, amount)
        last_commit: dict[int, int] = {}
        threads = []
        for w in range(self.warps):
            regs = {"%tid.x": 32 * w, "%ctaid.x": ctaid, "%ntid.x": 32 * self.warps, "%smid": 0,
                    "%laneid": 0, "%nctaid.x": int(self.rec["grid"][0])}
            threads.append({"w": w, "pc": 0, "regs": regs, "state": "run", "on": None})
        errors = []
        stores = []
        tma_log = [] if log_tma else None
        now = 0
        seq = 0
        steps = 0
        nthreads_total = 32 * self.warps

        def val_for(regs):
            def val(o):
                o = o.strip()
                if _IMM.match(o):
                    return int(o, 0)
                if o.startswith("%"):
                    return regs.get(o)
                if o in self.symbols:
                    return self.symbols[o]
                if re.match(r"^[A-Za-z_$]", o):
                    return 0                 # a shared-memory symbol: offsets are taken from 0
                return None
            return val

        def wake_mbar(addr):
            for t in threads:
                if t["state"] == "mbar" and t["on"] == addr:
                    t["state"] = "run"

        def arrive(addr, n=1):
            b = mbars.get(addr)
            if b is None:
                raise AssertionError(f"arrive on uninitialised mbarrier at {addr:#x}")
            b.pending -= n
            if b.pending < 0:
                raise AssertionError(f"mbarrier at {addr:#x}: more arrivals than its count {b.count}")
            if b.settle():
                wake_mbar(addr)

        def schedule(kind, addr, amount, thread_w=None):
            nonlocal seq
            t = now + rng.randint(*delay)
            if kind == "commit":
                t = max(t, last_commit.get(thread_w, 0) + 1)
                last_commit[thread_w] = t
            seq += 1
            heapq.heappush(inflight, (t, seq, kind, addr, amount))

        while True:
            runnable = [t for t in threads if t["state"] == "run"]
            if not runnable:
                if inflight:
                    t_, _, kind, addr, amount = heapq.heappop(inflight)
                    now = max(now, t_)
                    b = mbars[addr]
                    if kind == "tx":
                        b.tx -= amount
                        if b.tx < 0:
                            raise AssertionError(f"mbarrier at {addr:#x}: more bytes delivered than expected")
                    else:
                        b.pending -= 1
                        if b.pending < 0:
                            raise AssertionError(f"mbarrier at {addr:#x}: commit arrival over its count")
                    if b.settle():
                        wake_mbar(addr)
                    continue
                if all(t["state"] == "done" for t in threads):
                    return {"errors": errors, "steps": steps, "stores": stores, "tma": tma_log}
                where = [(t["w"], t["state"], t["on"], t.get("par") if t["state"] == "mbar" else None,
                          self.ins[t["pc"]].line) for t in threads if t["state"] != "done"]
                raise Deadlock(f"CTA {ctaid}: no thread can run: {where}")
            # deliver completions that are due
            while inflight and inflight[0][0] <= now:
                t_, _, kind, addr, amount = heapq.heappop(inflight)
                b = mbars[addr]
                if kind == "tx":
                    b.tx -= amount
                else:
                    b.pending -= 1
                if b.settle():
                    wake_mbar(addr)
            th = rng.choice(runnable)
            now += 1
            steps += 1
            if steps > max_steps:
                raise AssertionError(f"CTA {ctaid}: more than {max_steps} steps")
            regs = th["regs"]
            val = val_for(regs)
            x = self.ins[th["pc"]]
            th["pc"] += 1
            if x.label:
                continue
            if x.guard is not None:
                g = regs.get(x.guard)
                if g is None:
                    raise ValueError(f"guard {x.guard} unknown at line {x.line}: {x.op}")
                if bool(g) == x.neg:
                    continue
            op, ops = x.op, x.ops
            if op == "bra" or op.startswith("bra."):
                th["pc"] = self.labels[ops[-1]]
                continue
            if op in ("ret", "exit"):
                th["state"] = "done"
                continue
            if op.startswith("mbarrier.init"):
                mbars[self._addr(regs, ops[0])] = _MBar(val(ops[1]))
                continue
            if op.startswith("mbarrier.try_wait") or op.startswith("mbarrier.test_wait"):
                addr = self._addr(regs, ops[1])
                b = mbars.get(addr)
                if b is None:
                    raise AssertionError(f"wait on uninitialised mbarrier at {addr:#x}")
                par = val(ops[2]) & 1
                if (b.phase & 1) != par:          # the phase of that parity has completed
                    regs[ops[0]] = True
                else:
                    th["pc"] -= 1                 # sleep on the barrier and retry the wait
                    th["state"], th["on"] = "mbar", addr
                    th["par"] = (par, b.phase)
                continue
            if op.startswith("mbarrier.arrive.expect_tx"):
                addr = self._addr(regs, ops[1])
                mbars[addr].tx += val(ops[2])
                arrive(addr)
                continue
            if op.startswith("mbarrier.arrive"):
                n = val(ops[2]) if len(ops) > 2 else 1
                arrive(self._addr(regs, ops[1]), n)
                continue
            if op.startswith("mbarrier.expect_tx"):
                mbars[self._addr(regs, ops[0])].tx += val(ops[1])
                continue
            if op.startswith("cp.async.bulk.tensor") and "complete_tx" in op:
                tmap = self._addr(regs, "[" + ops[1].strip()[1:].split(",")[0] + "]")
                if tmap not in self.tmap_bytes:
                    raise AssertionError(f"TMA with an unknown tensor map at line {x.line}")
                schedule("tx", self._addr(regs, ops[2]), self.tmap_bytes[tmap])
                if tma_log is not None:
                    coords = ops[1].strip()[1:-1].split(",", 1)[1]
                    cs = tuple(val(c) for c in coords.strip().strip("{}").split(","))
                    tma_log.append((th["w"], self.tmap_name.get(tmap), cs, self._addr(regs, ops[0])))
                continue
            if op.startswith("tcgen05.commit"):
                schedule("commit", self._addr(regs, ops[0]), 1, th["w"])
                continue
            if op.startswith("tcgen05.alloc"):
                smem[self._addr(regs, ops[0])] = 0
                continue
            if op.startswith(("bar.sync", "bar.arrive", "barrier.sync", "barrier.arrive")) and not op.startswith("bar.warp"):
                bid = val(ops[0])
                cnt = val(ops[1]) if len(ops) > 1 else nthreads_total
                st = named.setdefault(bid, [0, [], cnt])
                if st[0] == 0:
                    st[2] = cnt
                elif st[2] != cnt:
                    raise AssertionError(f"named barrier {bid}: counts {st[2]} and {cnt} in one phase")
                st[0] += 32
                sync = ".sync" in op or op == "barrier.sync" or op.startswith("barrier.sync")
                if sync:
                    th["state"], th["on"] = "bar", bid
                    st[1].append(th)
                if st[0] >= st[2]:
                    if st[0] > st[2]:
                        raise AssertionError(f"named barrier {bid}: {st[0]} arrivals for a count of {st[2]}")
                    for t in st[1]:
                        t["state"], t["on"] = "run", None
                    named[bid] = [0, [], cnt]
                continue
            if op.startswith("st.shared"):
                smem[self._addr(regs, ops[0])] = val(ops[1])
                continue
            if op.startswith("ld.shared"):
                regs[ops[0]] = smem.get(self._addr(regs, ops[1]), 0)
                continue
            if op.startswith("ld.global") or op.startswith("ld.param"):
                v = 0 if global_load is None or op.startswith("ld.param") else global_load(x, regs)
                if ops[0].startswith("{"):
                    for r in ops[0].strip("{}").split(","):
                        regs[r.strip()] = v
                else:
                    regs[ops[0]] = v
                continue
            if op.startswith("st.global") and len(ops) == 2 and _IMM.match(ops[1].strip()):
                errors.append(int(ops[1], 0))
                continue
            if op.startswith("st.global"):
                stores.append((th["w"], self._addr(regs, ops[0])))
                continue

            if op.startswith("vote.sync.ballot"):
                regs[ops[0]] = _M32 if regs.get(ops[1]) else 0     # every lane of the warp agrees
                continue
            if op.startswith("vote.sync"):
                regs[ops[0]] = bool(regs.get(ops[1]))
                continue
            if op.startswith("setp.") and op.split(".")[-1].startswith("f"):
                regs[ops[0]] = False
                continue
            if alu(op, ops, regs, val):
                continue
            if ops and not op.startswith(("st.", "tcgen05.st", "tcgen05.mma", "cp.", "fence", "red.",
                                          "bar.warp", "tcgen05.wait", "tcgen05.fence", "tcgen05.dealloc",
                                          "tcgen05.relinquish", "griddepcontrol", "prefetch")):
                d = ops[0]
                if d.startswith("{"):
                    for r in d.strip("{}").split(","):
                        regs[r.strip()] = None
                elif d.startswith("%"):
                    regs[d] = None
