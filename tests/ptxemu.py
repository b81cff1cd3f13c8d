"""A SIMT emulator for the CUDA-core PTX this backend (and the reference emitter) produces.

It runs an entry over a grid on the CPU, one Python object per thread, with global memory held in
NumPy-backed allocations and one shared-memory array per CTA, so the parity tests can compare the
emitted PTX itself with the oracle without a GPU.  Semantics:

* integer, predicate and move instructions as in :func:`tests.ctasim.alu`;
* f32 arithmetic in IEEE single precision with round-to-nearest (``add``/``sub``/``mul``/``div.rn``/
  ``sqrt.rn``/``rcp.rn`` exactly; ``fma`` evaluated in double precision and rounded once more, which
  can differ from a fused result in the last bit on rare ties);
* the MUFU approximations (``ex2``, ``lg2``, ``rsqrt``, ``sin``, ``cos`` ``.approx``) as the exact
  functions rounded to f32 (the hardware's are within a few units in the last place of these);
* threads run independently and meet at warp collectives (``shfl.sync``, ``redux.sync``, ``vote``,
  ``bar.warp.sync``: every lane of the member mask must reach one) and at ``bar.sync`` (every thread
  of the CTA that has not exited); ``red.global`` is atomic because threads run one at a time.

Tensor-core and TMA instructions are not emulated.  It is test infrastructure only.
"""
from __future__ import annotations

import math
import re
import struct

import numpy as np

from emmy_ptx_b200.codegen.ptxcheck import _entries, _instructions
from tests.ctasim import alu

_IMM = re.compile(r"^-?(?:0[xX][0-9a-fA-F]+|\d+)$")
_M32 = (1 << 32) - 1
_M64 = (1 << 64) - 1
_SHARED = re.compile(r"^\.(?:extern\s+)?\.?shared\s+(?:\.align\s+(\d+)\s+)?\.(\w+)\s+([\w$]+)\[(\d*)\];", re.M)


def f2b(x) -> int:
    return struct.unpack("<I", struct.pack("<f", float(np.float32(x))))[0]


def b2f(b: int) -> np.float32:
    return np.frombuffer(struct.pack("<I", b & _M32), dtype=np.float32)[0]


def d2b(x) -> int:
    return struct.unpack("<Q", struct.pack("<d", float(x)))[0]


def b2d(b: int) -> float:
    return struct.unpack("<d", struct.pack("<Q", b & _M64))[0]


def _ftz(x: np.float32) -> np.float32:
    return np.float32(0.0) * np.float32(np.sign(x) if x != 0 else 1.0) if (x != 0 and abs(x) < np.float32(1.1754944e-38)) else x


def _bf16_rn(x: np.float32) -> int:
    b = f2b(x)
    if (b & 0x7F800000) == 0x7F800000 and (b & 0x7FFFFF):
        return ((b >> 16) | 0x40) & 0xFFFF            # quiet NaN
    return ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF


_PH = struct.Struct("<e")
_PU16 = struct.Struct("<H")


def _f16_rn(x) -> int:
    """f16 bits of x, rounded to nearest even; beyond the f16 range: infinity, as cvt.rn does."""
    x = float(x)
    try:
        return _PU16.unpack(_PH.pack(x))[0]
    except OverflowError:
        if x != x:
            return 0x7E00
        # |x| at or above 65520 (the midpoint above 65504) rounds to infinity; below it to 65504
        return (0xFC00 if x < 0 else 0x7C00) if abs(x) >= 65520.0 else (0xFBFF if x < 0 else 0x7BFF)


_PI, _PF = struct.Struct("<I"), struct.Struct("<f")
_FLT_ROUND_UP = 3.4028235677973366e38          # 2^128 - 2^103: the midpoint above the largest float
_TINY = 1.1754943508222875e-38                 # 2^-126


def _bf(b: int) -> float:
    return _PF.unpack(_PI.pack(b & _M32))[0]


def _fb(x: float) -> int:
    """f32 bits of x rounded to nearest even (a double holds every +,-,*,/,sqrt of two floats closely
    enough that this second rounding is exact, p >= 2*24 + 2)."""
    try:
        return _PI.unpack(_PF.pack(x))[0]
    except OverflowError:
        if x != x:
            return 0x7FFFFFFF
        big = abs(x) >= _FLT_ROUND_UP
        return (0xFF800000 if x < 0 else 0x7F800000) if big else (0xFF7FFFFF if x < 0 else 0x7F7FFFFF)


def _flush(x: float) -> float:
    return math.copysign(0.0, x) if x != 0.0 and abs(x) < _TINY else x


def _fdiv(a, b):
    if b == 0.0:
        if a != a or a == 0.0:
            return math.nan
        return math.copysign(math.inf, a) * math.copysign(1.0, b)
    return a / b


def _fsqrt(a):
    return math.nan if a < 0 or a != a else math.sqrt(a)


def _ex2(a):
    try:
        return math.pow(2.0, a)
    except OverflowError:
        return math.inf


def _lg2(a):
    if a != a or a < 0:
        return math.nan
    if a == 0:
        return -math.inf
    return math.log2(a) if a != math.inf else math.inf


def _rsqrt(a):
    if a != a or a < 0:
        return math.nan
    if a == 0:
        return math.copysign(math.inf, a)
    return 1.0 / math.sqrt(a) if a != math.inf else 0.0


def _fmax(*v):
    w = [x for x in v if x == x]
    return max(w) if w else math.nan


def _fmin(*v):
    w = [x for x in v if x == x]
    return min(w) if w else math.nan


_F32 = {"add": lambda a, b: a + b, "sub": lambda a, b: a - b, "mul": lambda a, b: a * b,
        "fma": lambda a, b, c: a * b + c, "mad": lambda a, b, c: a * b + c, "div": _fdiv,
        "neg": lambda a: -a, "abs": abs, "sqrt": _fsqrt, "rcp": lambda a: _fdiv(1.0, a), "rsqrt": _rsqrt,
        "ex2": _ex2, "lg2": _lg2, "max": _fmax, "min": _fmin,
        "sin": lambda a: math.sin(a) if math.isfinite(a) else math.nan,
        "cos": lambda a: math.cos(a) if math.isfinite(a) else math.nan,
        "tanh": math.tanh}


def _classify(o: str):
    """(0, register) | (1, immediate bits) | (2, symbol) for an operand string."""
    o = o.strip()
    if _IMM.match(o):
        return (1, int(o, 0))
    if o.startswith(("0f", "0d")):
        return (1, int(o[2:], 16))
    if o.startswith("%"):
        return (0, o)
    return (2, o)


class Memory:
    """Global memory: NumPy arrays registered at fake device addresses."""

    def __init__(self):
        self.bufs: list[np.ndarray] = []

    def alloc(self, array: np.ndarray) -> int:
        self.bufs.append(np.ascontiguousarray(array).view(np.uint8).reshape(-1).copy())
        return (len(self.bufs)) << 40

    def array(self, addr: int, dtype, shape) -> np.ndarray:
        buf = self.bufs[(addr >> 40) - 1]
        return buf.view(dtype).reshape(shape)

    def _loc(self, addr: int, n: int):
        k, off = (addr >> 40) - 1, addr & ((1 << 40) - 1)
        if k < 0 or k >= len(self.bufs) or off + n > self.bufs[k].size:
            raise IndexError(f"global access of {n} bytes at buffer {k} offset {off} is out of bounds")
        return self.bufs[k], off

    def load(self, addr: int, n: int) -> bytes:
        buf, off = self._loc(addr, n)
        return buf[off:off + n].tobytes()

    def store(self, addr: int, data: bytes) -> None:
        buf, off = self._loc(addr, len(data))
        buf[off:off + len(data)] = np.frombuffer(data, dtype=np.uint8)


_TY = {"f32": (4, "<f"), "b32": (4, "<I"), "u32": (4, "<I"), "s32": (4, "<i"), "f64": (8, "<d"),
       "b64": (8, "<Q"), "u64": (8, "<Q"), "s64": (8, "<q"), "b16": (2, "<H"), "u16": (2, "<H"),
       "s16": (2, "<h"), "f16": (2, "<H"), "bf16": (2, "<H"), "u8": (1, "<B"), "s8": (1, "<b"), "b8": (1, "<B")}


class _Thread:
    __slots__ = ("tid", "lane", "warp", "pc", "regs", "state", "coll")

    def __init__(self, tid, regs):
        self.tid, self.lane, self.warp = tid, tid & 31, tid >> 5
        self.pc, self.regs, self.state, self.coll = 0, regs, "run", None


class Emulator:
    def __init__(self, ptx: str, entry: str):
        self.ptx = ptx
        for name, body in _entries(ptx):
            if name == entry:
                self.ins = _instructions(body)
                break
        else:
            raise KeyError(entry)
        self.labels = {x.label: k for k, x in enumerate(self.ins) if x.label}
        self._dec = [None] * len(self.ins)
        self._opcache: dict = {}
        self._addrcache: dict = {}
        m = re.search(r"\.entry\s+" + re.escape(entry) + r"\s*\(([^)]*)\)", ptx, re.S)
        self.params = re.findall(r"\.param\s+\.\w+\s+([\w$]+)", m.group(1)) if m else []
        self.shared = []
        for al, ty, name, count in _SHARED.findall(ptx):
            elem = _TY[ty][0] if ty in _TY else 1
            self.shared.append((name, int(al) if al else elem, int(count) * elem if count else None))

    def run(self, grid: int, block: int, args: dict, mem: Memory, dyn_smem: int = 0, max_steps: int = 200_000_000):
        """Run the entry: ``args`` maps parameter names (``p_x``) to values (device addresses)."""
        steps = 0
        for cta in range(grid):
            # shared memory of this CTA: static buffers, then the dynamic pool
            smem_size, sym = 0, {}
            for name, al, size in self.shared:
                smem_size = (smem_size + al - 1) // al * al
                sym[name] = smem_size
                smem_size += size if size is not None else dyn_smem
            smem = bytearray(max(smem_size, 16))
            self._cta_begin(cta, smem)
            threads = []
            for t in range(block):
                regs = {"%tid.x": t, "%tid.y": 0, "%tid.z": 0, "%ntid.x": block, "%ntid.y": 1, "%ntid.z": 1,
                        "%ctaid.x": cta, "%ctaid.y": 0, "%ctaid.z": 0, "%nctaid.x": grid, "%nctaid.y": 1,
                        "%nctaid.z": 1, "%laneid": t & 31}
                threads.append(_Thread(t, regs))
            steps += self._run_cta(threads, args, sym, smem, mem, max_steps - steps)

    def _run_cta(self, threads, args, sym, smem, mem, budget) -> int:
        steps = 0
        warps: dict[int, list] = {}
        for th in threads:
            warps.setdefault(th.warp, []).append(th)
        while True:
            progressed = False
            for th in threads:
                if th.state != "run":
                    continue
                n = self._run_thread(th, args, sym, smem, mem)
                steps += n
                progressed = True
                if steps > budget:
                    raise RuntimeError("step budget exceeded")
            live = [t for t in threads if t.state != "done"]
            if not live:
                return steps
            # resolve collectives
            resolved = False
            waiting_bar = [t for t in live if t.state == "bar"]
            if waiting_bar and len(waiting_bar) == len(live):
                self._bar_release(waiting_bar)
                for t in waiting_bar:
                    t.state, t.coll = "run", None
                resolved = True
            for w, lanes in warps.items():
                pend = [t for t in lanes if t.state == "coll"]
                if not pend:
                    continue
                mask = pend[0].coll[1]
                members = [t for t in lanes if (mask >> t.lane) & 1]
                if all(t.state == "coll" for t in members):
                    pcs = {t.pc for t in members}
                    if len(pcs) != 1:
                        raise RuntimeError(f"warp {w}: lanes meet at different collectives {sorted(pcs)}")
                    self._collective(members, args)
                    for t in members:
                        t.state, t.coll = "run", None
                        t.pc += 1
                    resolved = True
                elif any(t.state == "done" for t in members):
                    raise RuntimeError(f"warp {w}: a collective's member lane has exited")
            if not resolved and not any(t.state == "run" for t in live) and self._drain_async():
                continue                               # deferred asynchronous work completed: retry
            if not resolved and not progressed:
                where = sorted({(t.state, self.ins[t.pc].op if t.pc < len(self.ins) else "end") for t in live})
                raise RuntimeError(f"deadlock: {where}")

    # ------------------------------------------------------------------ one thread until it blocks
    def _run_thread(self, th, args, sym, smem, mem) -> int:
        regs = th.regs
        ins = self.ins
        n = 0

        opc = self._opcache

        def val(o):
            c = opc.get(o)
            if c is None:
                c = opc[o] = _classify(o)
            kind, v = c
            if kind == 0:
                return regs.get(v)
            if kind == 1:
                return v
            if v in sym:
                return sym[v]
            if v in args:
                return args[v]
            raise KeyError(v)

        acache = self._addrcache

        def addr(o):
            c = acache.get(o)
            if c is None:
                inner = o.strip()[1:-1].replace(" ", "")
                m = re.match(r"^([%\w$.]+)(?:\+(-?\w+))?$", inner)
                c = acache[o] = (m.group(1), int(m.group(2), 0) if m.group(2) else 0)
            return val(c[0]) + c[1]

        dec = self._dec
        while True:
            if th.pc >= len(ins):
                th.state = "done"
                return n
            x = ins[th.pc]
            n += 1
            if x.label:
                th.pc += 1
                continue
            if x.guard is not None:
                g = regs.get(x.guard)
                if bool(g) == x.neg:
                    th.pc += 1
                    continue
            d = dec[th.pc]
            if d is None:
                d = dec[th.pc] = self._decode(x)
            code = d[0]
            if code == 7:                               # tensor-core / barrier extension
                th.pc += 1
                r = self._extra(th, x, x.op, x.ops, regs, val, addr, smem, mem)
                if r is None:
                    raise NotImplementedError(f"line {x.line}: {x.op}")
                if r == "block":
                    return n
                continue
            if code == 2:                               # integer / predicate / move
                th.pc += 1
                if not alu(x.op, x.ops, regs, val):
                    raise NotImplementedError(f"line {x.line}: {x.op}")
                continue
            if code == 3:
                th.pc += 1
                self._load(x.op, x.ops, regs, addr, smem, mem)
                continue
            if code == 4:
                th.pc += 1
                self._store(x.op, x.ops, regs, addr, val, smem, mem)
                continue
            if code == 5:
                th.pc += 1
                self._cvt(x.op, x.ops, regs, val)
                continue
            if code == 1:                               # f32 arithmetic, decoded once
                fn, dst, srcs, ftz = d[1], d[2], d[3], d[4]
                vals = [_bf(regs[o]) if isinstance(o, str) else o for o in srcs]
                if ftz:
                    vals = [_flush(v) for v in vals]
                r = fn(*vals)
                if ftz:
                    r = _flush(r)
                regs[dst] = _fb(r)
                th.pc += 1
                continue
            op, ops = x.op, x.ops
            if op == "bra" or op.startswith("bra."):
                th.pc = self.labels[ops[-1]]
                continue
            if op in ("ret", "exit"):
                th.state = "done"
                return n
            if (op.startswith("bar.sync") or op.startswith("barrier.sync")) and len(ops) == 1 and val(ops[0]) == 0:
                th.pc += 1
                th.state = "bar"                      # the whole CTA
                return n
            if op.startswith(("shfl.sync", "redux.sync", "vote.sync")):
                th.state, th.coll = "coll", (op, val(ops[-1]) & _M32)
                return n
            if op.startswith("bar.warp.sync"):
                th.state, th.coll = "coll", (op, val(ops[0]) & _M32)
                return n
            th.pc += 1
            if op.startswith("ld.param"):
                regs[ops[0]] = args[ops[1].strip()[1:-1]]
                continue
            if op.startswith(("ld.global", "ld.shared", "ldu.global", "ld.volatile", "ld.acquire", "ld.relaxed")):
                self._load(op, ops, regs, addr, smem, mem)
                continue
            if op.startswith(("st.global", "st.shared", "st.release", "st.relaxed")):
                self._store(op, ops, regs, addr, val, smem, mem)
                continue
            if op.startswith("mov.u64") and ops[1].strip() == "%globaltimer":
                # a nanosecond clock: the emulator's step count, so bounded waits end in emulated time
                regs[ops[0]] = 1000 * n
                continue
            if op.startswith("red.global") or op.startswith("atom.global"):
                self._red(op, ops, regs, addr, val, mem)
                continue
            if op.startswith("cp.async.cg.shared.global") or op.startswith("cp.async.ca.shared.global"):
                dst, src, size = addr(ops[0]) & _M32, addr(ops[1]) & _M64, val(ops[2])
                if dst + size > len(smem):
                    raise IndexError(f"line {x.line}: cp.async to shared offset {dst} past {len(smem)}")
                smem[dst:dst + size] = mem.load(src, size)
                continue
            if op.startswith(("cp.async.commit", "cp.async.wait", "fence", "membar", "griddepcontrol",
                              "prefetch", "setmaxnreg")):
                continue
            r = self._extra(th, x, op, ops, regs, val, addr, smem, mem)
            if r is not None:
                if r == "block":
                    return n
                continue
            try:
                if self._float(op, ops, regs, val):
                    continue
                if op.startswith("cvta"):
                    regs[ops[0]] = val(ops[1])
                    continue
                if alu(op, ops, regs, val):
                    continue
            except (TypeError, ValueError) as e:
                raise RuntimeError(f"thread {th.tid} line {x.line}: {op} {ops}: {e}") from None
            raise NotImplementedError(f"line {x.line}: {op} {ops}")

    # hooks for the tensor-core extension (tests/tcemu.py)
    def _cta_begin(self, cta, smem):
        pass

    def _bar_release(self, threads):
        pass

    def _extra(self, th, x, op, ops, regs, val, addr, smem, mem):
        return None

    def _drain_async(self) -> bool:
        """Complete deferred asynchronous work when no thread can run; True if there was some."""
        return False

    @staticmethod
    def _decode(x):
        """(1, function, destination, sources, ftz) for plain f32 arithmetic; (0,) otherwise.  Sources
        are register names or, for immediates, Python floats."""
        if x.label:
            return (0,)
        op = x.op
        if op.startswith(("mbarrier.", "tcgen05.", "cp.async.bulk", "prmt.", "lop3.", "max.u16x2", "min.u16x2")) or (
                ".f32x2" in op) or (op.startswith(("bar.arrive", "bar.red")) or (
                op.startswith(("bar.sync", "barrier.sync")) and len(x.ops) == 2)):
            return (7,)
        if not x.ops:
            return (0,)
        parts = x.op.split(".")
        if op.startswith(("ld.global", "ld.shared", "ldu.global")):
            return (3,)
        if op.startswith(("st.global", "st.shared")) and not (len(x.ops) == 2 and _IMM.match(x.ops[1].strip())):
            return (4,)
        if parts[0] == "cvt" and parts[-1] in ("f32", "f64", "bf16", "f16") or (parts[0] == "cvt" and parts[-2] in (
                "f32", "f64", "bf16", "f16", "bf16x2", "f16x2")):
            return (5,)
        if (parts[0] in ("add", "sub", "mul", "mad", "shl", "shr", "and", "or", "xor", "div", "rem", "min", "max",
                         "neg", "not", "selp") and parts[-1] in ("s32", "u32", "b32", "s64", "u64", "b64", "pred")
                and not x.ops[0].startswith("{")) or (parts[0] == "setp" and parts[-1][0] in "sub") or (
                op in ("mov.u32", "mov.b32", "mov.u64", "mov.b64", "mov.s32")
                and not x.ops[0].startswith("{") and not x.ops[1].strip().startswith(("{", "0f", "0d", "%globaltimer"))):
            return (2,)
        if parts[-1] != "f32" or parts[0] not in _F32 or x.ops[0].startswith("{"):
            return (0,)
        if any(p_ in ("sat", "rz", "rm", "rp") for p_ in parts[1:-1]):
            return (0,)
        srcs = []
        for o in x.ops[1:]:
            o = o.strip()
            if o.startswith("%"):
                srcs.append(o)
            elif o.startswith("0f"):
                srcs.append(_bf(int(o[2:], 16)))
            else:
                return (0,)
        return (1, _F32[parts[0]], x.ops[0], srcs, "ftz" in parts)

    # ------------------------------------------------------------------ memory
    def _load(self, op, ops, regs, addr, smem, mem):
        parts = op.split(".")
        ty = parts[-1]
        vec = 4 if ".v4" in op else (2 if ".v2" in op else (8 if ".v8" in op else 1))
        size, fmt = _TY[ty]
        a = addr(ops[1])
        if ".shared" in op:
            a &= _M32
            if a + size * vec > len(smem):
                raise IndexError(f"shared load at {a} past {len(smem)}")
            data = bytes(smem[a:a + size * vec])
        else:
            data = mem.load(a & _M64, size * vec)
        dsts = [r.strip() for r in ops[0].strip("{}").split(",")]
        for k, d in enumerate(dsts):
            chunk = data[k * size:(k + 1) * size]
            v = int.from_bytes(chunk, "little")
            if ty in ("s8", "s16"):
                v = v - (1 << (8 * size)) if v >> (8 * size - 1) else v
                v &= _M32
            regs[d] = v

    def _store(self, op, ops, regs, addr, val, smem, mem):
        ty = op.split(".")[-1]
        size, _ = _TY[ty]
        a = addr(ops[0])
        srcs = [s.strip() for s in ops[1].strip("{}").split(",")]
        data = b""
        for s in srcs:
            v = val(s)
            if isinstance(v, bool):
                v = int(v)
            data += (v & ((1 << (8 * size)) - 1)).to_bytes(size, "little")
        if ".shared" in op:
            a &= _M32
            if a + len(data) > len(smem):
                raise IndexError(f"shared store at {a} past {len(smem)}")
            smem[a:a + len(data)] = data
        else:
            mem.store(a & _M64, data)

    def _red(self, op, ops, regs, addr, val, mem):
        ty = op.split(".")[-1]
        a = addr(ops[0] if op.startswith("red") else ops[1])
        v = val(ops[1] if op.startswith("red") else ops[2])
        size, fmt = _TY[ty]
        old = int.from_bytes(mem.load(a, size), "little")
        if ".exch" in op:
            new = v & ((1 << (8 * size)) - 1)
        elif ".add" not in op:
            raise NotImplementedError(op)
        elif ty == "f32":
            new = f2b(b2f(old) + b2f(v))
        else:
            new = (old + v) & ((1 << (8 * size)) - 1)
        mem.store(a, new.to_bytes(size, "little"))
        if op.startswith("atom"):
            regs[ops[0]] = old

    # ------------------------------------------------------------------ floating point
    def _float(self, op, ops, regs, val) -> bool:
        parts = op.split(".")
        head = parts[0]
        ftz = ".ftz" in op
        if head == "cvt":
            return self._cvt(op, ops, regs, val)
        if head == "mov" and not ops[0].startswith("{") and (
                ops[1].strip().startswith(("0f", "0d")) or parts[-1] in ("f32", "f64")):
            regs[ops[0]] = val(ops[1])
            return True
        if op.startswith("mov.b64") and ops[0].startswith("{"):
            v = val(ops[1])
            d0, d1 = [r.strip() for r in ops[0].strip("{}").split(",")]
            regs[d0], regs[d1] = v & _M32, (v >> 32) & _M32
            return True
        if op.startswith("mov.b32") and ops[0].startswith("{"):
            v = val(ops[1])
            d0, d1 = [r.strip() for r in ops[0].strip("{}").split(",")]
            regs[d0], regs[d1] = v & 0xFFFF, (v >> 16) & 0xFFFF
            return True
        if op.startswith("testp.") and parts[-1] in ("f32", "f64"):
            x = self._fv(parts[-1], val(ops[1]))
            tiny = 2.0 ** -126 if parts[-1] == "f32" else 2.0 ** -1022
            fin = math.isfinite(x)
            regs[ops[0]] = {"finite": fin, "infinite": math.isinf(x), "number": not math.isnan(x),
                            "notanumber": math.isnan(x), "normal": fin and abs(x) >= tiny,
                            "subnormal": fin and 0 < abs(x) < tiny}[parts[1]]
            return True
        if op.startswith("setp.") and parts[-1] in ("f32", "f64"):
            a_, b_ = self._fv(parts[-1], val(ops[1])), self._fv(parts[-1], val(ops[2]))
            cmp = parts[1]
            nan = math.isnan(a_) or math.isnan(b_)
            base = cmp.rstrip("u") if cmp not in ("num", "nan") else cmp
            if cmp == "num":
                r = not nan
            elif cmp == "nan":
                r = nan
            elif nan:
                r = cmp.endswith("u")
            else:
                r = {"eq": a_ == b_, "ne": a_ != b_, "lt": a_ < b_, "le": a_ <= b_, "gt": a_ > b_,
                     "ge": a_ >= b_}[base]
            regs[ops[0]] = r
            return True
        if op.startswith("selp.f32") or op.startswith("selp.f64"):
            regs[ops[0]] = val(ops[1]) if regs.get(ops[3]) else val(ops[2])
            return True
        if parts[-1] == "f64" and head in ("add", "sub", "mul", "fma", "div", "neg", "abs", "max", "min"):
            f = [b2d(val(o)) for o in ops[1:]]
            r = {"add": lambda: f[0] + f[1], "sub": lambda: f[0] - f[1], "mul": lambda: f[0] * f[1],
                 "fma": lambda: f[0] * f[1] + f[2], "div": lambda: f[0] / f[1] if f[1] else math.copysign(math.inf, f[0]),
                 "neg": lambda: -f[0], "abs": lambda: abs(f[0]), "max": lambda: max(f), "min": lambda: min(f)}[head]()
            regs[ops[0]] = d2b(r)
            return True
        if parts[-1] != "f32" or head in ("ld", "st", "mov", "shfl", "redux"):
            return False
        f = [b2f(val(o)) for o in ops[1:]]
        if ftz:
            f = [_ftz(v) for v in f]
        with np.errstate(all="ignore"):
            if head == "add":
                r = f[0] + f[1]
            elif head == "sub":
                r = f[0] - f[1]
            elif head == "mul":
                r = f[0] * f[1]
            elif head in ("fma", "mad"):
                r = np.float32(float(f[0]) * float(f[1]) + float(f[2]))
            elif head == "div":
                r = f[0] / f[1]
            elif head == "neg":
                r = -f[0]
            elif head == "abs":
                r = np.abs(f[0])
            elif head in ("max", "min"):
                vals = [v for v in f if not np.isnan(v)]
                r = (np.float32(np.nan) if not vals else (max(vals) if head == "max" else min(vals)))
            elif head == "sqrt":
                r = np.sqrt(f[0])
            elif head == "rcp":
                r = np.float32(1.0) / f[0]
            elif head == "rsqrt":
                r = np.float32(1.0 / math.sqrt(float(f[0]))) if f[0] > 0 else (
                    np.float32(np.inf) if f[0] == 0 else np.float32(np.nan))
            elif head == "ex2":
                r = np.float32(np.exp2(np.float64(f[0])))
            elif head == "lg2":
                r = np.float32(np.log2(np.float64(f[0]))) if f[0] >= 0 else np.float32(np.nan)
            elif head == "sin":
                r = np.float32(np.sin(np.float64(f[0])))
            elif head == "cos":
                r = np.float32(np.cos(np.float64(f[0])))
            elif head == "tanh":
                r = np.float32(np.tanh(np.float64(f[0])))
            elif head == "copysign":
                r = np.copysign(f[1], f[0])
            else:
                return False
        r = np.float32(r)
        if ftz:
            r = _ftz(r)
        regs[ops[0]] = f2b(r)
        return True

    @staticmethod
    def _fv(ty, bits):
        return float(b2f(bits)) if ty == "f32" else b2d(bits)

    def _cvt(self, op, ops, regs, val) -> bool:
        parts = op.split(".")
        dst_t, src_t = parts[-2], parts[-1]
        mode = next((p for p in parts[1:-2] if p in ("rn", "rz", "rm", "rp", "rni", "rzi", "rmi", "rpi")), None)
        sat = "sat" in parts
        v = val(ops[1])
        if dst_t in ("bf16x2", "f16x2"):
            hi, lo = b2f(val(ops[1])), b2f(val(ops[2]))
            rnd = _bf16_rn if dst_t == "bf16x2" else _f16_rn
            regs[ops[0]] = (rnd(hi) << 16) | rnd(lo)
            return True
        # source value as a Python number
        if src_t == "f32":
            x = float(b2f(v))
        elif src_t == "f64":
            x = b2d(v)
        elif src_t == "bf16":
            x = float(b2f((v & 0xFFFF) << 16))
        elif src_t == "f16":
            x = float(np.array([v & 0xFFFF], dtype=np.uint16).view(np.float16)[0])
        elif src_t in ("s32", "s64", "s16", "s8"):
            bits = int(src_t[1:])
            x = v - (1 << bits) if (v >> (bits - 1)) & 1 else v
            x = int(x)
        else:
            x = int(v & ((1 << int(src_t[1:])) - 1)) if src_t[1:].isdigit() else v
        if dst_t == "f32":
            if isinstance(x, int) or src_t == "f64":
                r = np.float32(x) if mode in (None, "rn") else np.float32(x)
            else:
                r = np.float32(x)
                if mode == "rzi":
                    r = np.float32(math.trunc(x)) if math.isfinite(x) else r
                elif mode == "rmi":
                    r = np.float32(math.floor(x)) if math.isfinite(x) else r
                elif mode == "rpi":
                    r = np.float32(math.ceil(x)) if math.isfinite(x) else r
                elif mode == "rni":
                    r = np.float32(np.rint(x)) if math.isfinite(x) else r
            if "ftz" in parts:
                r = _ftz(r)
            regs[ops[0]] = f2b(r)
            return True
        if dst_t == "f64":
            regs[ops[0]] = d2b(float(x))
            return True
        if dst_t in ("bf16", "f16"):
            rnd = _bf16_rn if dst_t == "bf16" else _f16_rn
            regs[ops[0]] = rnd(np.float32(x))
            return True
        if dst_t[0] in "su" and dst_t[1:].isdigit():
            bits = int(dst_t[1:])
            if isinstance(x, float):
                if math.isnan(x):
                    iv = 0
                else:
                    f = {"rzi": math.trunc, "rmi": math.floor, "rpi": math.ceil, "rni": lambda z: int(np.rint(z)),
                         None: math.trunc}[mode](x) if math.isfinite(x) else (1 << 80 if x > 0 else -(1 << 80))
                    iv = int(f)
                lo_, hi_ = (-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if dst_t[0] == "s" else (0, (1 << bits) - 1)
                iv = min(max(iv, lo_), hi_)
            else:
                iv = int(x)
                if sat:
                    lo_, hi_ = (-(1 << (bits - 1)), (1 << (bits - 1)) - 1) if dst_t[0] == "s" else (0, (1 << bits) - 1)
                    iv = min(max(iv, lo_), hi_)
            regs[ops[0]] = iv & ((1 << max(bits, 32)) - 1) if bits <= 32 else iv & _M64
            return True
        return False

    # ------------------------------------------------------------------ warp collectives
    def _collective(self, members, args):
        op = members[0].coll[0]
        ins = self.ins[members[0].pc]
        ops = ins.ops
        by_lane = {t.lane: t for t in members}
        if op.startswith("bar.warp.sync"):
            return

        def val(t, o):
            o = o.strip()
            if _IMM.match(o):
                return int(o, 0)
            if o.startswith("0f"):
                return int(o[2:], 16)
            return t.regs.get(o)
        if op.startswith("shfl.sync"):
            mode = op.split(".")[2]
            dst = ops[0]
            pdst = None
            if "|" in dst:
                dst, pdst = [s.strip() for s in dst.split("|")]
            src = {t.lane: val(t, ops[1]) for t in members}
            out = {}
            for t in members:
                lane = t.lane
                b = val(t, ops[2]) & 31
                c = val(t, ops[3])
                cval, seg = c & 31, (c >> 8) & 31
                maxl = (lane & seg) | (cval & ~seg & 31)
                minl = lane & seg
                if mode == "up":
                    j = lane - b
                    ok = j >= maxl
                elif mode == "down":
                    j = lane + b
                    ok = j <= maxl
                elif mode == "bfly":
                    j = lane ^ b
                    ok = j <= maxl
                else:
                    j = minl | (b & ~seg & 31)
                    ok = j <= maxl
                if not ok or j not in src:
                    j = lane
                out[lane] = (src[j], ok)
            for t in members:
                t.regs[dst] = out[t.lane][0]
                if pdst:
                    t.regs[pdst] = out[t.lane][1]
            return
        if op.startswith("redux.sync"):
            kind, ty = op.split(".")[2], op.split(".")[-1]
            vals = [val(t, ops[1]) for t in members]
            if ty == "f32":
                fv = [float(b2f(v)) for v in vals if not math.isnan(float(b2f(v)))]
                r = f2b(max(fv) if kind == "max" else min(fv)) if fv else 0x7FFFFFFF
            else:
                if ty == "s32":
                    iv = [v - (1 << 32) if v >> 31 else v for v in vals]
                else:
                    iv = list(vals)
                r = {"add": sum, "min": min, "max": max}.get(kind)
                if r is not None:
                    r = r(iv) & _M32
                else:
                    acc = iv[0]
                    for v in iv[1:]:
                        acc = {"and": acc & v, "or": acc | v, "xor": acc ^ v}[kind]
                    r = acc & _M32
            for t in members:
                t.regs[ops[0]] = r
            return
        if op.startswith("vote.sync"):
            kind = op.split(".")[2]
            preds = {t.lane: bool(t.regs.get(ops[1].lstrip("!"))) != ops[1].startswith("!") for t in members}
            if kind == "ballot":
                r = sum(1 << ln for ln, p in preds.items() if p)
            elif kind == "all":
                r = all(preds.values())
            elif kind == "any":
                r = any(preds.values())
            else:
                r = len(set(preds.values())) == 1
            for t in members:
                t.regs[ops[0]] = r
            return
        raise NotImplementedError(op)
