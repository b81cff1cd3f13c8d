"""Tensor-core extension of the SIMT emulator: runs the tcgen05 / TMA kernels on the CPU.

On top of :class:`tests.ptxemu.Emulator` it models, per CTA:

* mbarriers (arrival count, transaction bytes, phase; ``try_wait.parity`` blocks the thread until the
  awaited phase has completed) and counted named barriers (``bar.sync`` / ``bar.arrive`` with a count;
  ``bar.red.or.pred`` across the CTA);
* TMA tile loads (``cp.async.bulk.tensor``): the box is read from global memory through the tensor
  map the launch record describes, written to shared memory with the 128-byte swizzle (16-byte chunk
  index XOR row mod 8 within each 1024-byte atom), zero-filled outside the tensor, and its bytes
  complete the mbarrier's transaction count at once;
* tensor memory (128 lanes x 512 columns of 32 bits), ``tcgen05.alloc`` (base address 0),
  ``tcgen05.ld`` / ``st`` (``32x32b``: warp w reaches lanes 32*(w%4) onwards through the address's lane
  field), and ``tcgen05.mma.cta_group::1.kind::f16``: A from a shared-memory matrix descriptor or from
  tensor memory (two 16-bit values per column), B from a descriptor, both decoded from the start
  address, leading / stride byte offsets and the 128-byte swizzle as the kernels encode them; the
  product is accumulated in f32 (as float64 sums rounded to f32 per MMA) into the D columns;
* ``tcgen05.commit`` arrives on its mbarrier as soon as it runs (the MMAs complete synchronously).

Because everything asynchronous completes at issue, this checks the data path and the hand-overs
of one legal order; :mod:`tests.ctasim` explores other orders of the same synchronisation.
It is test infrastructure only.
"""
from __future__ import annotations

import numpy as np

from tests.ptxemu import Emulator, _M32, _bf, _fb, _IMM
from tests.ctasim import _DTYPE_BYTES

class _MBar:
    __slots__ = ("count", "pending", "tx", "phase")

    def __init__(self, count):
        self.count, self.pending, self.tx, self.phase = count, count, 0, 0


def _halves_to_float(bits: np.ndarray, fmt: int) -> np.ndarray:
    """16-bit patterns (uint16 array) as float64: fmt 1 bf16, 0 f16."""
    bits = bits.astype(np.uint16)
    if fmt == 1:
        return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return bits.view(np.float16).astype(np.float64)


class TcEmulator(Emulator):
    """``tmaps``: parameter name (``p_tmQ``) -> (global address of the tensor, tensor-map spec)."""

    def __init__(self, ptx: str, entry: str, tmaps: dict | None = None, defer: bool = False):
        super().__init__(ptx, entry)
        # defer: TMA loads, MMAs and commits are queued and run only when no thread can run, TMA
        # writes first, then the MMAs and commits in issue order.  Anything the barrier protocol does
        # not order (an MMA reading a stage a later load overwrites, a load of data whose barrier was not
        # waited on) then reads the wrong data and shows in the result.
        self.defer = defer
        self.tmaps_by_param = tmaps or {}
        self.fake = {}
        for k, (pname, (gaddr, spec)) in enumerate(self.tmaps_by_param.items()):
            self.fake[0x7E00_0000_0000 + 0x1000 * k] = (gaddr, spec)

    def tmap_args(self) -> dict:
        return {pname: 0x7E00_0000_0000 + 0x1000 * k for k, pname in enumerate(self.tmaps_by_param)}

    # ------------------------------------------------------------------ per-CTA state
    def _cta_begin(self, cta, smem):
        self.smem = smem
        self.queue_tma: list = []
        self.queue_mma: list = []
        self.mbars: dict[int, _MBar] = {}
        self.nbars: dict[int, list] = {}
        self.tmem = np.zeros((128, 512), dtype=np.uint32)
        self.mbar_waiters: dict[int, list] = {}

    def _bar_release(self, threads):
        red = [t for t in threads if t.coll and t.coll[0] == "bar.red.or"]
        if red:
            r = any(t.coll[1] for t in red)
            for t in red:
                t.regs[t.coll[2]] = r

    def _arrive(self, addr, n=1):
        b = self.mbars.get(addr)
        if b is None:
            raise RuntimeError(f"arrive on an uninitialised mbarrier at {addr:#x}")
        b.pending -= n
        if b.pending < 0:
            raise RuntimeError(f"mbarrier at {addr:#x}: more arrivals than its count {b.count}")
        self._settle(addr, b)

    def _settle(self, addr, b):
        if b.pending == 0 and b.tx == 0:
            b.phase += 1
            b.pending = b.count
            for t in self.mbar_waiters.pop(addr, []):
                t.state = "run"

    # ------------------------------------------------------------------ instructions
    def _extra(self, th, x, op, ops, regs, val, addr, smem, mem):
        if ".f32x2" in op:
            head = op.split(".")[0]
            if head in ("fma", "add", "mul", "sub"):
                vs = [val(o) for o in ops[1:]]
                out = 0
                for h in range(2):
                    f = [_bf((v >> (32 * h)) & _M32) for v in vs]
                    r = (f[0] * f[1] + f[2] if head == "fma" else f[0] + f[1] if head == "add"
                         else f[0] * f[1] if head == "mul" else f[0] - f[1])
                    out |= _fb(r) << (32 * h)
                regs[ops[0]] = out
                return "cont"
        if op.startswith("tcgen05.ld"):
            self._tmem_ld(th, op, ops, regs, addr)
            return "cont"
        if op.startswith("tcgen05.st"):
            self._tmem_st(th, op, ops, regs, addr, val)
            return "cont"
        if op.startswith("mbarrier.init"):
            self.mbars[addr(ops[0]) & _M32] = _MBar(val(ops[1]))
            return "cont"
        if op.startswith("mbarrier.try_wait") or op.startswith("mbarrier.test_wait"):
            a = addr(ops[1]) & _M32
            b = self.mbars.get(a)
            if b is None:
                raise RuntimeError(f"wait on an uninitialised mbarrier at {a:#x}")
            if (b.phase & 1) != (val(ops[2]) & 1):
                regs[ops[0]] = True
                return "cont"
            th.pc -= 1                                   # retry when the barrier moves on
            th.state = "mbar"
            self.mbar_waiters.setdefault(a, []).append(th)
            return "block"
        if op.startswith("mbarrier.expect_tx"):
            a = addr(ops[0]) & _M32
            self.mbars[a].tx += val(ops[1])
            return "cont"
        if op.startswith("mbarrier.arrive.expect_tx"):
            a = addr(ops[1]) & _M32
            self.mbars[a].tx += val(ops[2])
            self._arrive(a)
            return "cont"
        if op.startswith("mbarrier.arrive"):
            self._arrive(addr(ops[1]) & _M32, val(ops[2]) if len(ops) > 2 else 1)
            return "cont"
        if op.startswith(("bar.sync", "barrier.sync", "bar.arrive", "barrier.arrive")):
            bid = val(ops[0])
            cnt = val(ops[1])
            st = self.nbars.setdefault(bid, [0, []])
            st[0] += 1
            if ".sync" in op:
                th.state = "nbar"
                st[1].append(th)
            if st[0] == cnt:
                for t in st[1]:
                    t.state = "run"
                self.nbars[bid] = [0, []]
            elif st[0] > cnt:
                raise RuntimeError(f"named barrier {bid}: {st[0]} arrivals for a count of {cnt}")
            return "block" if th.state == "nbar" else "cont"
        if op.startswith("bar.red.or.pred"):
            th.state = "bar"
            th.coll = ("bar.red.or", bool(regs.get(ops[2])), ops[0])
            return "block"
        if op.startswith("cp.async.bulk.tensor") and "complete_tx" in op:
            if self.defer:
                dst, tm, cs, mb = self._tma_args(ops, val, addr)
                self.queue_tma.append((dst, tm, cs, mb, mem))
            else:
                self._tma_load(ops, regs, val, addr, smem, mem)
            return "cont"
        if op.startswith("cp.async.bulk.prefetch"):
            return "cont"
        if op.startswith("tcgen05.alloc"):
            a = addr(ops[0]) & _M32
            smem[a:a + 4] = (0).to_bytes(4, "little")
            return "cont"
        if op.startswith(("tcgen05.relinquish", "tcgen05.dealloc", "tcgen05.fence", "tcgen05.wait")):
            return "cont"
        if op.startswith("tcgen05.commit"):
            if self.defer:
                self.queue_mma.append(("commit", addr(ops[0]) & _M32))
            else:
                self._arrive(addr(ops[0]) & _M32)
            return "cont"
        if op.startswith("tcgen05.mma"):
            if self.defer:
                # operands evaluated now (as the instruction reads its registers at issue)
                snap = {o.strip(): val(o.strip()) for o in ops if o.strip().startswith("%")}
                for o in ops:
                    o = o.strip()
                    if o.startswith("[") and "%" in o:
                        r = o[1:-1].split("+")[0].strip()
                        snap[r] = val(r)
                en = ops[4].strip()
                snap["__acc"] = bool(regs.get(en)) if en.startswith("%") else bool(int(en, 0))
                self.queue_mma.append(("mma", op, list(ops), snap))
            else:
                self._mma(op, ops, regs, val, smem)
            return "cont"
        if op.startswith("tcgen05.ld"):
            self._tmem_ld(th, op, ops, regs, addr)
            return "cont"
        if op.startswith("tcgen05.st"):
            self._tmem_st(th, op, ops, regs, addr, val)
            return "cont"
        if op.startswith("prmt.b32"):
            a_, b_, sel = val(ops[1]) & _M32, val(ops[2]) & _M32, val(ops[3])
            src = (a_ | (b_ << 32)).to_bytes(8, "little")
            regs[ops[0]] = int.from_bytes(bytes(src[(sel >> (4 * i)) & 7] for i in range(4)), "little")
            return "cont"
        if op.startswith("lop3.b32"):
            # d = LUT(a, b, c) bitwise: bit i of the immediate is the result for (a, b, c) = bits of i
            a_, b_, c_, lut = (val(o) & _M32 for o in ops[1:5])
            r = 0
            for i in range(8):
                if lut >> i & 1:
                    r |= ((a_ if i & 4 else ~a_) & (b_ if i & 2 else ~b_) & (c_ if i & 1 else ~c_)) & _M32
            regs[ops[0]] = r
            return "cont"
        if op.startswith("max.u16x2") or op.startswith("min.u16x2"):
            a_, b_ = val(ops[1]) & _M32, val(ops[2]) & _M32
            f = max if op.startswith("max") else min
            regs[ops[0]] = f(a_ & 0xFFFF, b_ & 0xFFFF) | (f(a_ >> 16, b_ >> 16) << 16)
            return "cont"
        if ".f32x2" in op and op.split(".")[0] in ("fma", "add", "mul", "sub"):
            head = op.split(".")[0]
            vs = [val(o) for o in ops[1:]]
            out = 0
            for h in range(2):
                f = [_bf((v >> (32 * h)) & _M32) for v in vs]
                r = {"fma": lambda: f[0] * f[1] + f[2], "add": lambda: f[0] + f[1],
                     "mul": lambda: f[0] * f[1], "sub": lambda: f[0] - f[1]}[head]()
                out |= _fb(r) << (32 * h)
            regs[ops[0]] = out
            return "cont"
        if op.startswith("mov.u64") and not ops[1].strip().startswith("%") and not _IMM.match(ops[1].strip()):
            regs[ops[0]] = val(ops[1])
            return "cont"
        return None

    def _drain_async(self) -> bool:
        if not (self.queue_tma or self.queue_mma):
            return False
        tmas, self.queue_tma = self.queue_tma, []
        for dst, tm, cs, mb, mem in tmas:
            self._tma_write(dst, tm, cs, mb, self.smem, mem)
        # the tensor core then advances only until some thread can run again, so work that the barrier
        # protocol lets other threads overtake stays pending as long as possible
        woke = [False]
        while self.queue_mma and not woke[0]:
            item = self.queue_mma.pop(0)
            if item[0] == "commit":
                before = sum(len(v) for v in self.mbar_waiters.values())
                self._arrive(item[1])
                woke[0] = sum(len(v) for v in self.mbar_waiters.values()) < before
            else:
                _, op, ops, snap = item
                regs = dict(snap)
                en = ops[4].strip()
                if en.startswith("%"):
                    regs[en] = snap["__acc"]

                def val(o, regs=regs):
                    o = o.strip()
                    if _IMM.match(o):
                        return int(o, 0)
                    return regs[o]
                self._mma(op, ops, regs, val, self.smem)
        return True

    # ------------------------------------------------------------------ TMA
    def _tma_args(self, ops, val, addr):
        dst = addr(ops[0]) & _M32
        inner = ops[1].strip()[1:-1]
        tm_op, coords = inner.split(",", 1)
        tm = val(tm_op.strip())
        cs = [val(c) for c in coords.strip().strip("{}").split(",")]
        return dst, tm, cs, addr(ops[2]) & _M32

    def _tma_load(self, ops, regs, val, addr, smem, mem):
        dst, tm, cs, mb = self._tma_args(ops, val, addr)
        self._tma_write(dst, tm, cs, mb, smem, mem)

    def _tma_write(self, dst, tm, cs, mb, smem, mem):
        gaddr, spec = self.fake[tm]
        es = _DTYPE_BYTES[spec["dtype"]]
        box = [int(b) for b in spec["box"]]
        dims = [int(d) for d in spec["dims"]]
        strides = [es] + [int(s_) for s_ in spec["strides"]]
        row_bytes = box[0] * es
        nrows = 1
        for b in box[1:]:
            nrows *= b
        out = bytearray(row_bytes * nrows)
        buf = mem.array(gaddr, np.uint8, (-1,))
        off0 = gaddr & ((1 << 40) - 1)
        r = 0
        import itertools
        for idx in itertools.product(*[range(b) for b in reversed(box[1:])]):
            outer = list(reversed(idx))                  # box coordinates of dims 1..
            pos = [cs[0]] + [cs[1 + i] + outer[i] for i in range(len(outer))]
            if all(0 <= pos[d] < dims[d] for d in range(1, len(dims))):
                base = sum(pos[d] * strides[d] for d in range(1, len(dims)))
                lo = max(0, pos[0])
                hi = min(dims[0], pos[0] + box[0])
                if hi > lo:
                    seg = buf[off0 + base + lo * es: off0 + base + hi * es]
                    out[r * row_bytes + (lo - pos[0]) * es: r * row_bytes + (hi - pos[0]) * es] = seg.tobytes()
            r += 1
        sw = spec.get("swizzle", "128B")
        for off in range(0, len(out), 16):
            a = dst + off
            if sw == "128B":
                a ^= ((a >> 7) & 7) << 4
            elif sw == "64B":
                a ^= ((a >> 7) & 3) << 4
            if a + 16 > len(smem):
                raise IndexError(f"TMA box past shared memory ({a})")
            smem[a:a + 16] = out[off:off + 16]
        self._complete_tx(mb, len(out))

    def _complete_tx(self, mb, nbytes):
        b = self.mbars[mb]
        b.tx -= nbytes
        if b.tx < 0:
            raise RuntimeError("TMA delivered more bytes than the mbarrier expects")
        self._settle(mb, b)

    # ------------------------------------------------------------------ tensor memory
    def _tmem_lane_col(self, th, a):
        lane = (a >> 16) & 0xFFFF
        col = a & 0xFFFF
        return lane + th.lane, col

    def _tmem_ld(self, th, op, ops, regs, addr):
        a = addr(ops[1]) & _M32
        lane, col = self._tmem_lane_col(th, a)
        dsts = [r.strip() for r in ops[0].strip("{}").split(",")]
        for k, d in enumerate(dsts):
            regs[d] = int(self.tmem[lane, col + k])

    def _tmem_st(self, th, op, ops, regs, addr, val):
        a = addr(ops[0]) & _M32
        lane, col = self._tmem_lane_col(th, a)
        srcs = [r.strip() for r in ops[1].strip("{}").split(",")]
        for k, s_ in enumerate(srcs):
            self.tmem[lane, col + k] = val(s_) & _M32

    # ------------------------------------------------------------------ MMA
    @staticmethod
    def _sw(a: np.ndarray) -> np.ndarray:
        return a ^ (((a >> 7) & 7) << 4)

    def _smem_matrix(self, desc: int, rows: int, k: int, mn_major: bool, fmt: int, smem) -> np.ndarray:
        """rows x k (M or N by K) operand from a SWIZZLE_128B descriptor, as float64."""
        start = (desc & 0x3FFF) << 4
        lbo = ((desc >> 16) & 0x3FFF) << 4
        sbo = ((desc >> 32) & 0x3FFF) << 4
        layout = (desc >> 61) & 7
        if layout not in (2, 4):
            raise NotImplementedError("only the 128- and 64-byte swizzles are emulated")
        span = 128 if layout == 2 else 64        # bytes of one swizzled row
        i = np.arange(rows)[:, None]
        kk = np.arange(k)[None, :]
        if not mn_major:
            a = start + (i // 8) * sbo + (i % 8) * span + kk * 2
        else:
            per = span // 2
            a = start + (i // per) * lbo + (kk // 8) * sbo + (kk % 8) * span + (i % per) * 2
        a = a.astype(np.int64)
        a = self._sw(a) if layout == 2 else a ^ (((a >> 7) & 3) << 4)
        sm = np.frombuffer(bytes(smem), dtype=np.uint8)
        bits = sm[a].astype(np.uint16) | (sm[a + 1].astype(np.uint16) << 8)
        return _halves_to_float(bits, fmt)

    def _mma(self, op, ops, regs, val, smem):
        if "kind::f16" not in op or "cta_group::1" not in op:
            raise NotImplementedError(op)
        d_addr = val(ops[0].strip()[1:-1]) & _M32
        idesc = val(ops[3]) & _M32
        en = ops[4].strip()
        acc = bool(regs.get(en)) if en.startswith("%") else bool(int(en, 0))
        fmt_a, fmt_b = (idesc >> 7) & 7, (idesc >> 10) & 7
        a_mn, b_mn = (idesc >> 15) & 1, (idesc >> 16) & 1
        n = ((idesc >> 17) & 0x3F) << 3
        m = ((idesc >> 24) & 0x1F) << 4
        if fmt_a != fmt_b or fmt_a not in (0, 1):
            raise RuntimeError(f"A and B formats differ or are not f16/bf16 ({fmt_a}, {fmt_b})")
        a_op = ops[1].strip()
        if a_op.startswith("["):
            ta = val(a_op[1:-1].split("+")[0].strip()) + (int(a_op[1:-1].split("+")[1], 0) if "+" in a_op else 0)
            lane0, col = (ta >> 16) & 0xFFFF, ta & 0xFFFF
            words = self.tmem[lane0:lane0 + m, col:col + 8]                 # K=16: 8 columns of two
            bits = np.stack([words & 0xFFFF, words >> 16], axis=-1).reshape(m, 16)
            A = _halves_to_float(bits, fmt_a)
        else:
            A = self._smem_matrix(val(a_op), m, 16, bool(a_mn), fmt_a, smem)
        B = self._smem_matrix(val(ops[2]), n, 16, bool(b_mn), fmt_b, smem)
        lane0, dcol = (d_addr >> 16) & 0xFFFF, d_addr & 0xFFFF
        prod = A @ B.T
        if acc:
            prev = self.tmem[lane0:lane0 + m, dcol:dcol + n].view(np.float32).astype(np.float64)
            prod = prev + prod
        self.tmem[lane0:lane0 + m, dcol:dcol + n] = prod.astype(np.float32).view(np.uint32)
