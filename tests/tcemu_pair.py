"""Clusters of two CTAs in the tensor-core emulator: runs the CTA-pair GEMM on the CPU.

:class:`PairEmulator` extends :class:`tests.tcemu.TcEmulator` to a cluster of two CTAs whose threads
are scheduled together, each CTA with its own shared memory, mbarriers and tensor memory:

* ``%cluster_ctarank``, ``%clusterid.x``, ``%nclusterid.x`` (clusters of two along x);
* ``mapa.shared::cluster`` gives a tagged address (bit 31, the target rank in bits 24-27, the offset
  in the target CTA below); an untagged address in a ``shared::cluster`` operand is the issuing
  CTA's own shared memory;
* ``barrier.cluster.arrive`` / ``wait``: a wait returns once every thread of both CTAs has arrived
  in the phase the thread arrived in;
* remote ``mbarrier.arrive``, and TMA loads whose mbarrier is the partner's (``.cta_group::2``): the
  bytes land in the issuing CTA's shared memory and complete the target barrier's transaction
  count (which may go below zero until the target's own ``expect_tx`` arrives, as on the GPU);
* ``tcgen05.mma.cta_group::2.kind::f16``: the 256-row A is 128 rows from each CTA's shared memory at
  the descriptor's offset, the N columns of B are the first half from CTA 0 and the second from CTA
  1, and each CTA's tensor memory receives its own 128 rows of the product;
* ``tcgen05.commit.cta_group::2`` arrives on the addressed CTA's barrier.

With ``defer`` the TMA loads, MMAs and commits are queued and run only when no thread can run, as in
the single-CTA emulator.  Test infrastructure only.
"""
from __future__ import annotations

import random

import numpy as np

from tests.ptxemu import _M32, _Thread
from tests.tcemu import TcEmulator, _MBar

TAG = 1 << 31


class _CThread(_Thread):
    __slots__ = ("rank",)


class _Cta:
    def __init__(self, rank, smem):
        self.rank, self.smem = rank, smem
        self.mbars: dict[int, _MBar] = {}
        self.nbars: dict[int, list] = {}
        self.tmem = np.zeros((128, 512), dtype=np.uint32)
        self.waiters: dict[int, list] = {}


class PairEmulator(TcEmulator):
    def __init__(self, ptx: str, entry: str, tmaps: dict | None = None, defer: bool = False, seed=None):
        # seed: completions in random order and amounts (half the TMA loads land at issue, so a
        # partner's bytes can reach a barrier before its owner's expect_tx; of the rest any subset lands
        # at a time; the tensor core runs a random number of its queued MMAs and commits, in issue
        # order), and the threads stepped in a random order each round
        super().__init__(ptx, entry, tmaps, defer=defer or seed is not None)
        self.rng = random.Random(seed) if seed is not None else None

    def run(self, grid: int, block: int, args: dict, mem, dyn_smem: int = 0, max_steps: int = 400_000_000):
        if grid % 2:
            raise ValueError("clusters of two CTAs need an even grid")
        steps = 0
        for c in range(grid // 2):
            smem_size, sym = 0, {}
            for name, al, size in self.shared:
                smem_size = (smem_size + al - 1) // al * al
                sym[name] = smem_size
                smem_size += size if size is not None else dyn_smem
            self.ctas = [_Cta(r, bytearray(max(smem_size, 16))) for r in range(2)]
            self.queue_tma, self.queue_mma = [], []
            self.cl_phase, self.cl_arrived, self.cl_waiters, self.cl_mine = 0, 0, [], {}
            self.cl_total = 2 * block
            threads = []
            for r in range(2):
                for t in range(block):
                    regs = {"%tid.x": t, "%tid.y": 0, "%tid.z": 0, "%ntid.x": block, "%ntid.y": 1, "%ntid.z": 1,
                            "%ctaid.x": 2 * c + r, "%ctaid.y": 0, "%ctaid.z": 0, "%nctaid.x": grid,
                            "%nctaid.y": 1, "%nctaid.z": 1, "%laneid": t & 31, "%cluster_ctarank": r,
                            "%clusterid.x": c, "%nclusterid.x": grid // 2, "%cluster_nctarank": 2}
                    th = _CThread(t, regs)
                    th.rank = r
                    threads.append(th)
            steps += self._run_cluster(threads, args, sym, mem, max_steps - steps)

    def _use(self, rank):
        st = self.ctas[rank]
        self.rank = rank
        self.smem, self.mbars, self.nbars, self.tmem, self.mbar_waiters = (st.smem, st.mbars, st.nbars, st.tmem,
                                                                            st.waiters)

    def _run_cluster(self, threads, args, sym, mem, budget) -> int:
        steps = 0
        warps: dict[tuple, list] = {}
        for th in threads:
            warps.setdefault((th.rank, th.warp), []).append(th)
        while True:
            progressed = False
            order = list(threads)
            if self.rng is not None:
                self.rng.shuffle(order)
            for th in order:
                if th.state != "run":
                    continue
                self._use(th.rank)
                steps += self._run_thread(th, args, sym, self.ctas[th.rank].smem, mem)
                progressed = True
                if steps > budget:
                    raise RuntimeError("step budget exceeded")
            live = [t for t in threads if t.state != "done"]
            if not live:
                return steps
            resolved = False
            for r in range(2):
                live_r = [t for t in live if t.rank == r]
                waiting = [t for t in live_r if t.state == "bar"]
                if waiting and len(waiting) == len(live_r):
                    self._use(r)
                    self._bar_release(waiting)
                    for t in waiting:
                        t.state, t.coll = "run", None
                    resolved = True
            for key, lanes in warps.items():
                pend = [t for t in lanes if t.state == "coll"]
                if not pend:
                    continue
                mask = pend[0].coll[1]
                members = [t for t in lanes if (mask >> t.lane) & 1]
                if all(t.state == "coll" for t in members):
                    if len({t.pc for t in members}) != 1:
                        raise RuntimeError(f"warp {key}: lanes meet at different collectives")
                    self._collective(members, args)
                    for t in members:
                        t.state, t.coll = "run", None
                        t.pc += 1
                    resolved = True
                elif any(t.state == "done" for t in members):
                    raise RuntimeError(f"warp {key}: a collective's member lane has exited")
            if not resolved and not any(t.state == "run" for t in live) and self._drain_async():
                continue
            if not resolved and not progressed:
                where = sorted({(t.rank, t.state, self.ins[t.pc].op if t.pc < len(self.ins) else "end") for t in live})
                raise RuntimeError(f"deadlock: {where}")

    # ------------------------------------------------------------------ addresses and barriers
    def _target(self, a):
        """(CTA state, local offset) of a shared::cluster address."""
        a &= _M32
        if a & TAG:
            return self.ctas[(a >> 24) & 0xF], a & 0xFFFFFF
        return self.ctas[self.rank], a

    def _arrive_at(self, st, addr, n=1):
        b = st.mbars.get(addr)
        if b is None:
            raise RuntimeError(f"arrive on an uninitialised mbarrier at CTA {st.rank} {addr:#x}")
        b.pending -= n
        if b.pending < 0:
            raise RuntimeError(f"mbarrier at CTA {st.rank} {addr:#x}: more arrivals than its count {b.count}")
        self._settle_at(st, addr, b)

    def _settle_at(self, st, addr, b):
        if b.pending == 0 and b.tx == 0:
            b.phase += 1
            b.pending = b.count
            for t in st.waiters.pop(addr, []):
                t.state = "run"

    def _arrive(self, addr, n=1):
        st, a = self._target(addr)
        self._arrive_at(st, a, n)

    def _complete_tx(self, mb, nbytes):
        st, a = self._target(mb)
        b = st.mbars[a]
        b.tx -= nbytes                     # may go below zero before the owner's expect_tx
        self._settle_at(st, a, b)

    # ------------------------------------------------------------------ instructions
    def _extra(self, th, x, op, ops, regs, val, addr, smem, mem):
        if op.startswith("mapa.shared::cluster"):
            a, r = val(ops[1]) & 0xFFFFFF, val(ops[2])
            regs[ops[0]] = TAG | (r << 24) | a
            return "cont"
        if op.startswith("barrier.cluster.arrive"):
            self.cl_mine[id(th)] = self.cl_phase
            self.cl_arrived += 1
            if self.cl_arrived == self.cl_total:
                self.cl_phase += 1
                self.cl_arrived = 0
                for t in self.cl_waiters:
                    t.state = "run"
                self.cl_waiters = []
            return "cont"
        if op.startswith("barrier.cluster.wait"):
            mine = self.cl_mine.get(id(th))
            if mine is None:
                raise RuntimeError("barrier.cluster.wait without an arrival")
            if self.cl_phase > mine:
                del self.cl_mine[id(th)]
                return "cont"
            th.pc -= 1
            th.state = "cwait"
            self.cl_waiters.append(th)
            return "block"
        if op.startswith("mbarrier.arrive") and "shared::cluster" in op and "expect_tx" not in op:
            self._arrive(addr(ops[1]), val(ops[2]) if len(ops) > 2 else 1)
            return "cont"
        if op.startswith("cp.async.bulk.tensor") and "complete_tx" in op:
            dst, tm, cs, mb = self._tma_args(ops, val, addr)
            if dst & TAG:
                if (dst >> 24) & 0xF != self.rank:
                    raise NotImplementedError("a TMA load into the partner's shared memory")
                dst &= 0xFFFFFF
            mbt = self._abs(mb)
            if self.defer and not (self.rng is not None and self.rng.random() < 0.5):
                self.queue_tma.append((self.rank, dst, tm, cs, mbt, mem))
            else:
                self._tma_write(dst, tm, cs, mbt, smem, mem)
            return "cont"
        if op.startswith("tcgen05.commit"):
            target = self._abs(addr(ops[0]))
            if self.defer:
                self.queue_mma.append(("commit", target))
            else:
                self._arrive(target)
            return "cont"
        if op.startswith("tcgen05.mma") and self.defer:
            self.queue_mma.append(("rank", self.rank))
        return super()._extra(th, x, op, ops, regs, val, addr, smem, mem)

    def _abs(self, a):
        """A shared::cluster address with the issuing CTA made explicit (tagged)."""
        a &= _M32
        return a if a & TAG else TAG | (self.rank << 24) | a

    def _drain_async(self) -> bool:
        if not (self.queue_tma or self.queue_mma):
            return False
        if self.rng is not None and self.queue_tma:
            # any subset of the loads in flight lands now (at least one), the rest later
            k = self.rng.randint(1, len(self.queue_tma))
            pick = set(self.rng.sample(range(len(self.queue_tma)), k))
            tmas = [x for i, x in enumerate(self.queue_tma) if i in pick]
            self.queue_tma = [x for i, x in enumerate(self.queue_tma) if i not in pick]
        else:
            tmas, self.queue_tma = self.queue_tma, []
        for rank, dst, tm, cs, mb, mem in tmas:
            self._use(rank)
            self._tma_write(dst, tm, cs, mb, self.ctas[rank].smem, mem)
        budget = self.rng.randint(1, 8) if self.rng is not None and tmas == [] else None
        woke = False
        while self.queue_mma and not woke and (budget is None or budget > 0):
            if budget is not None:
                budget -= 1
            item = self.queue_mma.pop(0)
            if item[0] == "rank":
                self._use(item[1])
                continue
            if item[0] == "commit":
                before = sum(len(v) for st in self.ctas for v in st.waiters.values())
                self._arrive(item[1])
                woke = sum(len(v) for st in self.ctas for v in st.waiters.values()) < before
                continue
            _, op, ops, snap = item
            regs = dict(snap)
            en = ops[4].strip()
            if en.startswith("%"):
                regs[en] = snap["__acc"]

            def val(o, regs=regs):
                from tests.ptxemu import _IMM
                o = o.strip()
                if _IMM.match(o):
                    return int(o, 0)
                return regs[o]
            self._mma(op, ops, regs, val, self.smem)
        return True

    def _mma(self, op, ops, regs, val, smem):
        if "cta_group::2" not in op:
            return super()._mma(op, ops, regs, val, smem)
        if "kind::f16" not in op or self.rank != 0:
            raise NotImplementedError(f"{op} from CTA {self.rank}")
        d_addr = val(ops[0].strip()[1:-1]) & _M32
        idesc = val(ops[3]) & _M32
        en = ops[4].strip()
        acc = bool(regs.get(en)) if en.startswith("%") else bool(int(en, 0))
        fmt_a, fmt_b = (idesc >> 7) & 7, (idesc >> 10) & 7
        a_mn, b_mn = (idesc >> 15) & 1, (idesc >> 16) & 1
        n = ((idesc >> 17) & 0x3F) << 3
        m = ((idesc >> 24) & 0x1F) << 4
        if fmt_a != fmt_b or fmt_a not in (0, 1) or m != 256:
            raise RuntimeError(f"pair MMA: formats ({fmt_a}, {fmt_b}), M={m}")
        if ops[1].strip().startswith("["):
            raise NotImplementedError("pair MMA with A in tensor memory")
        halves_a = [self._smem_matrix(val(ops[1]), m // 2, 16, bool(a_mn), fmt_a, st.smem) for st in self.ctas]
        halves_b = [self._smem_matrix(val(ops[2]), n // 2, 16, bool(b_mn), fmt_b, st.smem) for st in self.ctas]
        B = np.concatenate(halves_b, axis=0)
        lane0, dcol = (d_addr >> 16) & 0xFFFF, d_addr & 0xFFFF
        for st, A in zip(self.ctas, halves_a):
            prod = A @ B.T
            if acc:
                prod = st.tmem[lane0:lane0 + m // 2, dcol:dcol + n].view(np.float32).astype(np.float64) + prod
            st.tmem[lane0:lane0 + m // 2, dcol:dcol + n] = prod.astype(np.float32).view(np.uint32)
