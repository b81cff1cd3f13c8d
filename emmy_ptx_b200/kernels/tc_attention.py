"""Causal / full attention on the 5th-generation tensor cores: QK^T and PV with tcgen05, S, P and O in TMEM.

O = softmax(Q K^T * scale [+ causal mask]) V for Q, K, V, O bf16 [batch, heads, S, 128] — the online-softmax
Accum loop nest of the attention IR (config 5).  One CTA owns 256 query rows of one (batch, head) as two
128-row tiles that take turns on the tensor core:

* warp 0 issues TMA: both Q tiles once, then K_0, V_0, K_1, V_1, ... through a 4-stage ring of 32 KiB;
* warp 1 owns TMEM (512 columns: S_0, S_1, O_0, O_1, 128 each) and issues, from one thread,
  S_i = Q_i K_j^T (M=128, N=128, K=128 as 8 MMAs, both operands K-major in shared memory) and
  O_i += P_i V_j with P_i read from TMEM (V MN-major in shared memory), in the order
  PV_0(j), S_0(j+1), PV_1(j), S_1(j+1): the tensor core runs one tile while the other is in softmax;
* warps 4-7 (tile 0) and 8-11 (tile 1) run the online softmax, one thread per row: load the row of S
  from TMEM, mask the diagonal block, take the row max, compute p = 2^(s*scale*log2e - m) with the MUFU
  ``ex2``, accumulate the row sum, and write P back into S's TMEM columns (S_i(j+1) is issued after
  PV_i(j), and MMAs from one thread execute in order, so the next S never overwrites a P still being
  read).  O is rescaled in TMEM only when a row's running max grew by more than 2^8 (a stale max is
  exact as long as P and the row sum use the same one);
* blocks above the diagonal are never computed; CTAs start with the longest rows (causal work grows
  with the query index).

The tensor core multiplies bf16 by bf16, so P is written as two bf16 parts, P = P_hi + P_lo
(P_lo = bf16(p - P_hi)), and O_i += P_hi V + P_lo V: the product keeps ~16 significant bits of p,
so the result matches an f32-P computation to within the output's bf16 rounding.  ``precise=False``
drops P_lo (one PV pass, 2^-9 relative error per term).

Every mbarrier wait is bounded (see :mod:`.ptxasm`); a time-out writes a code to the status word and
leaves the loop, the producer waits (bounded) for its own loads, and TMEM is always freed.
"""
from __future__ import annotations

import math

from .ptxasm import Asm, idesc_f16, smem_desc_hi, wait_bar, wait_bar_warp

BQ = 128
BKV = 128
D = 128
TILES = 2
STAGES = 4
TILE_BYTES = BQ * D * 2          # 32 KiB: a Q, K or V tile
HALF = TILE_BYTES // 2           # one 64-column TMA box
THREADS = 384
TMEM_COLS = 512
LOG2E = 1.4426950408889634
RESCALE_THRESHOLD = 8.0          # log2 units: rescale O only when the max grew by more than 2^8

ERR_PRODUCER, ERR_MMA, ERR_SOFTMAX, ERR_EPILOGUE, ERR_DRAIN = 11, 12, 13, 14, 15

# barrier offsets (bytes from the barrier area)
QFULL, FULL, EMPTY, SFULL, PFULL, PFREE, SLOT = 0, 8, 40, 72, 88, 104, 120


def _f32(v: float) -> str:
    import struct
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", v))[0]


def attention_entry(name: str, batch: int, heads: int, seq: int, causal: bool, scale: float,
                    names=("Q", "K", "V", "O"), prefix: str = "", precise: bool = True) -> dict:
    if seq % (BQ * TILES) or seq % BKV:
        raise ValueError("tcgen05 attention needs S % 256 == 0")
    nt = seq // (BQ * TILES)
    grid = batch * heads * nt
    a = Asm()
    idesc_qk = idesc_f16(BQ, BKV, False, False)
    idesc_pv = idesc_f16(BQ, D, False, True)
    kdesc_hi = smem_desc_hi(16, 1024)            # K-major SW128 (Q, K)
    vdesc_hi = smem_desc_hi(HALF, 1024)          # MN-major SW128 (V): 64-column atoms 16 KiB apart
    cscale = _f32(scale * LOG2E)

    tid, warp, lane, cta = a.r(), a.r(), a.r(), a.r()
    a(f"mov.u32 {tid}, %tid.x;")
    a(f"shr.u32 {warp}, {tid}, 5;")
    a(f"and.b32 {lane}, {tid}, 31;")
    a(f"mov.u32 {cta}, %ctaid.x;")
    o_ptr, err = a.r("rd"), a.r("rd")
    a(f"ld.param.u64 {o_ptr}, [p_O];")
    a(f"cvta.to.global.u64 {o_ptr}, {o_ptr};")
    a(f"ld.param.u64 {err}, [p_err];")
    a(f"cvta.to.global.u64 {err}, {err};")
    tq, tk, tv = a.r("rd"), a.r("rd"), a.r("rd")
    for reg, pname in ((tq, "p_tmQ"), (tk, "p_tmK"), (tv, "p_tmV")):
        a(f"mov.u64 {reg}, {pname};")
        a(f"cvta.param.u64 {reg}, {reg};")

    # work unit: longest causal rows first
    t, bh, bb, hh = a.r(), a.r(), a.r(), a.r()
    a(f"div.u32 {t}, {cta}, {batch * heads};")
    a(f"sub.u32 {t}, {nt - 1}, {t};")
    a(f"rem.u32 {bh}, {cta}, {batch * heads};")
    a(f"div.u32 {bb}, {bh}, {heads};")
    a(f"rem.u32 {hh}, {bh}, {heads};")
    nb, row0 = a.r(), a.r()
    if causal:
        a(f"shl.b32 {nb}, {t}, 1;")
        a(f"add.u32 {nb}, {nb}, 2;")                    # tile 1 sees kv blocks 0..2t+1, tile 0 0..2t
    else:
        a(f"mov.u32 {nb}, {seq // BKV};")
    a(f"shl.b32 {row0}, {t}, 8;")                        # first query row of this CTA

    raw, base = a.r(), a.r()
    smem_sym = f"{prefix}attn_smem"
    a(f"mov.u32 {raw}, {smem_sym};")
    a(f"add.u32 {base}, {raw}, 1023;")
    a(f"and.b32 {base}, {base}, -1024;")
    sQ, sKV, bars = a.r(), a.r(), a.r()
    a(f"mov.u32 {sQ}, {base};")
    a(f"add.u32 {sKV}, {base}, {TILES * TILE_BYTES};")
    a(f"add.u32 {bars}, {base}, {TILES * TILE_BYTES + STAGES * TILE_BYTES};")

    p0 = a.r("p")
    a(f"setp.eq.u32 {p0}, {tid}, 0;")
    l_init = a.L("noinit")
    a(f"@!{p0} bra {l_init};")
    a(f"mbarrier.init.shared::cta.b64 [{bars}+{QFULL}], 1;")
    for s in range(STAGES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{FULL + 8 * s}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{EMPTY + 8 * s}], 1;")
    for i in range(TILES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{SFULL + 8 * i}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{PFULL + 8 * i}], 4;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{PFREE + 8 * i}], 1;")
    a("fence.mbarrier_init.release.cluster;")
    a("fence.proxy.async.shared::cta;")
    a.label(l_init)
    pw1 = a.r("p")
    a(f"setp.eq.u32 {pw1}, {warp}, 1;")
    l_noalloc = a.L("noalloc")
    a(f"@!{pw1} bra {l_noalloc};")
    a(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{bars}+{SLOT}], {TMEM_COLS};")
    a("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;")
    a("tcgen05.fence::before_thread_sync;")
    a.label(l_noalloc)
    a("bar.sync 0;")
    a("tcgen05.fence::after_thread_sync;")
    taddr = a.r()
    a(f"ld.shared.b32 {taddr}, [{bars}+{SLOT}];")

    l_end = a.L("end")
    l_prod, l_mma, l_soft = a.L("prod"), a.L("mma"), a.L("soft")
    pw0, pws = a.r("p"), a.r("p")
    a(f"setp.eq.u32 {pw0}, {warp}, 0;")
    a(f"setp.ge.u32 {pws}, {warp}, 4;")
    a(f"@{pw0} bra {l_prod};")
    a(f"@{pw1} bra {l_mma};")
    a(f"@{pws} bra {l_soft};")
    a(f"bra {l_end};")                                   # warps 2-3: no role

    def tma4(dst, tmap, c0, c1, mbar):
        a(f"cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
          f"[{dst}], [{tmap}, {{{c0}, {c1}, {hh}, {bb}}}], [{mbar}];")

    # ---------------- producer ------------------------------------------------------------
    a.label(l_prod)
    pl0 = a.r("p")
    a(f"setp.ne.u32 {pl0}, {lane}, 0;")
    a(f"@{pl0} bra {l_end};")
    qb = a.r()
    a(f"add.u32 {qb}, {bars}, {QFULL};")
    a(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{qb}], {TILES * TILE_BYTES};")
    for i in range(TILES):
        r_i = a.r()
        a(f"add.u32 {r_i}, {row0}, {BQ * i};")
        for half in range(2):
            d_ = a.r()
            a(f"add.u32 {d_}, {sQ}, {TILE_BYTES * i + HALF * half};")
            tma4(d_, tq, 64 * half, r_i, qb)
    n_, stage, phase = a.r(), a.r(), a.r()
    armed = [a.r() for _ in range(STAGES)]
    for r_ in armed:
        a(f"mov.u32 {r_}, 2;")
    a(f"mov.u32 {n_}, 0;")
    a(f"mov.u32 {stage}, 0;")
    a(f"mov.u32 {phase}, 0;")
    nitems = a.r()
    a(f"shl.b32 {nitems}, {nb}, 1;")
    l_pl, l_pdone = a.L("pl"), a.L("pdone")
    a.label(l_pl)
    pend = a.r("p")
    a(f"setp.ge.u32 {pend}, {n_}, {nitems};")
    a(f"@{pend} bra {l_pdone};")
    fb, eb, par = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {fb}, {stage}, 8, {bars};")
    a(f"add.u32 {eb}, {fb}, {EMPTY};")
    a(f"add.u32 {fb}, {fb}, {FULL};")
    a(f"xor.b32 {par}, {phase}, 1;")
    wait_bar(a, eb, par, err, ERR_PRODUCER, l_pdone)
    a(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {TILE_BYTES};")
    for s in range(STAGES):
        ps = a.r("p")
        a(f"setp.eq.u32 {ps}, {stage}, {s};")
        a(f"@{ps} mov.u32 {armed[s]}, {phase};")
    kvrow, dst, isv = a.r(), a.r(), a.r("p")
    a(f"shr.u32 {kvrow}, {n_}, 1;")
    a(f"shl.b32 {kvrow}, {kvrow}, 7;")
    a(f"mad.lo.u32 {dst}, {stage}, {TILE_BYTES}, {sKV};")
    tsel = a.r("rd")
    andn = a.r()
    a(f"and.b32 {andn}, {n_}, 1;")
    a(f"setp.ne.u32 {isv}, {andn}, 0;")
    a(f"selp.b64 {tsel}, {tv}, {tk}, {isv};")
    tma4(dst, tsel, 0, kvrow, fb)
    dst2 = a.r()
    a(f"add.u32 {dst2}, {dst}, {HALF};")
    tma4(dst2, tsel, 64, kvrow, fb)
    pw = a.r("p")
    a(f"add.u32 {stage}, {stage}, 1;")
    a(f"setp.eq.u32 {pw}, {stage}, {STAGES};")
    a(f"@{pw} mov.u32 {stage}, 0;")
    a(f"@{pw} xor.b32 {phase}, {phase}, 1;")
    a(f"add.u32 {n_}, {n_}, 1;")
    a(f"bra {l_pl};")
    a.label(l_pdone)
    for s in range(STAGES):
        skip = a.L("dskip")
        pn = a.r("p")
        a(f"setp.eq.u32 {pn}, {armed[s]}, 2;")
        a(f"@{pn} bra {skip};")
        fbs = a.r()
        a(f"add.u32 {fbs}, {bars}, {FULL + 8 * s};")
        wait_bar(a, fbs, armed[s], err, ERR_DRAIN, skip)
        a.label(skip)
    wait_q = a.L("dq")
    zero = a.r()
    a(f"mov.u32 {zero}, 0;")
    wait_bar(a, qb, zero, err, ERR_DRAIN, wait_q)
    a.label(wait_q)
    a(f"bra {l_end};")

    # ---------------- MMA issuer --------------------------------------------------------------
    a.label(l_mma)
    pl1 = a.r("p")
    a(f"setp.ne.u32 {pl1}, {lane}, 0;")
    a(f"@{pl1} bra {l_end};")
    l_mdone = a.L("mdone")
    qb2, zero2 = a.r(), a.r()
    a(f"add.u32 {qb2}, {bars}, {QFULL};")
    a(f"mov.u32 {zero2}, 0;")
    wait_bar(a, qb2, zero2, err, ERR_MMA, l_mdone)
    a("tcgen05.fence::after_thread_sync;")
    iqk, ipv = a.r(), a.r()
    a(f"mov.u32 {iqk}, {idesc_qk};")
    a(f"mov.u32 {ipv}, {idesc_pv};")
    ptrue, pfalse = a.r("p"), a.r("p")
    a(f"setp.eq.u32 {ptrue}, {lane}, {lane};")
    a(f"setp.ne.u32 {pfalse}, {lane}, {lane};")
    khi, vhi = a.r("rd"), a.r("rd")
    a(f"mov.b64 {khi}, {kdesc_hi};")
    a(f"mov.b64 {vhi}, {vdesc_hi};")
    last0 = a.r()
    a(f"sub.u32 {last0}, {nb}, {2 if causal else 1};")   # tile 0's last kv block

    def desc(addr_reg, off, hi):
        r1 = a.r()
        d_ = a.r("rd")
        a(f"add.u32 {r1}, {addr_reg}, {off};")
        a(f"shr.u32 {r1}, {r1}, 4;")
        a(f"cvt.u64.u32 {d_}, {r1};")
        a(f"or.b64 {d_}, {d_}, {hi};")
        return d_

    def item_stage(item):
        """(stage base address, full barrier, empty barrier) of ring item ``item``."""
        st_, fbr, ebr = a.r(), a.r(), a.r()
        a(f"rem.u32 {st_}, {item}, {STAGES};")
        a(f"mad.lo.u32 {fbr}, {st_}, 8, {bars};")
        a(f"add.u32 {ebr}, {fbr}, {EMPTY};")
        a(f"add.u32 {fbr}, {fbr}, {FULL};")
        sb = a.r()
        a(f"mad.lo.u32 {sb}, {st_}, {TILE_BYTES}, {sKV};")
        return sb, fbr, ebr

    def item_wait(item):
        sb, fbr, ebr = item_stage(item)
        par_ = a.r()
        a(f"div.u32 {par_}, {item}, {STAGES};")
        a(f"and.b32 {par_}, {par_}, 1;")
        wait_bar(a, fbr, par_, err, ERR_MMA, l_mdone)
        a("tcgen05.fence::after_thread_sync;")
        return sb, ebr

    def qk(i, kbase, jreg):
        """S_i = Q_i K^T for the K block at ``kbase``.  Issued after PV_i of the previous block, which
        read P_i from the same TMEM columns; the tensor core runs one thread's MMAs in order."""
        dcol = a.r()
        a(f"add.u32 {dcol}, {taddr}, {BKV * i};")
        qbase = a.r()
        a(f"add.u32 {qbase}, {sQ}, {TILE_BYTES * i};")
        for k in range(D // 16):
            off = (k // 4) * HALF + (k % 4) * 32
            da = desc(qbase, off, khi)
            db = desc(kbase, off, khi)
            a(f"tcgen05.mma.cta_group::1.kind::f16 [{dcol}], {da}, {db}, {iqk}, {ptrue if k else pfalse};")
        sfull = a.r()
        a(f"add.u32 {sfull}, {bars}, {SFULL + 8 * i};")
        a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{sfull}];")

    def pv(i, vbase, jreg):
        """O_i += P_i V for the V block at ``vbase`` (P_i in TMEM: hi part in S_i's columns 0-63, lo
        part in 64-127, two bf16 per column), once the softmax has written P_i."""
        pfb, par_ = a.r(), a.r()
        a(f"add.u32 {pfb}, {bars}, {PFULL + 8 * i};")
        a(f"and.b32 {par_}, {jreg}, 1;")
        wait_bar(a, pfb, par_, err, ERR_MMA, l_mdone)
        a("tcgen05.fence::after_thread_sync;")
        dcol = a.r()
        a(f"add.u32 {dcol}, {taddr}, {2 * BKV + D * i};")
        for part in range(2 if precise else 1):
            for k in range(BKV // 16):
                at = a.r()
                a(f"add.u32 {at}, {taddr}, {BKV * i + 64 * part + 8 * k};")
                db = desc(vbase, 2048 * k, vhi)
                if k == 0 and part == 0:
                    pacc = a.r("p")
                    a(f"setp.ne.u32 {pacc}, {jreg}, 0;")
                else:
                    pacc = ptrue
                a(f"tcgen05.mma.cta_group::1.kind::f16 [{dcol}], [{at}], {db}, {ipv}, {pacc};")
        pfree = a.r()
        a(f"add.u32 {pfree}, {bars}, {PFREE + 8 * i};")
        a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{pfree}];")

    def commit(bar_reg):
        a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{bar_reg}];")

    # prologue: S_0(0), S_1(0) from K_0 (ring item 0)
    j = a.r()
    item0 = a.r()
    a(f"mov.u32 {j}, 0;")
    a(f"mov.u32 {item0}, 0;")
    kb0, ke0 = item_wait(item0)
    qk(0, kb0, j)
    qk(1, kb0, j)
    commit(ke0)
    l_mj, l_mjend = a.L("mj"), a.L("mjend")
    a.label(l_mj)
    itv = a.r()
    a(f"shl.b32 {itv}, {j}, 1;")
    a(f"add.u32 {itv}, {itv}, 1;")                          # V_j is ring item 2j+1
    vb, ve = item_wait(itv)
    jn = a.r()
    a(f"add.u32 {jn}, {j}, 1;")
    have_next = a.r("p")
    a(f"setp.lt.u32 {have_next}, {jn}, {nb};")
    l_pv0 = a.L("nopv0")
    p0j = a.r("p")
    a(f"setp.gt.u32 {p0j}, {j}, {last0};")
    a(f"@{p0j} bra {l_pv0};")
    pv(0, vb, j)
    a.label(l_pv0)
    l_nok = a.L("nok")
    a(f"@!{have_next} bra {l_nok};")
    itk = a.r()
    a(f"shl.b32 {itk}, {jn}, 1;")                           # K_{j+1} is ring item 2j+2
    kb_, ke_ = item_wait(itk)
    l_qk0 = a.L("noqk0")
    p0n = a.r("p")
    a(f"setp.gt.u32 {p0n}, {jn}, {last0};")
    a(f"@{p0n} bra {l_qk0};")
    qk(0, kb_, jn)
    a.label(l_qk0)
    pv(1, vb, j)
    commit(ve)
    qk(1, kb_, jn)
    commit(ke_)
    a(f"mov.u32 {j}, {jn};")
    a(f"bra {l_mj};")
    a.label(l_nok)
    pv(1, vb, j)                                           # last block: no K_{j+1}
    commit(ve)
    a.label(l_mjend)
    a.label(l_mdone)
    a(f"bra {l_end};")

    # ---------------- softmax warps ------------------------------------------------------------
    a.label(l_soft)
    ti, q, rowl = a.r(), a.r(), a.r()
    a(f"sub.u32 {ti}, {warp}, 4;")
    a(f"shr.u32 {ti}, {ti}, 2;")                            # Q tile of this warpgroup
    a(f"and.b32 {q}, {warp}, 3;")
    a(f"mad.lo.u32 {rowl}, {q}, 32, {lane};")              # row within the tile (= TMEM lane)
    lanebase = a.r()
    a(f"shl.b32 {lanebase}, {q}, 21;")
    a(f"add.u32 {lanebase}, {lanebase}, {taddr};")
    scol, ocol = a.r(), a.r()
    a(f"mad.lo.u32 {scol}, {ti}, {BKV}, {lanebase};")
    a(f"mad.lo.u32 {ocol}, {ti}, {D}, {lanebase};")
    a(f"add.u32 {ocol}, {ocol}, {2 * BKV};")
    last = a.r()
    if causal:
        a(f"shl.b32 {last}, {t}, 1;")
        a(f"add.u32 {last}, {last}, {ti};")                # tile i's last (diagonal) kv block
    else:
        a(f"sub.u32 {last}, {nb}, 1;")
    sfb, pfb, pfr = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {sfb}, {ti}, 8, {bars};")
    a(f"add.u32 {pfb}, {sfb}, {PFULL};")
    a(f"add.u32 {pfr}, {sfb}, {PFREE};")
    a(f"add.u32 {sfb}, {sfb}, {SFULL};")
    s_ = [a.r("f") for _ in range(BKV)]
    mref, lsum, jj = a.r("f"), a.r("f"), a.r()
    a(f"mov.b32 {mref}, 0fFF800000;")
    a(f"mov.b32 {lsum}, 0f00000000;")
    a(f"mov.u32 {jj}, 0;")
    l_sj, l_sdone = a.L("sj"), a.L("sdone")
    a.label(l_sj)
    pj = a.r("p")
    a(f"setp.gt.u32 {pj}, {jj}, {last};")
    a(f"@{pj} bra {l_sdone};")
    par_s = a.r()
    a(f"and.b32 {par_s}, {jj}, 1;")
    wait_bar_warp(a, sfb, par_s, err, ERR_SOFTMAX, l_sdone)
    a("tcgen05.fence::after_thread_sync;")
    for c in range(BKV // 32):
        src = a.r()
        a(f"add.u32 {src}, {scol}, {32 * c};")
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(s_[32 * c:32 * c + 32])}}}, [{src}];")
    a("tcgen05.wait::ld.sync.aligned;")
    ple = a.r("p")
    a(f"setp.eq.u32 {ple}, {lane}, 0;")
    if causal:
        l_nomask = a.L("nomask")
        pdiag = a.r("p")
        a(f"setp.ne.u32 {pdiag}, {jj}, {last};")
        a(f"@{pdiag} bra {l_nomask};")
        for c in range(BKV):
            pm = a.r("p")
            a(f"setp.lt.u32 {pm}, {rowl}, {c};")
            a(f"@{pm} mov.b32 {s_[c]}, 0fFF800000;")
        a.label(l_nomask)
    # row max (tree), in the scaled log2 domain
    lvl = [a.r("f") for _ in range(8)]
    for k in range(8):
        a(f"max.f32 {lvl[k]}, {s_[k]}, {s_[k + 8]};")
        for c in range(k + 16, BKV, 8):
            a(f"max.f32 {lvl[k]}, {lvl[k]}, {s_[c]};")
    while len(lvl) > 1:
        nxt = []
        for k in range(0, len(lvl), 2):
            a(f"max.f32 {lvl[k]}, {lvl[k]}, {lvl[k + 1]};")
            nxt.append(lvl[k])
        lvl = nxt
    mblk, mnew = a.r("f"), a.r("f")
    a(f"mul.f32 {mblk}, {lvl[0]}, {cscale};")
    a(f"max.f32 {mnew}, {mref}, {mblk};")
    l_first, l_after = a.L("first"), a.L("after")
    # alpha (the O rescale factor) is 1 unless this block raises the running max past the
    # threshold; it is written on both paths so every later read has a definition
    alpha = a.r("f")
    a(f"mov.b32 {alpha}, 0f3F800000;")
    pfirst = a.r("p")
    a(f"setp.eq.u32 {pfirst}, {jj}, 0;")
    a(f"@{pfirst} bra {l_first};")
    # later blocks: O_i and P_i are free once the previous PV has completed
    par_p = a.r()
    a(f"sub.u32 {par_p}, {jj}, 1;")
    a(f"and.b32 {par_p}, {par_p}, 1;")
    wait_bar_warp(a, pfr, par_p, err, ERR_SOFTMAX, l_sdone)
    need, anyneed = a.r("p"), a.r("p")
    thr = a.r("f")
    a(f"add.f32 {thr}, {mref}, {_f32(RESCALE_THRESHOLD)};")
    a(f"setp.gt.f32 {need}, {mnew}, {thr};")
    a(f"vote.sync.any.pred {anyneed}, {need}, -1;")
    l_norescale = a.L("norescale")
    a(f"@!{anyneed} bra {l_norescale};")
    dm = a.r("f")
    a(f"sub.f32 {dm}, {mref}, {mnew};")
    a(f"ex2.approx.ftz.f32 {alpha}, {dm};")
    a(f"mov.b32 {mref}, {mnew};")
    a(f"mul.f32 {lsum}, {lsum}, {alpha};")
    a.label(l_norescale)
    a(f"bra {l_after};")
    a.label(l_first)
    a(f"mov.b32 {mref}, {mnew};")
    a(f"setp.ne.u32 {anyneed}, {lane}, {lane};")
    a.label(l_after)
    # p = 2^(s*c - m), row sum, and P back into S_i's TMEM columns as bf16 pairs (hi, then lo)
    negm = a.r("f")
    a(f"neg.f32 {negm}, {mref};")
    parts = [a.r("f") for _ in range(4)]
    for pp in parts:
        a(f"mov.b32 {pp}, 0f00000000;")
    for c16 in range(BKV // 32):                        # 32 values -> 16 packed columns per part
        hi_w, lo_w = [], []
        for k in range(16):
            i0, i1 = 32 * c16 + 2 * k, 32 * c16 + 2 * k + 1
            for idx in (i0, i1):
                a(f"fma.rn.f32 {s_[idx]}, {s_[idx]}, {cscale}, {negm};")
                a(f"ex2.approx.ftz.f32 {s_[idx]}, {s_[idx]};")
                a(f"add.f32 {parts[idx & 3]}, {parts[idx & 3]}, {s_[idx]};")
            w = a.r()
            a(f"cvt.rn.bf16x2.f32 {w}, {s_[i1]}, {s_[i0]};")
            hi_w.append(w)
            if precise:
                h0, h1, r0, r1, wl = a.r("f"), a.r("f"), a.r("f"), a.r("f"), a.r()
                a(f"shl.b32 {h0}, {w}, 16;")
                a(f"and.b32 {h1}, {w}, -65536;")
                a(f"sub.f32 {r0}, {s_[i0]}, {h0};")
                a(f"sub.f32 {r1}, {s_[i1]}, {h1};")
                a(f"cvt.rn.bf16x2.f32 {wl}, {r1}, {r0};")
                lo_w.append(wl)
        dst = a.r()
        a(f"add.u32 {dst}, {scol}, {16 * c16};")
        a(f"tcgen05.st.sync.aligned.32x32b.x16.b32 [{dst}], {{{', '.join(hi_w)}}};")
        if precise:
            dst2 = a.r()
            a(f"add.u32 {dst2}, {scol}, {64 + 16 * c16};")
            a(f"tcgen05.st.sync.aligned.32x32b.x16.b32 [{dst2}], {{{', '.join(lo_w)}}};")
    p01, p23 = a.r("f"), a.r("f")
    a(f"add.f32 {p01}, {parts[0]}, {parts[1]};")
    a(f"add.f32 {p23}, {parts[2]}, {parts[3]};")
    a(f"add.f32 {p01}, {p01}, {p23};")
    a(f"add.f32 {lsum}, {lsum}, {p01};")
    # the lazy O rescale (the previous PV has completed: waited above)
    l_norescale2 = a.L("norescale2")
    a(f"@!{anyneed} bra {l_norescale2};")
    a("tcgen05.fence::after_thread_sync;")
    for c in range(D // 32):
        src = a.r()
        a(f"add.u32 {src}, {ocol}, {32 * c};")
        regs = s_[32 * c:32 * c + 32]
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{src}];")
        a("tcgen05.wait::ld.sync.aligned;")
        for r_ in regs:
            a(f"mul.f32 {r_}, {r_}, {alpha};")
        a(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{src}], {{{', '.join(regs)}}};")
    a.label(l_norescale2)
    a("tcgen05.wait::st.sync.aligned;")
    a("tcgen05.fence::before_thread_sync;")
    a("bar.warp.sync -1;")
    a(f"@{ple} mbarrier.arrive.shared::cta.b64 _, [{pfb}];")
    a(f"add.u32 {jj}, {jj}, 1;")
    a(f"bra {l_sj};")
    a.label(l_sdone)
    # epilogue: after the last PV, O / l to global memory as bf16
    l_noepi = a.L("noepi")
    pok = a.r("p")
    a(f"setp.le.u32 {pok}, {jj}, {last};")                  # left early (time-out): no store
    a(f"@{pok} bra {l_noepi};")
    par_e = a.r()
    a(f"and.b32 {par_e}, {last}, 1;")
    wait_bar_warp(a, pfr, par_e, err, ERR_EPILOGUE, l_noepi)
    a("tcgen05.fence::after_thread_sync;")
    inv = a.r("f")
    a(f"rcp.rn.f32 {inv}, {lsum};")
    grow, oaddr = a.r(), a.r("rd")
    a(f"mad.lo.u32 {grow}, {ti}, {BQ}, {row0};")
    a(f"add.u32 {grow}, {grow}, {rowl};")
    a(f"mad.lo.u32 {grow}, {bh}, {seq}, {grow};")          # row of O in [batch*heads*S, D]
    a(f"mul.wide.u32 {oaddr}, {grow}, {D * 2};")
    a(f"add.s64 {oaddr}, {oaddr}, {o_ptr};")
    for c in range(D // 32):
        src = a.r()
        a(f"add.u32 {src}, {ocol}, {32 * c};")
        regs = s_[32 * c:32 * c + 32]
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{src}];")
        a("tcgen05.wait::ld.sync.aligned;")
        words = []
        for k in range(16):
            w = a.r()
            a(f"mul.f32 {regs[2 * k]}, {regs[2 * k]}, {inv};")
            a(f"mul.f32 {regs[2 * k + 1]}, {regs[2 * k + 1]}, {inv};")
            a(f"cvt.rn.bf16x2.f32 {w}, {regs[2 * k + 1]}, {regs[2 * k]};")
            words.append(w)
        a(f"st.global.v8.b32 [{oaddr}+{64 * c}], {{{', '.join(words[:8])}}};")
        a(f"st.global.v8.b32 [{oaddr}+{64 * c + 32}], {{{', '.join(words[8:])}}};")
    a.label(l_noepi)

    # ---------------- teardown ---------------------------------------------------------------
    a.label(l_end)
    a("barrier.sync 0;")
    a("bar.warp.sync -1;")
    l_nodealloc = a.L("nodealloc")
    a(f"@!{pw1} bra {l_nodealloc};")
    a("tcgen05.fence::after_thread_sync;")
    a(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {taddr}, {TMEM_COLS};")
    a.label(l_nodealloc)

    dyn = TILES * TILE_BYTES + STAGES * TILE_BYTES + 256 + 1024
    entry = [f".visible .entry {name}(",
             "\t.param .u64 p_Q,", "\t.param .u64 p_K,", "\t.param .u64 p_V,", "\t.param .u64 p_O,",
             "\t.param .align 64 .b8 p_tmQ[128],", "\t.param .align 64 .b8 p_tmK[128],",
             "\t.param .align 64 .b8 p_tmV[128],", "\t.param .u64 p_err", ")",
             f".reqntid {THREADS}, 1, 1", ".maxnreg 168", "{"]
    entry += a.decls() + a.lines + ["\tret;", "}"]
    qn, kn, vn, on = names
    dims = [D, seq, heads, batch]
    strides = [D * 2, seq * D * 2, heads * seq * D * 2]
    tmaps = [{"name": f"tm{x}", "tensor": nm, "dtype": "bf16", "dims": dims, "strides": strides,
              "box": [64, 128, 1, 1], "swizzle": "128B"} for x, nm in (("Q", qn), ("K", kn), ("V", vn))]
    return {
        "name": name, "kind": "tcgen05_attention", "params": [qn, kn, vn, on],
        "raw_entry": entry, "raw_decls": [f".extern .shared .align 1024 .b8 {smem_sym}[];"],
        "grid": [grid, 1, 1], "block": [THREADS, 1, 1], "dyn_smem": dyn,
        "align": {qn: 16, kn: 16, vn: 16, on: 32}, "zero_outputs": [], "tmaps": tmaps,
        "extra": [{"name": "__err", "kind": "errword"}],
    }
