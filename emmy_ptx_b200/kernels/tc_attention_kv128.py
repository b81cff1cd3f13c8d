"""Attention on the tcgen05 tensor cores with 128-row key/value blocks (one score buffer per tile).

O = softmax(Q K^T * scale [+ causal mask]) V for Q, K, V, O bf16 [batch, heads, S, 128]: the same
online-softmax nest as :mod:`.tc_attention`, scheduled for a QK^T that is bound by the tensor core
rather than by shared memory.  A 128 x 64 x 16 MMA reads 4 KiB of Q and 2 KiB of K from shared memory
(48 cycles at 128 B per cycle against 32 cycles of math); a 128 x 128 x 16 one reads 8 KiB for 64
cycles of math, so the key/value block here is 128 rows.

One CTA owns 256 query rows of one (batch, head) as two 128-row tiles:

* warp 0 issues TMA: both Q tiles once, then K_0, V_0, K_1, V_1, ... through a 4-stage ring of
  32 KiB stages (each stage two 64-column boxes of 128 rows, 128-byte swizzle);
* one thread of warp 1 issues tile 0's ``tcgen05.mma``, one of warp 2 tile 1's.  TMEM holds
  O_0 | O_1 | S_0 | S_1, 128 columns each.  Per block j a tile's issuer runs O_i += P_i(j) V_j
  (M=128, N=128, K=128; P read from TMEM, V MN-major in shared memory) and then
  S_i(j+1) = Q_i K_(j+1)^T (M=128, N=128, K=128, both operands K-major) into the same columns;
* warps 4-7 (tile 0) and 8-11 (tile 1) run the online softmax, one thread per row: load the row of
  S_i(j) from TMEM, mask the diagonal block, take the row max, compute p = 2^(s*scale*log2e - m) on
  the MUFU, accumulate the row sum, and write P over the first 64 (f16) or all 128 (bf16 hi + lo)
  columns of S_i.  The two warpgroups take turns on the MUFU (named barriers 1 and 2), so one tile's
  exps overlap the other tile's MMAs.  O is rescaled in TMEM only when a row's running max grew by
  more than 2^8, after the previous PV has completed.

P_i(j) and S_i(j+1) share TMEM columns, so S_i(j+1) may only be written once PV_i(j) has read P.
``ordered=False`` (the default) makes the issuer wait for PV_i(j)'s completion (its commit to the
PV-done barrier) before issuing S_i(j+1): the order the tcgen05 memory model guarantees.  With
``ordered=True`` it relies on the tensor core running one thread's MMAs in issue order across
accumulators, which the PTX memory model promises only for MMAs into the same accumulator.

The value pre-pass (:mod:`.vconv`, 128-row blocks) provides the f16 copy of V and one flag per block,
exactly as for :mod:`.tc_attention`: f16 P with the f16 copy, or for a flagged block bf16 P_hi + P_lo
(columns 0-63 and 64-127) with V itself in two PV passes.

Every mbarrier wait is bounded (see :mod:`.ptxasm`); a time-out writes a code to the status word and
leaves the loop, the producer waits (bounded) for its own loads, the softmax warpgroups keep making
their turn hand-overs without the work, and TMEM is always freed.
"""
from __future__ import annotations

from .ptxasm import Asm, idesc_f16, smem_desc_hi, wait_bar, wait_bar_warp

BQ = 128                         # query rows per tile
BKV = 128                        # key/value rows per block
D = 128
TILES = 2
STAGES = 4
Q_BYTES = BQ * D * 2             # 32 KiB: one Q tile
Q_HALF = Q_BYTES // 2            # one 64-column TMA box of a Q tile
KV_BYTES = BKV * D * 2           # 32 KiB: one K or V block
KV_HALF = KV_BYTES // 2          # one 64-column TMA box of a K/V block
THREADS = 384
TMEM_COLS = 512
S_COL0 = TILES * D               # S_i at S_COL0 + BKV*i
LOG2E = 1.4426950408889634
RESCALE_THRESHOLD = 8.0          # log2 units: rescale O only when the max grew by more than 2^8

ERR_PRODUCER, ERR_MMA, ERR_SOFTMAX, ERR_EPILOGUE, ERR_DRAIN = 31, 32, 33, 34, 35

# barrier offsets (bytes from the barrier area): QFULL, FULL[4], EMPTY[4], SFULL[tile], PFULL[tile],
# PFREE[tile], then the TMEM address slot.  Each per-tile barrier completes once per kv block.
QFULL = 0
FULL = 8
EMPTY = FULL + 8 * STAGES
SFULL = EMPTY + 8 * STAGES
PFULL = SFULL + 8 * TILES
PFREE = PFULL + 8 * TILES
SLOT = PFREE + 8 * TILES
VFLAGS = 256                     # per kv block of this (batch, head): 1 when V did not fit f16 (64 words)
BAR_BYTES = 512
DYN_SMEM = TILES * Q_BYTES + STAGES * KV_BYTES + BAR_BYTES + 1024
REGS_LAUNCH = 65536 // THREADS // 8 * 8      # 168 a thread at launch
REGS_CONTROL = 96                            # warps 0-3 (producer, issuers) after setmaxnreg.dec
REGS_SOFTMAX = 200                           # warps 4-11 after setmaxnreg.inc
assert 128 * REGS_CONTROL + 256 * REGS_SOFTMAX <= THREADS * REGS_LAUNCH


def _f32(v: float) -> str:
    import struct
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", v))[0]


def attention_kv128_entry(name: str, batch: int, heads: int, seq: int, causal: bool, scale: float,
                          names=("Q", "K", "V", "O"), prefix: str = "", half: bool = True,
                          pingpong: bool = True, ordered: bool = False, pack_in_turn: bool = False,
                          scratch_names: tuple[str, str] | None = None) -> dict:
    """The kernel's launch record and PTX (see the module docstring for the schedule).
    ``half``: f16 P with the pre-pass's f16 copy of V where it fits (else bf16 P_hi + P_lo for every
    block); ``pingpong``: MUFU turns between the two tiles' softmax warpgroups; ``ordered``: issue
    S_i(j+1) straight after PV_i(j) without waiting for the PV to complete; ``pack_in_turn``: the
    second half's f16 packing stays inside the MUFU turn."""
    if seq % (BQ * TILES):
        raise ValueError("tcgen05 attention needs S % 256 == 0")
    nblk = seq // BKV
    if half and nblk > (BAR_BYTES - VFLAGS) // 4:
        raise ValueError("the f16 path keeps one flag per kv block in shared memory: S <= 8192")
    if pack_in_turn and not pingpong:
        raise ValueError("pack_in_turn needs the MUFU turns")
    threads = THREADS
    nt = seq // (BQ * TILES)
    nbh = batch * heads
    grid = nbh * nt
    a = Asm()
    idesc_qk = idesc_f16(BQ, BKV, False, False)
    idesc_pv = idesc_f16(BQ, D, False, True)
    idesc_pv16 = idesc_f16(BQ, D, False, True, half=True)
    kdesc_hi = smem_desc_hi(16, 1024)            # K-major SW128 (Q, K): 8-row groups 1 KiB apart
    vdesc_hi = smem_desc_hi(KV_HALF, 1024)       # MN-major SW128 (V): 64-column atoms 16 KiB apart
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
    tmaps_used = [(tq, "p_tmQ"), (tk, "p_tmK"), (tv, "p_tmV")]
    tv16 = None
    if half:
        tv16 = a.r("rd")
        tmaps_used.append((tv16, "p_tmV16"))
    for reg, pname in tmaps_used:
        a(f"mov.u64 {reg}, {pname};")
        a(f"cvta.param.u64 {reg}, {reg};")

    # work unit: longest causal rows first
    t, bh, bb, hh = a.r(), a.r(), a.r(), a.r()
    a(f"div.u32 {t}, {cta}, {nbh};")
    a(f"sub.u32 {t}, {nt - 1}, {t};")
    a(f"rem.u32 {bh}, {cta}, {nbh};")
    a(f"div.u32 {bb}, {bh}, {heads};")
    a(f"rem.u32 {hh}, {bh}, {heads};")
    nb, row0 = a.r(), a.r()
    if causal:
        a(f"shl.b32 {nb}, {t}, 1;")
        a(f"add.u32 {nb}, {nb}, 2;")                    # tile 1 sees kv blocks 0..2t+1, tile 0 0..2t
    else:
        a(f"mov.u32 {nb}, {nblk};")
    a(f"shl.b32 {row0}, {t}, 8;")                        # first query row of this CTA

    raw, base = a.r(), a.r()
    smem_sym = f"{prefix}attn128_smem"
    a(f"mov.u32 {raw}, {smem_sym};")
    a(f"add.u32 {base}, {raw}, 1023;")
    a(f"and.b32 {base}, {base}, -1024;")
    sQ, sKV, bars = a.r(), a.r(), a.r()
    a(f"mov.u32 {sQ}, {base};")
    a(f"add.u32 {sKV}, {base}, {TILES * Q_BYTES};")
    a(f"add.u32 {bars}, {base}, {TILES * Q_BYTES + STAGES * KV_BYTES};")

    p0 = a.r("p")
    a(f"setp.eq.u32 {p0}, {tid}, 0;")
    l_init = a.L("noinit")
    a(f"@!{p0} bra {l_init};")
    a(f"mbarrier.init.shared::cta.b64 [{bars}+{QFULL}], 1;")
    for s in range(STAGES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{FULL + 8 * s}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{EMPTY + 8 * s}], {TILES};")
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
    l_prod, l_mma, l_mma1, l_soft = a.L("prod"), a.L("mma"), a.L("mma1"), a.L("soft")
    pw0, pw2, pws = a.r("p"), a.r("p"), a.r("p")
    a(f"setp.eq.u32 {pw0}, {warp}, 0;")
    a(f"setp.eq.u32 {pw2}, {warp}, 2;")
    a(f"setp.ge.u32 {pws}, {warp}, 4;")
    # registers move from the producer / issuer warpgroup to the softmax warpgroups, which hold a
    # 128-column score row each: 128 x 96 + 256 x 200 = 63,488 of the 384 x 168 = 64,512 launched
    l_regs = a.L("regs")
    a(f"@{pws} bra {l_regs};")
    a(f"setmaxnreg.dec.sync.aligned.u32 {REGS_CONTROL};")
    a(f"@{pw0} bra {l_prod};")
    a(f"@{pw1} bra {l_mma};")
    a(f"@{pw2} bra {l_mma1};")
    a(f"bra {l_end};")                                   # warp 3: no role
    a.label(l_regs)
    a(f"setmaxnreg.inc.sync.aligned.u32 {REGS_SOFTMAX};")
    a(f"bra {l_soft};")

    def tma4(dst, tmap, c0, c1, mbar):
        a(f"cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
          f"[{dst}], [{tmap}, {{{c0}, {c1}, {hh}, {bb}}}], [{mbar}];")

    # ---------------- producer ------------------------------------------------------------
    a.label(l_prod)
    if half:
        # the value pre-pass's per-block flags of this (batch, head) into shared memory (lane l
        # loads blocks l and l + 32); they are published with the Q barrier's arrival below
        vfp, vbase = a.r("rd"), a.r()
        a(f"ld.param.u64 {vfp}, [p_vflag];")
        a(f"cvta.to.global.u64 {vfp}, {vfp};")
        a(f"mul.lo.u32 {vbase}, {bh}, {nblk};")
        for k in range(2):
            bk, pk, fk, ga, sa = a.r(), a.r("p"), a.r(), a.r("rd"), a.r()
            a(f"add.u32 {bk}, {lane}, {32 * k};")
            a(f"setp.lt.u32 {pk}, {bk}, {nb};")
            a(f"add.u32 {fk}, {vbase}, {bk};")
            a(f"mul.wide.u32 {ga}, {fk}, 4;")
            a(f"add.s64 {ga}, {ga}, {vfp};")
            a(f"@{pk} ld.global.nc.u32 {fk}, [{ga}];")
            a(f"mad.lo.u32 {sa}, {bk}, 4, {bars};")
            a(f"@{pk} st.shared.u32 [{sa}+{VFLAGS}], {fk};")
        a("fence.acq_rel.cta;")
        a("bar.warp.sync -1;")
    pl0 = a.r("p")
    a(f"setp.ne.u32 {pl0}, {lane}, 0;")
    a(f"@{pl0} bra {l_end};")
    qb = a.r()
    a(f"add.u32 {qb}, {bars}, {QFULL};")
    a(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{qb}], {TILES * Q_BYTES};")
    for i in range(TILES):
        r_i = a.r()
        a(f"add.u32 {r_i}, {row0}, {BQ * i};")
        for hb in range(2):
            d_ = a.r()
            a(f"add.u32 {d_}, {sQ}, {Q_BYTES * i + Q_HALF * hb};")
            tma4(d_, tq, 64 * hb, r_i, qb)
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
    a(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {KV_BYTES};")
    for s in range(STAGES):
        ps = a.r("p")
        a(f"setp.eq.u32 {ps}, {stage}, {s};")
        a(f"@{ps} mov.u32 {armed[s]}, {phase};")
    kvrow, dst, isv = a.r(), a.r(), a.r("p")
    a(f"shr.u32 {kvrow}, {n_}, 1;")
    a(f"shl.b32 {kvrow}, {kvrow}, 7;")
    a(f"mad.lo.u32 {dst}, {stage}, {KV_BYTES}, {sKV};")
    tsel = a.r("rd")
    andn = a.r()
    a(f"and.b32 {andn}, {n_}, 1;")
    a(f"setp.ne.u32 {isv}, {andn}, 0;")
    if half:
        # a V block that fit f16 comes from the pre-pass's f16 copy, a flagged one from V itself
        vfl, vfa2, pvf = a.r(), a.r(), a.r("p")
        a(f"shr.u32 {vfa2}, {n_}, 1;")
        a(f"mad.lo.u32 {vfa2}, {vfa2}, 4, {bars};")
        a(f"ld.shared.u32 {vfl}, [{vfa2}+{VFLAGS}];")
        a(f"setp.eq.u32 {pvf}, {vfl}, 0;")
        tvs = a.r("rd")
        a(f"selp.b64 {tvs}, {tv16}, {tv}, {pvf};")
        a(f"selp.b64 {tsel}, {tvs}, {tk}, {isv};")
    else:
        a(f"selp.b64 {tsel}, {tv}, {tk}, {isv};")
    tma4(dst, tsel, 0, kvrow, fb)
    dst2 = a.r()
    a(f"add.u32 {dst2}, {dst}, {KV_HALF};")
    tma4(dst2, tsel, 64, kvrow, fb)
    pw = a.r("p")
    a(f"add.u32 {stage}, {stage}, 1;")
    a(f"setp.eq.u32 {pw}, {stage}, {STAGES};")
    a(f"@{pw} mov.u32 {stage}, 0;")
    a(f"@{pw} xor.b32 {phase}, {phase}, 1;")
    a(f"add.u32 {n_}, {n_}, 1;")
    a(f"bra {l_pl};")
    a.label(l_pdone)
    # before leaving: every load this thread issued has landed (bounded waits), so no TMA write
    # into shared memory is still in flight when the CTA ends
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

    # ---------------- MMA issuers ---------------------------------------------------------------
    # one issuing thread per query tile (warp 1: tile 0, warp 2: tile 1); each ring stage is released
    # when both issuers' MMAs that read it have completed (empty barriers count two arrivals)
    def issuer(i, l_label):
        a.label(l_label)
        pl = a.r("p")
        a(f"setp.ne.u32 {pl}, {lane}, 0;")
        a(f"@{pl} bra {l_end};")
        l_mdone = a.L(f"mdone{i}")
        qb2, zero2 = a.r(), a.r()
        a(f"add.u32 {qb2}, {bars}, {QFULL};")
        a(f"mov.u32 {zero2}, 0;")
        wait_bar(a, qb2, zero2, err, ERR_MMA, l_mdone)
        a("tcgen05.fence::after_thread_sync;")
        iqk, ipv, ipv16 = a.r(), a.r(), a.r()
        a(f"mov.u32 {iqk}, {idesc_qk};")
        a(f"mov.u32 {ipv}, {idesc_pv};")
        a(f"mov.u32 {ipv16}, {idesc_pv16};")
        ptrue, pfalse = a.r("p"), a.r("p")
        a(f"setp.eq.u32 {ptrue}, {lane}, {lane};")
        a(f"setp.ne.u32 {pfalse}, {lane}, {lane};")
        khi, vhi = a.r("rd"), a.r("rd")
        a(f"mov.b64 {khi}, {kdesc_hi};")
        a(f"mov.b64 {vhi}, {vdesc_hi};")
        lasti = a.r()                                      # this tile's last kv block
        a(f"sub.u32 {lasti}, {nb}, {(2 if causal else 1) if i == 0 else 1};")

        def base_desc(addr_reg, hi):
            """The shared-memory matrix descriptor of ``addr_reg``; a byte offset ``off`` within the
            same operand is the descriptor plus off >> 4 (the start-address field holds addr >> 4)."""
            r1 = a.r()
            d_ = a.r("rd")
            a(f"shr.u32 {r1}, {addr_reg}, 4;")
            a(f"cvt.u64.u32 {d_}, {r1};")
            a(f"or.b64 {d_}, {d_}, {hi};")
            return d_

        def plus(d0, off):
            if not off:
                return d0
            d_ = a.r("rd")
            a(f"add.s64 {d_}, {d0}, {off >> 4};")
            return d_

        qb_i = a.r()
        a(f"add.u32 {qb_i}, {sQ}, {Q_BYTES * i};")
        q0 = base_desc(qb_i, khi)
        qdesc = [plus(q0, (k // 4) * Q_HALF + (k % 4) * 32) for k in range(D // 16)]
        kd, vd = [], []
        for st_ in range(STAGES):
            sb = a.r()
            a(f"add.u32 {sb}, {sKV}, {st_ * KV_BYTES};")
            kd.append(base_desc(sb, khi))
            vd.append(base_desc(sb, vhi))
        scol_c, ocol_c = a.r(), a.r()
        a(f"add.u32 {ocol_c}, {taddr}, {D * i};")
        a(f"add.u32 {scol_c}, {taddr}, {S_COL0 + BKV * i};")

        def ring_wait(stage_c, par):
            wait_bar(a, f"{bars}+{FULL + 8 * stage_c}", par, err, ERR_MMA, l_mdone)
            a("tcgen05.fence::after_thread_sync;")

        def qk(stage_c):
            """S_i = Q_i K^T (K in ring stage ``stage_c``) over S_i's 128 columns."""
            for k in range(D // 16):
                db = plus(kd[stage_c], (k // 4) * KV_HALF + (k % 4) * 32)
                a(f"tcgen05.mma.cta_group::1.kind::f16 [{scol_c}], {qdesc[k]}, {db}, {iqk}, "
                  f"{ptrue if k else pfalse};")
            a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{bars}+{SFULL + 8 * i}];")

        def pv(stage_c, jreg):
            """O_i += P_i(j) V_j (V_j in ring stage ``stage_c``) once the softmax has written P_i(j)
            over S_i (the P-full barrier's phase j, parity j & 1).  The block's pre-pass flag picks
            f16 P (columns 0-63) times the f16 copy of V, or bf16 P_hi (0-63) and P_lo (64-127) times
            V itself."""
            vds = [plus(vd[stage_c], 2048 * k) for k in range(BKV // 16)]
            pacc = a.r("p")
            a(f"setp.ne.u32 {pacc}, {jreg}, 0;")
            p16 = None
            if half:
                fa_, fmt = a.r(), a.r()
                p16 = a.r("p")
                a(f"mad.lo.u32 {fa_}, {jreg}, 4, {bars};")
                a(f"ld.shared.u32 {fmt}, [{fa_}+{VFLAGS}];")
                a(f"setp.eq.u32 {p16}, {fmt}, 0;")
            pp = a.r()
            a(f"and.b32 {pp}, {jreg}, 1;")
            wait_bar(a, f"{bars}+{PFULL + 8 * i}", pp, err, ERR_MMA, l_mdone)
            a("tcgen05.fence::after_thread_sync;")
            l_bf, l_done = a.L("pvbf"), a.L("pvdone")
            if half:
                a(f"@!{p16} bra {l_bf};")
                for k in range(BKV // 16):
                    acc = pacc if k == 0 else ptrue
                    a(f"tcgen05.mma.cta_group::1.kind::f16 [{ocol_c}], [{scol_c}+{8 * k}], "
                      f"{vds[k]}, {ipv16}, {acc};")
                a(f"bra {l_done};")
            a.label(l_bf)
            for part in range(2):
                for k in range(BKV // 16):
                    acc = pacc if (k == 0 and part == 0) else ptrue
                    a(f"tcgen05.mma.cta_group::1.kind::f16 [{ocol_c}], [{scol_c}+{(BKV // 2) * part + 8 * k}], "
                      f"{vds[k]}, {ipv}, {acc};")
            a.label(l_done)
            a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{bars}+{PFREE + 8 * i}];")

        def release(stage_c, used):
            """This issuer's arrival on the stage's empty barrier: after its MMAs that read the stage
            complete, or at once (``used`` False) for a block this tile does not compute."""
            if used:
                a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
                  f"[{bars}+{EMPTY + 8 * stage_c}];")
            else:
                a(f"mbarrier.arrive.shared::cta.b64 _, [{bars}+{EMPTY + 8 * stage_c}];")

        # prologue: S_i(0) from K_0 (ring item 0, stage 0)
        j, gp, gpn = a.r(), a.r(), a.r()
        a(f"mov.u32 {j}, 0;")
        a(f"mov.u32 {gp}, 0;")
        ring_wait(0, gp)
        qk(0)
        release(0, True)
        l_mg = a.L(f"mg{i}")
        a.label(l_mg)
        a(f"xor.b32 {gpn}, {gp}, 1;")
        for u in range(STAGES // 2):                       # block j = 2g + u: K_j in stage 2u, V_j in 2u+1
            vs = 2 * u + 1
            ring_wait(vs, gp)
            l_pv, l_pvd = a.L("nopv"), a.L("pvd")
            pj_ = a.r("p")
            a(f"setp.gt.u32 {pj_}, {j}, {lasti};")
            a(f"@{pj_} bra {l_pv};")
            pv(vs, j)
            release(vs, True)
            a(f"bra {l_pvd};")
            a.label(l_pv)
            release(vs, False)
            a.label(l_pvd)
            # the next block's scores into the same TMEM columns (K_{j+1} = item 2j+2)
            have_next = a.r("p")
            jn = a.r()
            a(f"add.u32 {jn}, {j}, 1;")
            a(f"setp.lt.u32 {have_next}, {jn}, {nb};")
            a(f"@!{have_next} bra {l_mdone};")
            ks = (2 * u + 2) % STAGES
            ring_wait(ks, gpn if u == STAGES // 2 - 1 else gp)
            l_qk, l_qkd = a.L("noqk"), a.L("qkd")
            pn_ = a.r("p")
            a(f"setp.gt.u32 {pn_}, {jn}, {lasti};")
            a(f"@{pn_} bra {l_qk};")
            if not ordered:
                # PV_i(j) has read P_i(j) from these columns before S_i(j+1) overwrites them
                pq = a.r()
                a(f"and.b32 {pq}, {j}, 1;")
                wait_bar(a, f"{bars}+{PFREE + 8 * i}", pq, err, ERR_MMA, l_mdone)
                a("tcgen05.fence::after_thread_sync;")
            qk(ks)
            release(ks, True)
            a(f"bra {l_qkd};")
            a.label(l_qk)
            release(ks, False)
            a.label(l_qkd)
            a(f"mov.u32 {j}, {jn};")
        a(f"mov.u32 {gp}, {gpn};")
        a(f"bra {l_mg};")
        a.label(l_mdone)
        a(f"bra {l_end};")

    issuer(0, l_mma)
    issuer(1, l_mma1)

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
    a(f"add.u32 {scol}, {scol}, {S_COL0};")                # S_ti
    a(f"mad.lo.u32 {ocol}, {ti}, {D}, {lanebase};")
    last, grow0 = a.r(), a.r()
    if causal:
        a(f"shl.b32 {last}, {t}, 1;")
        a(f"add.u32 {last}, {last}, {ti};")                # tile i's last kv block: 2t + i
    else:
        a(f"sub.u32 {last}, {nb}, 1;")
    a(f"mad.lo.u32 {grow0}, {ti}, {BQ}, {row0};")
    a(f"add.u32 {grow0}, {grow0}, {rowl};")                # this thread's query row
    sfb, pfb, pfr = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {sfb}, {ti}, 8, {bars};")
    a(f"add.u32 {pfb}, {sfb}, {PFULL};")
    a(f"add.u32 {pfr}, {sfb}, {PFREE};")
    a(f"add.u32 {sfb}, {sfb}, {SFULL};")

    def pv_done(blk, bail, code):
        """Wait until PV_ti(blk) has completed (the PV-done barrier's phase blk, parity blk & 1)."""
        pr_ = a.r()
        a(f"and.b32 {pr_}, {blk}, 1;")
        wait_bar_warp(a, pfr, pr_, err, code, bail)
    ple = a.r("p")
    a(f"setp.eq.u32 {ple}, {lane}, 0;")
    jj, failed = a.r(), a.r()
    a(f"mov.u32 {jj}, 0;")
    a(f"mov.u32 {failed}, 0;")
    l_sdone = a.L("sdone")
    l_drain, l_drain_post = (a.L("drain"), a.L("drainpost")) if pingpong else (l_sdone, l_sdone)
    if pingpong:
        # The two tiles' softmax warpgroups take turns on the MUFU: tile 0's exps of block j, then
        # tile 1's, then tile 0's of block j+1, ...  Each hands the turn over with a named barrier
        # (tile 0 waits on barrier 1 and passes on barrier 2, tile 1 the reverse; 256 threads: one
        # warpgroup syncs, the other arrives).  Tile 1 has one block more than tile 0 on the causal
        # diagonal and runs it alone.  Every softmax thread executes the same sequence of barrier
        # operations whatever happens: a time-out leaves the work but not the hand-overs (the drain
        # below), so neither warpgroup can be left waiting on the other.
        last0, arr_lim = a.r(), a.r()
        tile0 = a.r("p")
        if causal:
            a(f"shl.b32 {last0}, {t}, 1;")                 # tile 0's last kv block
        else:
            a(f"sub.u32 {last0}, {nb}, 1;")
        a(f"setp.eq.u32 {tile0}, {ti}, 0;")
        a(f"sub.u32 {arr_lim}, {last0}, {ti};")
        a(f"add.u32 {arr_lim}, {arr_lim}, 1;")             # pass the turn while jj < arr_lim
        pt1_, l_noinit = a.r("p"), a.L("noturn0")
        a(f"setp.eq.u32 {pt1_}, {ti}, 1;")
        a(f"@!{pt1_} bra {l_noinit};")
        a("bar.arrive 1, 256;")                              # tile 0 goes first
        a.label(l_noinit)

    def turn_wait():
        if not pingpong:
            return
        pw_, l_ = a.r("p"), a.L("noturnw")
        a(f"setp.gt.u32 {pw_}, {jj}, {last0};")
        a(f"@{pw_} bra {l_};")
        a(f"@{tile0} bar.sync 1, 256;")
        a(f"@!{tile0} bar.sync 2, 256;")
        a.label(l_)

    def turn_pass():
        if not pingpong:
            return
        pp_, l_ = a.r("p"), a.L("noturnp")
        a(f"setp.ge.u32 {pp_}, {jj}, {arr_lim};")
        a(f"@{pp_} bra {l_};")
        a(f"@{tile0} bar.arrive 2, 256;")
        a(f"@!{tile0} bar.arrive 1, 256;")
        a.label(l_)

    s_ = [a.r("f") for _ in range(BKV)]
    mref, lsum = a.r("f"), a.r("f")
    a(f"mov.b32 {mref}, 0fFF800000;")
    a(f"mov.b32 {lsum}, 0f00000000;")
    if half:
        # the producer published the per-block flags with its Q-barrier arrival
        qbs, zqs = a.r(), a.r()
        a(f"add.u32 {qbs}, {bars}, {QFULL};")
        a(f"mov.u32 {zqs}, 0;")
        wait_bar_warp(a, qbs, zqs, err, ERR_SOFTMAX, l_drain if pingpong else l_end)

    l_sj = a.L("sj")
    a.label(l_sj)
    pj = a.r("p")
    a(f"setp.gt.u32 {pj}, {jj}, {last};")
    a(f"@{pj} bra {l_sdone};")
    par_s = a.r()
    a(f"and.b32 {par_s}, {jj}, 1;")
    wait_bar_warp(a, sfb, par_s, err, ERR_SOFTMAX, l_drain)
    p16 = None
    if half:
        # the value pre-pass's flag for this block: f16 P (rounded to nearest, 2^-12 relative) when
        # V_j fit f16, else bf16 hi + lo
        vfa, fmt = a.r(), a.r()
        p16 = a.r("p")
        a(f"mad.lo.u32 {vfa}, {jj}, 4, {bars};")
        a(f"ld.shared.u32 {fmt}, [{vfa}+{VFLAGS}];")
        a(f"setp.eq.u32 {p16}, {fmt}, 0;")
    a("tcgen05.fence::after_thread_sync;")
    for c in range(BKV // 32):
        src = a.r()
        a(f"add.u32 {src}, {scol}, {32 * c};")
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(s_[32 * c:32 * c + 32])}}}, [{src}];")
    a("tcgen05.wait::ld.sync.aligned;")
    if causal:
        # kv = 128*jj + c is masked when kv > query row, i.e. c > grow0 - 128*jj; only the tile's last
        # block (the diagonal one) has masked columns
        l_nomask = a.L("nomask")
        lim, kv0 = a.r(), a.r()
        a(f"shl.b32 {kv0}, {jj}, 7;")
        a(f"sub.s32 {lim}, {grow0}, {kv0};")
        pnm, vnm = a.r("p"), a.r("p")
        a(f"setp.ge.s32 {pnm}, {lim}, {BKV - 1};")
        a(f"vote.sync.all.pred {vnm}, {pnm}, -1;")
        a(f"@{vnm} bra {l_nomask};")
        for c in range(BKV):
            pm = a.r("p")
            a(f"setp.lt.s32 {pm}, {lim}, {c};")
            a(f"@{pm} mov.b32 {s_[c]}, 0fFF800000;")
        a.label(l_nomask)
    # row max in the scaled log2 domain: 8 independent chains of three-input maxima (columns k,
    # k+8, ...), then 8 -> 3 -> 1
    lvl = [a.r("f") for _ in range(8)]
    for k in range(8):
        col = list(range(k, BKV, 8))
        a(f"max.f32 {lvl[k]}, {s_[col[0]]}, {s_[col[1]]}, {s_[col[2]]};")
        rest = col[3:]
        while len(rest) >= 2:
            a(f"max.f32 {lvl[k]}, {lvl[k]}, {s_[rest[0]]}, {s_[rest[1]]};")
            rest = rest[2:]
        if rest:
            a(f"max.f32 {lvl[k]}, {lvl[k]}, {s_[rest[0]]};")
    a(f"max.f32 {lvl[0]}, {lvl[0]}, {lvl[1]}, {lvl[2]};")
    a(f"max.f32 {lvl[3]}, {lvl[3]}, {lvl[4]}, {lvl[5]};")
    a(f"max.f32 {lvl[6]}, {lvl[6]}, {lvl[7]};")
    a(f"max.f32 {lvl[0]}, {lvl[0]}, {lvl[3]}, {lvl[6]};")
    mblk, mnew = a.r("f"), a.r("f")
    a(f"mul.f32 {mblk}, {lvl[0]}, {cscale};")
    a(f"max.f32 {mnew}, {mref}, {mblk};")
    # alpha (the O rescale factor) is 1 unless this block raises the running max past the
    # threshold; it is written on every path so every later read has a definition
    alpha = a.r("f")
    a(f"mov.b32 {alpha}, 0f3F800000;")
    l_first, l_after = a.L("first"), a.L("after")
    need, anyneed = a.r("p"), a.r("p")
    pfirst = a.r("p")
    a(f"setp.eq.u32 {pfirst}, {jj}, 0;")
    a(f"@{pfirst} bra {l_first};")
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
    negm = a.r("f")
    a(f"neg.f32 {negm}, {mref};")
    parts = [a.r("f") for _ in range(4)]
    for pp in parts:
        a(f"mov.b32 {pp}, 0f00000000;")
    cf, cp2, np2 = a.r("f"), a.r("rd"), a.r("rd")
    a(f"mov.b32 {cf}, {cscale};")
    a(f"mov.b64 {cp2}, {{{cf}, {cf}}};")
    a(f"mov.b64 {np2}, {{{negm}, {negm}}};")

    def exp_block(cols):
        """p = 2^(s*c - m) over ``cols`` (pairs: the scale and subtract as one f32x2 fma, the exps
        on the MUFU), summed into ``parts`` two at a time."""
        acc = [a.r("rd"), a.r("rd")]
        a(f"mov.b64 {acc[0]}, {{{parts[0]}, {parts[1]}}};")
        a(f"mov.b64 {acc[1]}, {{{parts[2]}, {parts[3]}}};")
        for k, idx in enumerate(list(cols)[::2]):
            x0, x1 = s_[idx], s_[idx + 1]
            xp = a.r("rd")
            a(f"mov.b64 {xp}, {{{x0}, {x1}}};")
            a(f"fma.rn.f32x2 {xp}, {xp}, {cp2}, {np2};")
            a(f"mov.b64 {{{x0}, {x1}}}, {xp};")
            a(f"ex2.approx.ftz.f32 {x0}, {x0};")
            a(f"ex2.approx.ftz.f32 {x1}, {x1};")
            ep = a.r("rd")
            a(f"mov.b64 {ep}, {{{x0}, {x1}}};")
            a(f"add.rn.f32x2 {acc[k & 1]}, {acc[k & 1]}, {ep};")
        a(f"mov.b64 {{{parts[0]}, {parts[1]}}}, {acc[0]};")
        a(f"mov.b64 {{{parts[2]}, {parts[3]}}}, {acc[1]};")

    l_pdone = a.L("pdone")
    turn_wait()
    half_n = BKV // 2
    if half:
        l_pbf = a.L("pbf")
        a(f"@!{p16} bra {l_pbf};")

        def pack_store(pairs, col):
            hw = []
            for k in pairs:
                w = a.r()
                a(f"cvt.rn.f16x2.f32 {w}, {s_[2 * k + 1]}, {s_[2 * k]};")
                hw.append(w)
            dsth = a.r()
            a(f"add.u32 {dsth}, {scol}, {col};")
            a(f"tcgen05.st.sync.aligned.32x32b.x{len(hw)}.b32 [{dsth}], {{{', '.join(hw)}}};")
        for h in range(2):
            # each half of the row is packed (f16 pairs, columns 32h .. 32h+31) and stored as soon as
            # its exps are done; the turn passes after the second half's exps (or its packing too,
            # with pack_in_turn)
            exp_block(range(half_n * h, half_n * (h + 1)))
            if h == 1 and not pack_in_turn:
                turn_pass()
            pack_store(range(half_n * h // 2, half_n * (h + 1) // 2), half_n * h // 2)
        if pack_in_turn:
            turn_pass()
        a(f"bra {l_pdone};")
        a.label(l_pbf)
    exp_block(range(BKV))
    turn_pass()
    # bf16 P_hi (columns 0-63) and the exact remainder's bf16 P_lo (64-127), both by truncation
    for h in range(2):
        hi_w, lo_w = [], []
        for k in range(half_n * h // 2, half_n * (h + 1) // 2):
            i0, i1 = 2 * k, 2 * k + 1
            w, h0, h1, wl = a.r(), a.r("f"), a.r("f"), a.r()
            a(f"prmt.b32 {w}, {s_[i0]}, {s_[i1]}, 0x7632;")
            a(f"and.b32 {h0}, {s_[i0]}, -65536;")
            a(f"and.b32 {h1}, {s_[i1]}, -65536;")
            a(f"sub.f32 {h0}, {s_[i0]}, {h0};")
            a(f"sub.f32 {h1}, {s_[i1]}, {h1};")
            a(f"prmt.b32 {wl}, {h0}, {h1}, 0x7632;")
            hi_w.append(w)
            lo_w.append(wl)
        dh, dl = a.r(), a.r()
        a(f"add.u32 {dh}, {scol}, {half_n * h // 2};")
        a(f"add.u32 {dl}, {scol}, {half_n + half_n * h // 2};")
        a(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{dh}], {{{', '.join(hi_w)}}};")
        a(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{dl}], {{{', '.join(lo_w)}}};")
    a.label(l_pdone)
    p01, p23 = a.r("f"), a.r("f")
    a(f"add.f32 {p01}, {parts[0]}, {parts[1]};")
    a(f"add.f32 {p23}, {parts[2]}, {parts[3]};")
    a(f"add.f32 {p01}, {p01}, {p23};")
    a(f"add.f32 {lsum}, {lsum}, {p01};")
    # the lazy O rescale, once the previous PV into O has completed
    l_norescale2 = a.L("norescale2")
    a(f"@!{anyneed} bra {l_norescale2};")
    prev = a.r()
    a(f"sub.u32 {prev}, {jj}, 1;")
    pv_done(prev, l_drain_post, ERR_SOFTMAX)
    a("tcgen05.fence::after_thread_sync;")
    for c in range(D // 32):
        src = a.r()
        a(f"add.u32 {src}, {ocol}, {32 * c};")
        regs = s_[:32]
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
    if pingpong:
        # after a time-out: the remaining blocks' turn hand-overs without their work (from block jj,
        # or from jj + 1 when block jj's were already made)
        l_dl = a.L("dloop")
        a.label(l_drain_post)
        a(f"add.u32 {jj}, {jj}, 1;")
        a.label(l_drain)
        a(f"mov.u32 {failed}, 1;")
        a.label(l_dl)
        pdx = a.r("p")
        a(f"setp.gt.u32 {pdx}, {jj}, {last};")
        a(f"@{pdx} bra {l_sdone};")
        turn_wait()
        turn_pass()
        a(f"add.u32 {jj}, {jj}, 1;")
        a(f"bra {l_dl};")
    a.label(l_sdone)
    # epilogue: after the last PV, O / l to global memory as bf16
    l_noepi = a.L("noepi")
    pok, pfl = a.r("p"), a.r("p")
    a(f"setp.le.u32 {pok}, {jj}, {last};")                  # left early (time-out): no store
    a(f"setp.ne.u32 {pfl}, {failed}, 0;")
    a(f"or.pred {pok}, {pok}, {pfl};")
    a(f"@{pok} bra {l_noepi};")
    pv_done(last, l_noepi, ERR_EPILOGUE)                    # the last PV, and so every earlier one
    a("tcgen05.fence::after_thread_sync;")
    inv = a.r("f")
    a(f"rcp.rn.f32 {inv}, {lsum};")
    grow, oaddr = a.r(), a.r("rd")
    a(f"mad.lo.u32 {grow}, {bh}, {seq}, {grow0};")         # row of O in [batch*heads*S, D]
    a(f"mul.wide.u32 {oaddr}, {grow}, {D * 2};")
    a(f"add.s64 {oaddr}, {oaddr}, {o_ptr};")
    for c in range(D // 32):
        src = a.r()
        a(f"add.u32 {src}, {ocol}, {32 * c};")
        regs = s_[:32]
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

    params = ["\t.param .u64 p_Q,", "\t.param .u64 p_K,", "\t.param .u64 p_V,", "\t.param .u64 p_O,"]
    if half:
        params += ["\t.param .u64 p_V16,", "\t.param .u64 p_vflag,"]
    params += ["\t.param .align 64 .b8 p_tmQ[128],", "\t.param .align 64 .b8 p_tmK[128],",
               "\t.param .align 64 .b8 p_tmV[128],"]
    if half:
        params.append("\t.param .align 64 .b8 p_tmV16[128],")
    params.append("\t.param .u64 p_err")
    entry = [f".visible .entry {name}("] + params + [")", f".reqntid {threads}, 1, 1",
                                                       f".maxnreg {REGS_LAUNCH}", "{"]
    entry += a.decls() + a.lines + ["\tret;", "}"]
    qn, kn, vn, on = names
    dims = [D, seq, heads, batch]
    strides = [D * 2, seq * D * 2, heads * seq * D * 2]
    tmaps = [{"name": "tmQ", "tensor": qn, "dtype": "bf16", "dims": dims, "strides": strides,
              "box": [64, BQ, 1, 1], "swizzle": "128B"}]
    tmaps += [{"name": f"tm{x}", "tensor": nm, "dtype": "bf16", "dims": dims, "strides": strides,
               "box": [64, BKV, 1, 1], "swizzle": "128B"} for x, nm in (("K", kn), ("V", vn))]
    uparams = [qn, kn, vn, on]
    if half:
        v16n, vfn = scratch_names or (f"{prefix}{name}__v16", f"{prefix}{name}__vflag")
        uparams += [v16n, vfn]
        tmaps.append({"name": "tmV16", "tensor": v16n, "dtype": "f16", "dims": dims, "strides": strides,
                      "box": [64, BKV, 1, 1], "swizzle": "128B"})
    return {
        "name": name, "kind": "tcgen05_attention", "params": uparams,
        "raw_entry": entry, "raw_decls": [f".extern .shared .align 1024 .b8 {smem_sym}[];"],
        "grid": [grid, 1, 1], "block": [threads, 1, 1], "dyn_smem": DYN_SMEM,
        "align": {qn: 16, kn: 16, vn: 16, on: 32, **({uparams[4]: 16, uparams[5]: 4} if half else {})},
        "zero_outputs": [], "tmaps": tmaps,
        "extra": [{"name": "__err", "kind": "errword"}],
    }
