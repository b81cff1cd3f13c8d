"""Persistent form of the tcgen05 causal / full attention (opt-in, ``attn_persistent``).

The same arithmetic as :mod:`.tc_attention` (QK^T and PV on the tensor cores with S, P and O in TMEM,
the online softmax one thread per row, f16 P with the value pre-pass's f16 V, or two bf16 parts of P
for blocks flagged as not fitting f16), scheduled differently:

* one CTA per SM walks a list of work units (256 query rows of one (batch, head)), the longest causal
  rows first, assigned zig-zag: CTA c takes unit k*P + c on even rounds k and k*P + (P-1-c) on odd
  ones (P CTAs), which balances the total work per CTA to within a fraction of a unit;
* the two softmax warpgroups swap the lower and the upper 128 rows on every unit (warpgroup w has the
  upper rows of its k-th unit when k + w is odd).  With causal masking the upper rows need two more
  64-row key/value blocks, so over each pair of units both warpgroups do the same number of blocks;
  their MUFU turns then pair across unit boundaries (one global turn sequence per warpgroup), and a
  warpgroup that finished its unit's lower rows starts its next unit while the other finishes the
  upper rows, at most two blocks behind (the K/V ring, 8 stages of 16 KiB, holds four blocks);
* warp 3 loads each warpgroup's Q tile for its next unit as soon as that warpgroup's last QK^T of the
  current unit has completed, and publishes the unit's f16/bf16 block flags as a 64-bit mask beside
  it; warp 0 streams K and V of all units through the ring without stopping between units;
* warpgroup w's O accumulator is reused once its epilogue has read the previous unit's O (an
  O-free barrier per warpgroup); scores and P stay double-buffered per warpgroup as before.

Every mbarrier wait is bounded.  A softmax warp that times out makes the rest of its warpgroup's
turn hand-overs without the work, so the other warpgroup is never left waiting on a named barrier.
"""
from __future__ import annotations

from .ptxasm import Asm, idesc_f16, smem_desc_hi, wait_bar, wait_bar_warp
from .tc_attention import (BKV, BQ, D, KV_BYTES, KV_HALF, LOG2E, Q_BYTES, Q_HALF, RESCALE_THRESHOLD, S_COL0,
                           STAGES, THREADS, TILES, TMEM_COLS, _f32)

# barrier offsets (bytes from the barrier area)
FULL = 0
EMPTY = FULL + 8 * STAGES
QFULL = EMPTY + 8 * STAGES          # [warpgroup]
QEMPTY = QFULL + 16                 # [warpgroup]
OFREE = QEMPTY + 16                 # [warpgroup]
SFULL = OFREE + 16                  # [warpgroup][buffer]
PFULL = SFULL + 32
PFREE = PFULL + 32
SLOT = PFREE + 32
MASKS = 512                         # 4 x 64-bit block-flag masks, by unit index mod 4
BAR_BYTES = 1024

ERR_PRODUCER, ERR_MMA, ERR_SOFTMAX, ERR_EPILOGUE, ERR_DRAIN, ERR_QLOAD = 21, 22, 23, 24, 25, 26


def persistent_attention_entry(name: str, batch: int, heads: int, seq: int, causal: bool, scale: float,
                               names=("Q", "K", "V", "O"), prefix: str = "", half: bool = True,
                               ctas: int = 148, scratch_names: tuple[str, str] | None = None) -> dict:
    """The kernel's launch record and PTX (``ctas`` CTAs, one per SM)."""
    if seq % (BQ * TILES):
        raise ValueError("tcgen05 attention needs S % 256 == 0")
    nblk = seq // BKV
    if half and nblk > 64:
        raise ValueError("the f16 path keeps a 64-bit block-flag mask per unit: S <= 4096")
    nt = seq // (BQ * TILES)
    nbh = batch * heads
    total = nbh * nt
    P = max(1, min(int(ctas), total))
    a = Asm()
    idesc_qk = idesc_f16(BQ, BKV, False, False)
    idesc_pv = idesc_f16(BQ, D, False, True)
    idesc_pv16 = idesc_f16(BQ, D, False, True, half=True)
    kdesc_hi = smem_desc_hi(16, 1024)
    vdesc_hi = smem_desc_hi(KV_HALF, 1024)
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
    # zig-zag mirror of this CTA for odd rounds
    ctam = a.r()
    a(f"sub.u32 {ctam}, {P - 1}, {cta};")

    raw, base = a.r(), a.r()
    smem_sym = f"{prefix}attn_smem"
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
    for s in range(STAGES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{FULL + 8 * s}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{EMPTY + 8 * s}], {TILES};")
    for w in range(TILES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{QFULL + 8 * w}], 1;")
        # Q-empty: the issuer's commit after its unit's last QK^T, and one arrival per softmax warp once
        # it has read the unit's flag mask, so Q-full can never run two phases ahead of a waiter
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{QEMPTY + 8 * w}], 5;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{OFREE + 8 * w}], 4;")
        for b_ in range(2):
            a(f"mbarrier.init.shared::cta.b64 [{bars}+{SFULL + 16 * w + 8 * b_}], 1;")
            a(f"mbarrier.init.shared::cta.b64 [{bars}+{PFULL + 16 * w + 8 * b_}], 4;")
            a(f"mbarrier.init.shared::cta.b64 [{bars}+{PFREE + 16 * w + 8 * b_}], 1;")
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
    l_prod, l_mma0, l_mma1, l_qld, l_soft = a.L("prod"), a.L("mma0"), a.L("mma1"), a.L("qld"), a.L("soft")
    pw0, pw2, pw3, pws = a.r("p"), a.r("p"), a.r("p"), a.r("p")
    a(f"setp.eq.u32 {pw0}, {warp}, 0;")
    a(f"setp.eq.u32 {pw2}, {warp}, 2;")
    a(f"setp.eq.u32 {pw3}, {warp}, 3;")
    a(f"setp.ge.u32 {pws}, {warp}, 4;")
    a(f"@{pw0} bra {l_prod};")
    a(f"@{pw1} bra {l_mma0};")
    a(f"@{pw2} bra {l_mma1};")
    a(f"@{pw3} bra {l_qld};")
    a(f"@{pws} bra {l_soft};")
    a(f"bra {l_end};")

    def unit(k, l_done):
        """The k-th unit of this CTA: branches to ``l_done`` past the last one; returns
        (t, bh, bb, hh, n_hi, n_lo, row0)."""
        u, t, bh, bb, hh = a.r(), a.r(), a.r(), a.r(), a.r()
        odd, who = a.r("p"), a.r()
        a(f"and.b32 {who}, {k}, 1;")
        a(f"setp.ne.u32 {odd}, {who}, 0;")
        a(f"selp.u32 {who}, {ctam}, {cta}, {odd};")
        a(f"mad.lo.u32 {u}, {k}, {P}, {who};")
        pdone = a.r("p")
        a(f"setp.ge.u32 {pdone}, {u}, {total};")
        a(f"@{pdone} bra {l_done};")
        a(f"div.u32 {t}, {u}, {nbh};")
        a(f"sub.u32 {t}, {nt - 1}, {t};")
        a(f"rem.u32 {bh}, {u}, {nbh};")
        a(f"div.u32 {bb}, {bh}, {heads};")
        a(f"rem.u32 {hh}, {bh}, {heads};")
        n_hi, n_lo, row0 = a.r(), a.r(), a.r()
        if causal:
            a(f"shl.b32 {n_hi}, {t}, 2;")
            a(f"add.u32 {n_hi}, {n_hi}, 4;")
            a(f"sub.u32 {n_lo}, {n_hi}, 2;")
        else:
            a(f"mov.u32 {n_hi}, {nblk};")
            a(f"mov.u32 {n_lo}, {nblk};")
        a(f"shl.b32 {row0}, {t}, 8;")
        return t, bh, bb, hh, n_hi, n_lo, row0

    def is_upper(k, w):
        """Predicate: warpgroup w has the upper 128 rows in its k-th unit."""
        x, p_ = a.r(), a.r("p")
        a(f"add.u32 {x}, {k}, {w};")
        a(f"and.b32 {x}, {x}, 1;")
        a(f"setp.ne.u32 {p_}, {x}, 0;")
        return p_

    def tma4(dst, tmap, c0, c1, hh, bb, mbar, guard=None):
        g = f"@{guard} " if guard else ""
        a(f"{g}cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
          f"[{dst}], [{tmap}, {{{c0}, {c1}, {hh}, {bb}}}], [{mbar}];")

    def flag_mask(bh, nb):
        """The unit's 64 block flags as a 64-bit mask (every lane of the warp takes part)."""
        vfp, vbase, m64 = a.r("rd"), a.r(), a.r("rd")
        a(f"ld.param.u64 {vfp}, [p_vflag];")
        a(f"cvta.to.global.u64 {vfp}, {vfp};")
        a(f"mul.lo.u32 {vbase}, {bh}, {nblk};")
        words = []
        for kx in range(2):
            bk, pk, fk, ga, pf, mw = a.r(), a.r("p"), a.r(), a.r("rd"), a.r("p"), a.r()
            a(f"add.u32 {bk}, {lane}, {32 * kx};")
            a(f"setp.lt.u32 {pk}, {bk}, {nb};")
            a(f"add.u32 {fk}, {vbase}, {bk};")
            a(f"mul.wide.u32 {ga}, {fk}, 4;")
            a(f"add.s64 {ga}, {ga}, {vfp};")
            a(f"mov.u32 {fk}, 0;")
            a(f"@{pk} ld.global.nc.u32 {fk}, [{ga}];")
            a(f"setp.ne.u32 {pf}, {fk}, 0;")
            a(f"vote.sync.ballot.b32 {mw}, {pf}, -1;")
            words.append(mw)
        a(f"mov.b64 {m64}, {{{words[0]}, {words[1]}}};")
        return m64

    def mask_bit(m64, j):
        """Predicate: block j is flagged (bit j of the mask)."""
        sh, lo, p_ = a.r("rd"), a.r(), a.r("p")
        a(f"shr.b64 {sh}, {m64}, {j};")
        a(f"cvt.u32.u64 {lo}, {sh};")
        a(f"and.b32 {lo}, {lo}, 1;")
        a(f"setp.ne.u32 {p_}, {lo}, 0;")
        return p_

    # ---------------- warp 0: K / V ring over all units ------------------------------------
    a.label(l_prod)
    k0, stage, phase = a.r(), a.r(), a.r()
    armed = [a.r() for _ in range(STAGES)]
    for r_ in armed:
        a(f"mov.u32 {r_}, 2;")
    a(f"mov.u32 {k0}, 0;")
    a(f"mov.u32 {stage}, 0;")
    a(f"mov.u32 {phase}, 0;")
    ple0 = a.r("p")
    a(f"setp.eq.u32 {ple0}, {lane}, 0;")
    l_pu, l_pdone = a.L("pu"), a.L("pdone")
    a.label(l_pu)
    _, _, bbp, hhp, nhp, _, _ = unit(k0, l_pdone)
    bhp = a.r()
    a(f"mad.lo.u32 {bhp}, {bbp}, {heads}, {hhp};")
    m64p = flag_mask(bhp, nhp) if half else None
    n_, nitems = a.r(), a.r()
    a(f"mov.u32 {n_}, 0;")
    a(f"shl.b32 {nitems}, {nhp}, 1;")
    l_pl, l_pnext = a.L("pl"), a.L("pnext")
    a.label(l_pl)
    pend = a.r("p")
    a(f"setp.ge.u32 {pend}, {n_}, {nitems};")
    a(f"@{pend} bra {l_pnext};")
    fb, eb, par = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {fb}, {stage}, 8, {bars};")
    a(f"add.u32 {eb}, {fb}, {EMPTY};")
    a(f"add.u32 {fb}, {fb}, {FULL};")
    a(f"xor.b32 {par}, {phase}, 1;")
    wait_bar_warp(a, eb, par, err, ERR_PRODUCER, l_pdone)
    a(f"@{ple0} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {KV_BYTES};")
    for s in range(STAGES):
        ps = a.r("p")
        a(f"setp.eq.u32 {ps}, {stage}, {s};")
        a(f"@{ps} mov.u32 {armed[s]}, {phase};")
    jv, kvrow, dst, isv, andn = a.r(), a.r(), a.r(), a.r("p"), a.r()
    a(f"shr.u32 {jv}, {n_}, 1;")
    a(f"shl.b32 {kvrow}, {jv}, 6;")
    a(f"mad.lo.u32 {dst}, {stage}, {KV_BYTES}, {sKV};")
    a(f"and.b32 {andn}, {n_}, 1;")
    a(f"setp.ne.u32 {isv}, {andn}, 0;")
    tsel = a.r("rd")
    if half:
        flagged = mask_bit(m64p, jv)
        tvs = a.r("rd")
        a(f"selp.b64 {tvs}, {tv}, {tv16}, {flagged};")
        a(f"selp.b64 {tsel}, {tvs}, {tk}, {isv};")
    else:
        a(f"selp.b64 {tsel}, {tv}, {tk}, {isv};")
    tma4(dst, tsel, 0, kvrow, hhp, bbp, fb, ple0)
    dst2 = a.r()
    a(f"add.u32 {dst2}, {dst}, {KV_HALF};")
    tma4(dst2, tsel, 64, kvrow, hhp, bbp, fb, ple0)
    pwr = a.r("p")
    a(f"add.u32 {stage}, {stage}, 1;")
    a(f"setp.eq.u32 {pwr}, {stage}, {STAGES};")
    a(f"@{pwr} mov.u32 {stage}, 0;")
    a(f"@{pwr} xor.b32 {phase}, {phase}, 1;")
    a(f"add.u32 {n_}, {n_}, 1;")
    a(f"bra {l_pl};")
    a.label(l_pnext)
    a(f"add.u32 {k0}, {k0}, 1;")
    a(f"bra {l_pu};")
    a.label(l_pdone)
    # the producer's own loads in flight land before the CTA ends (bounded)
    for s in range(STAGES):
        skip = a.L("dskip")
        pn = a.r("p")
        a(f"setp.eq.u32 {pn}, {armed[s]}, 2;")
        a(f"@{pn} bra {skip};")
        fbs = a.r()
        a(f"add.u32 {fbs}, {bars}, {FULL + 8 * s};")
        wait_bar_warp(a, fbs, armed[s], err, ERR_DRAIN, skip)
        a.label(skip)
    a(f"bra {l_end};")

    # ---------------- warp 3: Q tiles and block-flag masks ---------------------------------
    a.label(l_qld)
    k3, last_k3 = a.r(), a.r()
    a(f"mov.u32 {k3}, 0;")
    a(f"mov.u32 {last_k3}, 0;")
    ple3 = a.r("p")
    a(f"setp.eq.u32 {ple3}, {lane}, 0;")
    l_qu, l_qdone = a.L("qu"), a.L("qdone")
    a.label(l_qu)
    _, _, bbq, hhq, nhq, _, row0q = unit(k3, l_qdone)
    a(f"add.u32 {last_k3}, {k3}, 1;")
    pq = a.r()
    a(f"add.u32 {pq}, {k3}, 1;")
    a(f"and.b32 {pq}, {pq}, 1;")                       # parity of the previous unit's phase
    # the warpgroup with the upper rows in unit k had the lower rows in unit k-1: its Q frees first
    for order in range(2):
        l_w1, l_wnext = a.L("qw1"), a.L("qwnext")
        first_is_1 = a.r("p")
        kk_ = a.r()
        a(f"and.b32 {kk_}, {k3}, 1;")
        a(f"setp.eq.u32 {first_is_1}, {kk_}, 0;")      # k even: warpgroup 1 has the upper rows
        if order == 1:
            a(f"not.pred {first_is_1}, {first_is_1};")
        for w in range(TILES):
            l_skipw = a.L("qskip")
            if w == 0:
                a(f"@{first_is_1} bra {l_skipw};")
            else:
                a(f"@!{first_is_1} bra {l_skipw};")
            qeb = a.r()
            a(f"add.u32 {qeb}, {bars}, {QEMPTY + 8 * w};")
            wait_bar_warp(a, qeb, pq, err, ERR_QLOAD, l_qdone)
            up = is_upper(k3, w)
            rq = a.r()
            a(f"selp.u32 {rq}, 128, 0, {up};")
            a(f"add.u32 {rq}, {rq}, {row0q};")
            qfb = a.r()
            a(f"add.u32 {qfb}, {bars}, {QFULL + 8 * w};")
            if order == 0 and half:
                # the unit's flags, published with the first Q tile's arrival
                bhq = a.r()
                a(f"mad.lo.u32 {bhq}, {bbq}, {heads}, {hhq};")
                m64 = flag_mask(bhq, nhq)
                ma, ks = a.r(), a.r()
                a(f"and.b32 {ks}, {k3}, 3;")
                a(f"mad.lo.u32 {ma}, {ks}, 8, {bars};")
                a(f"@{ple3} st.shared.b64 [{ma}+{MASKS}], {m64};")
            a(f"@{ple3} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{qfb}], {Q_BYTES};")
            for hb in range(2):
                d_ = a.r()
                a(f"add.u32 {d_}, {sQ}, {Q_BYTES * w + Q_HALF * hb};")
                tma4(d_, tq, 64 * hb, rq, hhq, bbq, qfb, ple3)
            a(f"bra {l_wnext};")
            a.label(l_skipw)
        a.label(l_wnext)
    a(f"add.u32 {k3}, {k3}, 1;")
    a(f"bra {l_qu};")
    a.label(l_qdone)
    # the last unit's Q loads land before the CTA ends (bounded)
    pnone = a.r("p")
    a(f"setp.eq.u32 {pnone}, {last_k3}, 0;")
    l_qend = a.L("qend")
    a(f"@{pnone} bra {l_qend};")
    lpar = a.r()
    a(f"sub.u32 {lpar}, {last_k3}, 1;")
    a(f"and.b32 {lpar}, {lpar}, 1;")
    for w in range(TILES):
        qfb2 = a.r()
        a(f"add.u32 {qfb2}, {bars}, {QFULL + 8 * w};")
        wait_bar_warp(a, qfb2, lpar, err, ERR_DRAIN, l_qend)
    a.label(l_qend)
    a(f"bra {l_end};")

    # ---------------- warps 1, 2: MMA issuers (one thread each) -----------------------------
    def issuer(w, l_label):
        a.label(l_label)
        pl = a.r("p")
        a(f"setp.ne.u32 {pl}, {lane}, 0;")
        a(f"@{pl} bra {l_end};")
        l_mdone = a.L(f"mdone{w}")
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

        def base_desc(addr_reg, hi):
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

        qb_w = a.r()
        a(f"add.u32 {qb_w}, {sQ}, {Q_BYTES * w};")
        q0 = base_desc(qb_w, khi)
        qdesc = [plus(q0, (k // 4) * Q_HALF + (k % 4) * 32) for k in range(D // 16)]
        kd, vd = [], []
        for st_ in range(STAGES):
            sb = a.r()
            a(f"add.u32 {sb}, {sKV}, {st_ * KV_BYTES};")
            kd.append(base_desc(sb, khi))
            vd.append(base_desc(sb, vhi))
        scol_c = [a.r() for _ in range(2)]
        ocol_c = a.r()
        a(f"add.u32 {ocol_c}, {taddr}, {D * w};")
        for b_ in range(2):
            a(f"add.u32 {scol_c[b_]}, {taddr}, {S_COL0 + 2 * BKV * w + BKV * b_};")

        k_, gp, gpn, pb, j, lasti, nb = a.r(), a.r(), a.r(), a.r(), a.r(), a.r(), a.r()
        a(f"mov.u32 {k_}, 0;")
        a(f"mov.u32 {gp}, 0;")
        a(f"mov.u32 {pb}, 0;")
        m64 = a.r("rd")
        a(f"mov.u64 {m64}, 0;")

        def ring_wait(stage_c, par):
            wait_bar(a, f"{bars}+{FULL + 8 * stage_c}", par, err, ERR_MMA, l_mdone)
            a("tcgen05.fence::after_thread_sync;")

        def qk(stage_c, buf_c):
            for k in range(D // 16):
                db = plus(kd[stage_c], (k // 4) * KV_HALF + (k % 4) * 32)
                a(f"tcgen05.mma.cta_group::1.kind::f16 [{scol_c[buf_c]}], {qdesc[k]}, {db}, {iqk}, "
                  f"{ptrue if k else pfalse};")
            a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bars}+{SFULL + 16 * w + 8 * buf_c}];")

        def release(stage_c, used):
            if used:
                a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
                  f"[{bars}+{EMPTY + 8 * stage_c}];")
            else:
                a(f"mbarrier.arrive.shared::cta.b64 _, [{bars}+{EMPTY + 8 * stage_c}];")

        def pv(stage_c, buf_c, u):
            vds = [plus(vd[stage_c], 2048 * k) for k in range(BKV // 16)]
            pacc = a.r("p")
            a(f"setp.ne.u32 {pacc}, {j}, 0;")
            # a new unit's first PV overwrites O: its previous contents must have been read out
            l_nofree = a.L("nofree")
            a(f"@{pacc} bra {l_nofree};")
            ofp = a.r()
            a(f"add.u32 {ofp}, {k_}, 1;")
            a(f"and.b32 {ofp}, {ofp}, 1;")
            wait_bar(a, f"{bars}+{OFREE + 8 * w}", ofp, err, ERR_MMA, l_mdone)
            a.label(l_nofree)
            pfpar = a.r()
            a(f"xor.b32 {pfpar}, {pb}, {(u >> 1) & 1};")
            wait_bar(a, f"{bars}+{PFULL + 16 * w + 8 * buf_c}", pfpar, err, ERR_MMA, l_mdone)
            a("tcgen05.fence::after_thread_sync;")
            l_bf, l_done = a.L("pvbf"), a.L("pvdone")
            if half:
                flagged = mask_bit(m64, j)
                a(f"@{flagged} bra {l_bf};")
                for k in range(BKV // 16):
                    acc = pacc if k == 0 else ptrue
                    a(f"tcgen05.mma.cta_group::1.kind::f16 [{ocol_c}], [{scol_c[buf_c]}+{8 * k}], "
                      f"{vds[k]}, {ipv16}, {acc};")
                a(f"bra {l_done};")
            a.label(l_bf)
            for part in range(2):
                for k in range(BKV // 16):
                    acc = pacc if (k == 0 and part == 0) else ptrue
                    a(f"tcgen05.mma.cta_group::1.kind::f16 [{ocol_c}], "
                      f"[{scol_c[buf_c]}+{(BKV // 2) * part + 8 * k}], {vds[k]}, {ipv}, {acc};")
            a.label(l_done)
            a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bars}+{PFREE + 16 * w + 8 * buf_c}];")

        l_unit, l_unit_end = a.L(f"iu{w}"), a.L(f"iue{w}")
        a.label(l_unit)
        _, _, _, _, n_hi, n_lo, _ = unit(k_, l_mdone)
        up = is_upper(k_, w)
        a(f"mov.u32 {nb}, {n_hi};")
        a(f"selp.u32 {lasti}, {n_hi}, {n_lo}, {up};")
        a(f"sub.u32 {lasti}, {lasti}, 1;")
        qpar = a.r()
        a(f"and.b32 {qpar}, {k_}, 1;")
        wait_bar(a, f"{bars}+{QFULL + 8 * w}", qpar, err, ERR_MMA, l_mdone)
        a("tcgen05.fence::after_thread_sync;")
        if half:
            ks, ma = a.r(), a.r()
            a(f"and.b32 {ks}, {k_}, 3;")
            a(f"mad.lo.u32 {ma}, {ks}, 8, {bars};")
            a(f"ld.shared.b64 {m64}, [{ma}+{MASKS}];")
        # S(0) from K_0 (the unit's ring item 0, stage 0)
        a(f"mov.u32 {j}, 0;")
        ring_wait(0, gp)
        qk(0, 0)
        release(0, True)
        l_mg = a.L(f"mg{w}")
        a.label(l_mg)
        a(f"xor.b32 {gpn}, {gp}, 1;")
        for u in range(4):                                 # block j = 4g + u of the unit
            have_next, jn = a.r("p"), a.r()
            a(f"add.u32 {jn}, {j}, 1;")
            a(f"setp.lt.u32 {have_next}, {jn}, {nb};")
            l_nok = a.L("nok")
            a(f"@!{have_next} bra {l_nok};")
            ks_ = (2 * u + 2) % STAGES
            ring_wait(ks_, gpn if u == 3 else gp)
            l_qk, l_qkd = a.L("noqk"), a.L("qkd")
            pn_ = a.r("p")
            a(f"setp.gt.u32 {pn_}, {jn}, {lasti};")
            a(f"@{pn_} bra {l_qk};")
            qk(ks_, (u + 1) & 1)
            release(ks_, True)
            # after the unit's last QK^T, the Q tile may be reloaded for the next unit
            plq, l_noq = a.r("p"), a.L("noqe")
            a(f"setp.ne.u32 {plq}, {jn}, {lasti};")
            a(f"@{plq} bra {l_noq};")
            a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{bars}+{QEMPTY + 8 * w}];")
            a.label(l_noq)
            a(f"bra {l_qkd};")
            a.label(l_qk)
            release(ks_, False)
            a.label(l_qkd)
            a.label(l_nok)
            vs = 2 * u + 1
            ring_wait(vs, gp)
            l_pv, l_pvd = a.L("nopv"), a.L("pvd")
            pj_ = a.r("p")
            a(f"setp.gt.u32 {pj_}, {j}, {lasti};")
            a(f"@{pj_} bra {l_pv};")
            pv(vs, u & 1, u)
            release(vs, True)
            a(f"bra {l_pvd};")
            a.label(l_pv)
            release(vs, False)
            a.label(l_pvd)
            a(f"@!{have_next} bra {l_unit_end};")
            a(f"mov.u32 {j}, {jn};")
        a(f"mov.u32 {gp}, {gpn};")
        a(f"bra {l_mg};")
        a.label(l_unit_end)
        # a unit is a whole number of ring laps (8 items per 4 blocks), so the ring parity turns once
        # more; the S/P barrier parity turns with every odd pair count
        a(f"xor.b32 {gp}, {gp}, 1;")
        nm, hb_ = a.r(), a.r()
        a(f"add.u32 {nm}, {lasti}, 1;")
        a(f"shr.u32 {hb_}, {nm}, 1;")
        a(f"and.b32 {hb_}, {hb_}, 1;")
        a(f"xor.b32 {pb}, {pb}, {hb_};")
        a(f"add.u32 {k_}, {k_}, 1;")
        a(f"bra {l_unit};")
        a.label(l_mdone)
        a(f"bra {l_end};")

    issuer(0, l_mma0)
    issuer(1, l_mma1)

    # ---------------- warps 4-11: softmax warpgroups ----------------------------------------------
    a.label(l_soft)
    wg, q, rowl = a.r(), a.r(), a.r()
    a(f"sub.u32 {wg}, {warp}, 4;")
    a(f"shr.u32 {wg}, {wg}, 2;")
    a(f"and.b32 {q}, {warp}, 3;")
    a(f"mad.lo.u32 {rowl}, {q}, 32, {lane};")
    lanebase = a.r()
    a(f"shl.b32 {lanebase}, {q}, 21;")
    a(f"add.u32 {lanebase}, {lanebase}, {taddr};")
    scol0, ocol = a.r(), a.r()
    a(f"mad.lo.u32 {scol0}, {wg}, {2 * BKV}, {lanebase};")
    a(f"add.u32 {scol0}, {scol0}, {S_COL0};")
    a(f"mad.lo.u32 {ocol}, {wg}, {D}, {lanebase};")
    sfb0, pfb0, pfr0 = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {sfb0}, {wg}, 16, {bars};")
    a(f"add.u32 {pfb0}, {sfb0}, {PFULL};")
    a(f"add.u32 {pfr0}, {sfb0}, {PFREE};")
    a(f"add.u32 {sfb0}, {sfb0}, {SFULL};")
    qfw, ofw = a.r(), a.r()
    a(f"mad.lo.u32 {qfw}, {wg}, 8, {bars};")
    a(f"add.u32 {ofw}, {qfw}, {OFREE};")
    a(f"add.u32 {qfw}, {qfw}, {QFULL};")
    ple = a.r("p")
    a(f"setp.eq.u32 {ple}, {lane}, 0;")
    tile0 = a.r("p")
    a(f"setp.eq.u32 {tile0}, {wg}, 0;")

    # both warpgroups' total blocks over this CTA's units (the turn sequence's lengths)
    T0, T1, kt = a.r(), a.r(), a.r()
    a(f"mov.u32 {T0}, 0;")
    a(f"mov.u32 {T1}, 0;")
    a(f"mov.u32 {kt}, 0;")
    l_tu, l_tdone = a.L("tu"), a.L("tdone")
    a.label(l_tu)
    _, _, _, _, nht, nlt, _ = unit(kt, l_tdone)
    ev, n0t, n1t = a.r("p"), a.r(), a.r()
    par_t = a.r()
    a(f"and.b32 {par_t}, {kt}, 1;")
    a(f"setp.eq.u32 {ev}, {par_t}, 0;")                 # even unit: warpgroup 0 has the lower rows
    a(f"selp.u32 {n0t}, {nlt}, {nht}, {ev};")
    a(f"selp.u32 {n1t}, {nht}, {nlt}, {ev};")
    a(f"add.u32 {T0}, {T0}, {n0t};")
    a(f"add.u32 {T1}, {T1}, {n1t};")
    a(f"add.u32 {kt}, {kt}, 1;")
    a(f"bra {l_tu};")
    a.label(l_tdone)
    Town, sync_lim, pass_lim = a.r(), a.r(), a.r()
    a(f"selp.u32 {Town}, {T0}, {T1}, {tile0};")
    # warpgroup 0 waits for its turn while turn kk <= T1 and passes while kk < T1; warpgroup 1
    # waits while kk < T0 and passes while kk + 1 < T0 (after an opening arrival)
    a(f"add.u32 {sync_lim}, {T1}, 1;")
    a(f"selp.u32 {sync_lim}, {sync_lim}, {T0}, {tile0};")
    a(f"sub.u32 {pass_lim}, {T0}, 1;")
    a(f"selp.u32 {pass_lim}, {T1}, {pass_lim}, {tile0};")
    l_noopen = a.L("noopen")
    popen = a.r("p")
    a(f"setp.eq.u32 {popen}, {T0}, 0;")
    a(f"@{tile0} bra {l_noopen};")
    a(f"@{popen} bra {l_noopen};")
    a("bar.arrive 1, 256;")                              # warpgroup 0 goes first
    a.label(l_noopen)

    kk, failed = a.r(), a.r()
    a(f"mov.u32 {kk}, 0;")
    a(f"mov.u32 {failed}, 0;")

    def turn_wait():
        ps_, l_ = a.r("p"), a.L("tw")
        a(f"setp.ge.u32 {ps_}, {kk}, {sync_lim};")
        a(f"@{ps_} bra {l_};")
        a(f"@{tile0} bar.sync 1, 256;")
        a(f"@!{tile0} bar.sync 2, 256;")
        a.label(l_)

    def turn_pass():
        pp_, l_ = a.r("p"), a.L("tp")
        a(f"setp.ge.u32 {pp_}, {kk}, {pass_lim};")
        a(f"@{pp_} bra {l_};")
        a(f"@{tile0} bar.arrive 2, 256;")
        a(f"@!{tile0} bar.arrive 1, 256;")
        a.label(l_)

    s_ = [a.r("f") for _ in range(BKV)]
    mref, lsum = a.r("f"), a.r("f")
    a(f"mov.b32 {mref}, 0fFF800000;")
    a(f"mov.b32 {lsum}, 0f00000000;")
    l_drain, l_drain_post, l_sall = a.L("drain"), a.L("drainpost"), a.L("sall")
    ks, pbs, jj, last, grow0 = a.r(), a.r(), a.r(), a.r(), a.r()
    a(f"mov.u32 {ks}, 0;")
    a(f"mov.u32 {pbs}, 0;")
    a(f"mov.u32 {jj}, 0;")
    a(f"mov.u32 {last}, 0;")
    a(f"mov.u32 {grow0}, 0;")
    m64s = a.r("rd")
    a(f"mov.u64 {m64s}, 0;")
    l_su, l_sunit_end = a.L("su"), a.L("sue")
    a.label(l_su)
    ts, bhs_, bbs, hhs, nhs, nls, row0s = unit(ks, l_sall)
    bhs = a.r()
    a(f"mad.lo.u32 {bhs}, {bbs}, {heads}, {hhs};")
    ups = a.r("p")
    xk = a.r()
    a(f"add.u32 {xk}, {ks}, {wg};")
    a(f"and.b32 {xk}, {xk}, 1;")
    a(f"setp.ne.u32 {ups}, {xk}, 0;")
    a(f"selp.u32 {last}, {nhs}, {nls}, {ups};")
    a(f"sub.u32 {last}, {last}, 1;")
    rup = a.r()
    a(f"selp.u32 {rup}, 128, 0, {ups};")
    a(f"add.u32 {grow0}, {row0s}, {rup};")
    a(f"add.u32 {grow0}, {grow0}, {rowl};")              # this thread's query row
    if half:
        qps = a.r()
        a(f"and.b32 {qps}, {ks}, 1;")
        wait_bar_warp(a, qfw, qps, err, ERR_SOFTMAX, l_drain)
        k4, ma = a.r(), a.r()
        a(f"and.b32 {k4}, {ks}, 3;")
        a(f"mad.lo.u32 {ma}, {k4}, 8, {bars};")
        a(f"ld.shared.b64 {m64s}, [{ma}+{MASKS}];")
    qeb_s = a.r()
    a(f"add.u32 {qeb_s}, {qfw}, {QEMPTY - QFULL};")
    a("bar.warp.sync -1;")
    a(f"@{ple} mbarrier.arrive.shared::cta.b64 _, [{qeb_s}];")
    a(f"mov.b32 {mref}, 0fFF800000;")
    a(f"mov.b32 {lsum}, 0f00000000;")
    a(f"mov.u32 {jj}, 0;")

    def pv_done(blk, bail, code):
        bb_, br_, pr_ = a.r(), a.r(), a.r()
        a(f"and.b32 {bb_}, {blk}, 1;")
        a(f"mad.lo.u32 {br_}, {bb_}, 8, {pfr0};")
        a(f"shr.u32 {pr_}, {blk}, 1;")
        a(f"xor.b32 {pr_}, {pr_}, {pbs};")
        a(f"and.b32 {pr_}, {pr_}, 1;")
        wait_bar_warp(a, br_, pr_, err, code, bail)

    l_sj = a.L("sj")
    a.label(l_sj)
    pj = a.r("p")
    a(f"setp.gt.u32 {pj}, {jj}, {last};")
    a(f"@{pj} bra {l_sunit_end};")
    bsel, sfb, pfb, par_s, scol = a.r(), a.r(), a.r(), a.r(), a.r()
    a(f"and.b32 {bsel}, {jj}, 1;")
    a(f"mad.lo.u32 {sfb}, {bsel}, 8, {sfb0};")
    a(f"mad.lo.u32 {pfb}, {bsel}, 8, {pfb0};")
    a(f"shr.u32 {par_s}, {jj}, 1;")
    a(f"xor.b32 {par_s}, {par_s}, {pbs};")
    a(f"and.b32 {par_s}, {par_s}, 1;")
    a(f"mad.lo.u32 {scol}, {bsel}, {BKV}, {scol0};")
    wait_bar_warp(a, sfb, par_s, err, ERR_SOFTMAX, l_drain)
    p16 = None
    if half:
        fl = mask_bit(m64s, jj)
        p16 = a.r("p")
        a(f"not.pred {p16}, {fl};")
    a("tcgen05.fence::after_thread_sync;")
    for c in range(BKV // 32):
        src = a.r()
        a(f"add.u32 {src}, {scol}, {32 * c};")
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(s_[32 * c:32 * c + 32])}}}, [{src}];")
    a("tcgen05.wait::ld.sync.aligned;")
    if causal:
        l_nomask = a.L("nomask")
        lim, kv0 = a.r(), a.r()
        a(f"shl.b32 {kv0}, {jj}, 6;")
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
    alpha = a.r("f")
    a(f"mov.b32 {alpha}, 0f3F800000;")
    l_first, l_after = a.L("first"), a.L("after")
    need, anyneed, pfirst = a.r("p"), a.r("p"), a.r("p")
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

    def exp_block(cols):
        cols = list(cols)
        cf, cp2, np2 = a.r("f"), a.r("rd"), a.r("rd")
        a(f"mov.b32 {cf}, {cscale};")
        a(f"mov.b64 {cp2}, {{{cf}, {cf}}};")
        a(f"mov.b64 {np2}, {{{negm}, {negm}}};")
        acc = [a.r("rd"), a.r("rd")]
        a(f"mov.b64 {acc[0]}, {{{parts[0]}, {parts[1]}}};")
        a(f"mov.b64 {acc[1]}, {{{parts[2]}, {parts[3]}}};")
        for k, idx in enumerate(cols[::2]):
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

    l_pdn = a.L("pdn")
    turn_wait()
    if half:
        l_pbf = a.L("pbf")
        a(f"@!{p16} bra {l_pbf};")
        half_n = BKV // 2
        for h in range(2):
            exp_block(range(half_n * h, half_n * (h + 1)))
            if h == 1:
                turn_pass()
            hw = []
            for k in range(half_n * h // 2, half_n * (h + 1) // 2):
                w_ = a.r()
                a(f"cvt.rn.f16x2.f32 {w_}, {s_[2 * k + 1]}, {s_[2 * k]};")
                hw.append(w_)
            dsth = a.r()
            a(f"add.u32 {dsth}, {scol}, {len(hw) * h};")
            a(f"tcgen05.st.sync.aligned.32x32b.x16.b32 [{dsth}], {{{', '.join(hw)}}};")
        a(f"bra {l_pdn};")
        a.label(l_pbf)
    exp_block(range(BKV))
    turn_pass()
    hi_w, lo_w = [], []
    for k in range(BKV // 2):
        i0, i1 = 2 * k, 2 * k + 1
        w_, h0, h1, wl = a.r(), a.r("f"), a.r("f"), a.r()
        a(f"prmt.b32 {w_}, {s_[i0]}, {s_[i1]}, 0x7632;")
        a(f"and.b32 {h0}, {s_[i0]}, -65536;")
        a(f"and.b32 {h1}, {s_[i1]}, -65536;")
        a(f"sub.f32 {h0}, {s_[i0]}, {h0};")
        a(f"sub.f32 {h1}, {s_[i1]}, {h1};")
        a(f"prmt.b32 {wl}, {h0}, {h1}, 0x7632;")
        hi_w.append(w_)
        lo_w.append(wl)
    a(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{scol}], {{{', '.join(hi_w)}}};")
    dst2s = a.r()
    a(f"add.u32 {dst2s}, {scol}, {BKV // 2};")
    a(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{dst2s}], {{{', '.join(lo_w)}}};")
    a.label(l_pdn)
    p01, p23 = a.r("f"), a.r("f")
    a(f"add.f32 {p01}, {parts[0]}, {parts[1]};")
    a(f"add.f32 {p23}, {parts[2]}, {parts[3]};")
    a(f"add.f32 {p01}, {p01}, {p23};")
    a(f"add.f32 {lsum}, {lsum}, {p01};")
    l_nores2 = a.L("nores2")
    a(f"@!{anyneed} bra {l_nores2};")
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
    a.label(l_nores2)
    a("tcgen05.wait::st.sync.aligned;")
    a("tcgen05.fence::before_thread_sync;")
    a("bar.warp.sync -1;")
    a(f"@{ple} mbarrier.arrive.shared::cta.b64 _, [{pfb}];")
    a(f"add.u32 {jj}, {jj}, 1;")
    a(f"add.u32 {kk}, {kk}, 1;")
    a(f"bra {l_sj};")

    a.label(l_sunit_end)
    # epilogue of the unit: after its last PV, O / l to global memory as bf16; O's columns are
    # handed back to the issuer as soon as they have been read
    pv_done(last, l_drain, ERR_EPILOGUE)
    a("tcgen05.fence::after_thread_sync;")
    inv = a.r("f")
    a(f"rcp.rn.f32 {inv}, {lsum};")
    grow, oaddr = a.r(), a.r("rd")
    a(f"mad.lo.u32 {grow}, {bhs}, {seq}, {grow0};")
    a(f"mul.wide.u32 {oaddr}, {grow}, {D * 2};")
    a(f"add.s64 {oaddr}, {oaddr}, {o_ptr};")
    for c in range(D // 32):
        src = a.r()
        a(f"add.u32 {src}, {ocol}, {32 * c};")
        regs = s_[:32]
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{src}];")
        a("tcgen05.wait::ld.sync.aligned;")
        if c == D // 32 - 1:
            a("tcgen05.fence::before_thread_sync;")
            a("bar.warp.sync -1;")
            a(f"@{ple} mbarrier.arrive.shared::cta.b64 _, [{ofw}];")
        words = []
        for k in range(16):
            w_ = a.r()
            a(f"mul.f32 {regs[2 * k]}, {regs[2 * k]}, {inv};")
            a(f"mul.f32 {regs[2 * k + 1]}, {regs[2 * k + 1]}, {inv};")
            a(f"cvt.rn.bf16x2.f32 {w_}, {regs[2 * k + 1]}, {regs[2 * k]};")
            words.append(w_)
        a(f"st.global.v8.b32 [{oaddr}+{64 * c}], {{{', '.join(words[:8])}}};")
        a(f"st.global.v8.b32 [{oaddr}+{64 * c + 32}], {{{', '.join(words[8:])}}};")
    nm2, hb2 = a.r(), a.r()
    a(f"add.u32 {nm2}, {last}, 1;")
    a(f"shr.u32 {hb2}, {nm2}, 1;")
    a(f"and.b32 {hb2}, {hb2}, 1;")
    a(f"xor.b32 {pbs}, {pbs}, {hb2};")
    a(f"add.u32 {ks}, {ks}, 1;")
    a(f"bra {l_su};")

    # after a time-out: the rest of this warpgroup's turn hand-overs without the work (from turn kk,
    # or kk + 1 when turn kk's were made)
    l_dl = a.L("dloop")
    a.label(l_drain_post)
    a(f"add.u32 {kk}, {kk}, 1;")
    a.label(l_drain)
    a(f"mov.u32 {failed}, 1;")
    a.label(l_dl)
    pdx = a.r("p")
    a(f"setp.ge.u32 {pdx}, {kk}, {Town};")
    a(f"@{pdx} bra {l_sall};")
    turn_wait()
    turn_pass()
    a(f"add.u32 {kk}, {kk}, 1;")
    a(f"bra {l_dl};")
    a.label(l_sall)

    # ---------------- teardown ---------------------------------------------------------------
    a.label(l_end)
    a("barrier.sync 0;")
    a("bar.warp.sync -1;")
    l_nodealloc = a.L("nodealloc")
    a(f"@!{pw1} bra {l_nodealloc};")
    a("tcgen05.fence::after_thread_sync;")
    a(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {taddr}, {TMEM_COLS};")
    a.label(l_nodealloc)

    dyn = TILES * Q_BYTES + STAGES * KV_BYTES + BAR_BYTES + 1024
    params = ["\t.param .u64 p_Q,", "\t.param .u64 p_K,", "\t.param .u64 p_V,", "\t.param .u64 p_O,"]
    if half:
        params += ["\t.param .u64 p_V16,", "\t.param .u64 p_vflag,"]
    params += ["\t.param .align 64 .b8 p_tmQ[128],", "\t.param .align 64 .b8 p_tmK[128],",
               "\t.param .align 64 .b8 p_tmV[128],"]
    if half:
        params.append("\t.param .align 64 .b8 p_tmV16[128],")
    params.append("\t.param .u64 p_err")
    threads = THREADS
    entry = [f".visible .entry {name}("] + params + [")", f".reqntid {threads}, 1, 1",
                                                       f".maxnreg {65536 // threads // 8 * 8}", "{"]
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
        "grid": [P, 1, 1], "block": [threads, 1, 1], "dyn_smem": dyn,
        "align": {qn: 16, kn: 16, vn: 16, on: 32, **({uparams[4]: 16, uparams[5]: 4} if half else {})},
        "zero_outputs": [], "tmaps": tmaps, "extra": [{"name": "__err", "kind": "errword"}],
    }
