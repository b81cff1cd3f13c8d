"""Causal / full attention on the 5th-generation tensor cores: QK^T and PV with tcgen05, S, P and O in TMEM.

O = softmax(Q K^T * scale [+ causal mask]) V for Q, K, V, O bf16 [batch, heads, S, D] (D = 128 below; 64 and
32 shrink the tiles, see ``attention_entry``) — the online-softmax
Accum loop nest of the attention IR (config 5).  One CTA owns 256 query rows of one (batch, head) as two
128-row tiles and walks the key/value sequence in 64-row blocks:

* warp 0 issues TMA: both Q tiles once, then K_0, V_0, K_1, V_1, ... through an 8-stage ring of 16 KiB;
* warp 1 owns TMEM; one thread of warp 1 issues tile 0's ``tcgen05.mma`` and one thread of warp 2
  tile 1's, so one issuer's waits and bookkeeping overlap the other's MMAs (the tensor core's
  instruction queue is shallow).  TMEM holds O_0 | O_1 (128 columns each) and, per tile, two
  64-column score buffers S_i[0], S_i[1]: the scores of block j+1 are computed into the other
  buffer while the softmax of block j runs, so a tile's softmax never waits for its own previous
  PV.  Per block j each issuer runs S_i(j+1) (M=128, N=64, K=128, both operands K-major in shared
  memory), then O_i += P_i(j) V_j (M=128, N=128, K=64, P read from TMEM, V MN-major in shared
  memory);
* warps 4-7 (tile 0) and 8-11 (tile 1) run the online softmax, one thread per row: load the row of
  S_i(j) from TMEM, mask the diagonal blocks, take the row max, compute p = 2^(s*scale*log2e - m)
  with the MUFU ``ex2``, accumulate the row sum, and write P over the same TMEM columns.  O is
  rescaled in TMEM only when a row's running max grew by more than 2^8 (a stale max is exact as
  long as P and the row sum use the same one), after the previous PV has completed;
* blocks above the diagonal are never computed; CTAs start with the longest rows.

The tensor core multiplies operands of one type.  By default (``half``) the value pre-pass
(:mod:`.vconv`, a separate launch just before this kernel) writes an f16 copy of V and one flag per
64-row block; the producer loads a block's V from that copy when its flag is clear, the softmax writes P
in f16 (rounded to nearest, 2^-12 relative) and one PV pass runs f16 x f16.  A flagged block (some |v|
above 65,280, so it does not fit f16) is loaded from V itself and P is written as two bf16 parts,
P = P_hi + P_lo (p truncated to bf16, and the exact remainder truncated to bf16, taken with integer
masks and byte permutes), with two PV passes: p to within 2^-14.  The MMA accumulates both kinds into
the same f32 O, so the choice is per block.  Either way the result matches an f32-P computation to
within the output's bf16 rounding.  ``half=False`` uses the bf16 pair for every block;
``precise=False`` writes one bf16 P (rounded to nearest, 2^-9 relative error per term).

Every mbarrier wait is bounded (see :mod:`.ptxasm`); a time-out writes a code to the status word and
leaves the loop, the producer waits (bounded) for its own loads, and TMEM is always freed.
"""
from __future__ import annotations

from .ptxasm import Asm, idesc_f16, smem_desc_hi, wait_bar, wait_bar_warp

BQ = 128                         # query rows per tile
BKV = 64                         # key/value rows per block
D = 128
TILES = 2
STAGES = 8
Q_BYTES = BQ * D * 2             # 32 KiB: one Q tile
Q_HALF = Q_BYTES // 2            # one 64-column TMA box of a Q tile
KV_BYTES = BKV * D * 2           # 16 KiB: one K or V block
KV_HALF = KV_BYTES // 2          # one 64-column TMA box of a K/V block
THREADS = 384
TMEM_COLS = 512
F16_MAX_BF16_BITS = 0x477F       # the largest bf16 magnitude (65280) below the f16 overflow threshold
POLY_EVERY = 0                   # f16 path: every n-th exp2 on the FMA pipe (cubic); 0 = all on the MUFU, which measured fastest
# 2^f on [-1/2, 1/2] as c0 + c1 f + c2 f^2 + c3 f^3 (f32 bit patterns): a least-squares fit in relative
# error on 4000 Chebyshev nodes; evaluated by f32 Horner it stays within 7.8e-5 relative, below the
# f16 rounding of P (tests/test_emitter.py re-derives the bound)
EXP2_C = ("0f3F7FFB58", "0f3F317A8D", "0f3E786D32", "0f3D61A4AC")
S_COL0 = TILES * D               # S_i[b] at S_COL0 + 2*BKV*i + BKV*b
LOG2E = 1.4426950408889634
RESCALE_THRESHOLD = 8.0          # log2 units: rescale O only when the max grew by more than 2^8

ERR_PRODUCER, ERR_MMA, ERR_SOFTMAX, ERR_EPILOGUE, ERR_DRAIN = 11, 12, 13, 14, 15

# barrier offsets (bytes from the barrier area): QFULL, FULL[8], EMPTY[8], SFULL[tile][buf],
# PFULL[tile][buf], PFREE[tile][buf], then the TMEM address slot.  The S, P and PV-done handovers
# have one barrier per buffer: the softmax runs up to two blocks ahead of the PVs (its next scores
# are already computed), and a single barrier per tile could then be two phases away from a
# parity wait, which cannot tell those phases apart.
QFULL = 0
FULL = 8
EMPTY = FULL + 8 * STAGES
SFULL = EMPTY + 8 * STAGES
PFULL = SFULL + 8 * 2 * TILES
PFREE = PFULL + 8 * 2 * TILES
SLOT = PFREE + 8 * 2 * TILES
VFLAGS = 256                     # per kv block of this CTA: 1 when V did not fit f16 (64 words)
BAR_BYTES = 512

TRACE_SLOTS = 66                 # per-CTA trace rows: kv blocks 0..64, then one row of CTA facts
TRACE_EVENTS = 24


def _f32(v: float) -> str:
    import struct
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", v))[0]


def attention_entry(name: str, batch: int, heads: int, seq: int, causal: bool, scale: float,
                    names=("Q", "K", "V", "O"), prefix: str = "", precise: bool = True,
                    trace: bool = False, half: bool = True, poly_every: int = POLY_EVERY,
                    pingpong: bool = True, f16_int: int = 0, pack_after_turn: bool = False,
                    defer_sum: bool = False, bh_range: tuple[int, int] | None = None,
                    scratch_names: tuple[str, str] | None = None, prefetch_next: int = 0,
                    pack_in_turn: bool = False, pair_poly: int = 0, dim: int = 128,
                    mask_name: str | None = None) -> dict:
    """The kernel's launch record and PTX.  ``trace`` adds a ``__trace`` buffer parameter of
    grid x 66 x 24 u64 clock64 stamps (a pipeline timeline probe, see :func:`trace_events`).
    ``pingpong`` makes the two tiles' softmax warpgroups take turns on the MUFU exps.
    ``bh_range`` = (first, count) restricts the launch to those flattened (batch, head) pairs.
    ``prefetch_next`` = n > 0 makes the producer prefetch into L2, after its last load, the Q tiles and
    first K / V block of CTA index + n (the one likely to start when this one ends).  ``pack_in_turn``
    keeps all of a block's f16 packing inside its MUFU turn.  ``pair_poly`` = n (0-4) takes n of every
    4 score pairs of the f16 path off the MUFU: a cubic exp2 on the FMA pipe, two scores per f32x2
    instruction (the MUFU ``ex2`` and the f16 ``cvt`` packing share the XU pipe, which bounds the exp
    phase).  ``mask_name`` adds an explicit boolean mask M [S, S] (u8, nonzero = the key takes part, as
    torch's ``attn_mask``): each softmax thread reads its row's 64 bytes per key block and sets the
    masked scores to -inf; a row whose keys so far are all masked keeps a running max of -inf and
    exponentiates against 0, and a row with every key masked ends as 0 / 0 = NaN, as in torch."""
    if dim not in (32, 64, 128):
        raise ValueError("tcgen05 attention takes head dim 32, 64 or 128")
    # the head dim sets the tile sizes: a Q tile or K/V block is dim / BOXC TMA boxes of BOXC columns,
    # 64 columns (128-byte rows, SWIZZLE_128B) or, at head dim 32, 32 columns (64-byte rows, SWIZZLE_64B)
    D = dim
    BOXC = min(D, 64)
    SW = 2 * BOXC                 # row bytes of a box = the swizzle span
    KPB = BOXC // 16              # K=16 MMA steps per box
    Q_BYTES = BQ * D * 2
    Q_HALF = BQ * BOXC * 2        # one TMA box of a Q tile
    KV_BYTES = BKV * D * 2
    KV_HALF = BKV * BOXC * 2      # one TMA box of a K/V block
    S_COL0 = TILES * D
    if not 0 <= pair_poly <= 4:
        raise ValueError("pair_poly takes 0-4 of every 4 score pairs")
    if pair_poly and poly_every:
        raise ValueError("pair_poly and poly_every are alternatives")
    if seq < 1:
        raise ValueError("tcgen05 attention needs S >= 1")
    # a sequence that is no multiple of the CTA's 256 query rows: the last CTA's rows past S (and the
    # key rows past S of its blocks) are zero-filled by TMA, also when a whole box reaches past the
    # tensor (S < 128 or 64); their results are not stored, and a full (non-causal) launch masks the keys
    # past S in the last block
    nt = -(-seq // (BQ * TILES))
    spad = nt * BQ * TILES
    nblk = -(-seq // BKV)                        # key/value blocks holding data (value flags)
    ragged = seq != spad
    if half and precise and spad // BKV > (BAR_BYTES - VFLAGS) // 4:
        raise ValueError("the f16 path keeps one flag per kv block in shared memory: S <= 4096")
    if trace and spad // BKV + 1 >= TRACE_SLOTS:
        raise ValueError("trace supports at most 64 key/value blocks")
    half = half and precise
    mask = mask_name is not None
    if mask and seq % 16:
        raise ValueError("the masked attention reads its mask rows in 16-byte pieces: S % 16 == 0")
    if pack_in_turn and (pack_after_turn or not pingpong):
        raise ValueError("pack_in_turn applies to the default split packing with turns")
    if defer_sum and (poly_every or not pack_after_turn):
        raise ValueError("defer_sum goes with the MUFU-only exps packed after the turn")
    threads = THREADS
    bh0, nbh = bh_range if bh_range is not None else (0, batch * heads)
    if not (0 <= bh0 and nbh > 0 and bh0 + nbh <= batch * heads):
        raise ValueError(f"bh_range {bh_range} outside the {batch * heads} (batch, head) pairs")
    grid = nbh * nt
    a = Asm()
    idesc_qk = idesc_f16(BQ, BKV, False, False)
    idesc_pv = idesc_f16(BQ, D, False, True)
    idesc_pv16 = idesc_f16(BQ, D, False, True, half=True)
    kdesc_hi = smem_desc_hi(16, 8 * SW, SW)      # K-major (Q, K): 8-row groups of SW-byte rows
    vdesc_hi = smem_desc_hi(KV_HALF, 8 * SW, SW)  # MN-major (V): BOXC-column atoms KV_HALF apart
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
    trc = None
    if trace:
        trc = a.r("rd")
        a(f"ld.param.u64 {trc}, [p_trace];")
        a(f"cvta.to.global.u64 {trc}, {trc};")
        tcta = a.r("rd")
        a(f"mul.wide.u32 {tcta}, {cta}, {TRACE_SLOTS * TRACE_EVENTS * 8};")
        a(f"add.s64 {trc}, {trc}, {tcta};")          # this CTA's trace rows

    def stamp(event, jreg, guard=None):
        """clock64 into trace[cta][j][event] (j = TRACE_SLOTS-1 for per-CTA facts)."""
        if not trace:
            return
        off, ck, ad = a.r(), a.r("rd"), a.r("rd")
        if isinstance(jreg, int):
            a(f"mov.u32 {off}, {jreg * TRACE_EVENTS};")
        else:
            a(f"mul.lo.u32 {off}, {jreg}, {TRACE_EVENTS};")
        if not isinstance(event, int) or event:
            a(f"add.u32 {off}, {off}, {event};")
        a(f"mul.wide.u32 {ad}, {off}, 8;")
        a(f"add.s64 {ad}, {ad}, {trc};")
        a(f"mov.u64 {ck}, %clock64;")
        a(f"{'@' + guard + ' ' if guard else ''}st.global.u64 [{ad}], {ck};")

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
    if bh0:
        a(f"add.u32 {bh}, {bh}, {bh0};")
    a(f"div.u32 {bb}, {bh}, {heads};")
    a(f"rem.u32 {hh}, {bh}, {heads};")
    nb, row0 = a.r(), a.r()
    if causal:
        a(f"shl.b32 {nb}, {t}, 2;")
        a(f"add.u32 {nb}, {nb}, 4;")                    # tile 1 sees kv blocks 0..4t+3, tile 0 0..4t+1
    else:
        a(f"mov.u32 {nb}, {nblk};")
    a(f"shl.b32 {row0}, {t}, 8;")                        # first query row of this CTA

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
    a(f"mbarrier.init.shared::cta.b64 [{bars}+{QFULL}], 1;")
    for s in range(STAGES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{FULL + 8 * s}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{EMPTY + 8 * s}], {TILES};")
    for i in range(TILES):
        for b_ in range(2):
            a(f"mbarrier.init.shared::cta.b64 [{bars}+{SFULL + 8 * (2 * i + b_)}], 1;")
            a(f"mbarrier.init.shared::cta.b64 [{bars}+{PFULL + 8 * (2 * i + b_)}], 4;")
            a(f"mbarrier.init.shared::cta.b64 [{bars}+{PFREE + 8 * (2 * i + b_)}], 1;")
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
    if trace:
        pt0 = a.r("p")
        a(f"setp.eq.u32 {pt0}, {tid}, 0;")
        stamp(0, TRACE_SLOTS - 1, pt0)
        smid, sm64, sad = a.r(), a.r("rd"), a.r("rd")
        a(f"mov.u32 {smid}, %smid;")
        a(f"cvt.u64.u32 {sm64}, {smid};")
        a(f"add.s64 {sad}, {trc}, {((TRACE_SLOTS - 1) * TRACE_EVENTS + 2) * 8};")
        a(f"@{pt0} st.global.u64 [{sad}], {sm64};")

    l_end = a.L("end")
    l_prod, l_mma, l_mma1, l_soft = a.L("prod"), a.L("mma"), a.L("mma1"), a.L("soft")
    pw0, pw2, pws = a.r("p"), a.r("p"), a.r("p")
    a(f"setp.eq.u32 {pw0}, {warp}, 0;")
    a(f"setp.eq.u32 {pw2}, {warp}, 2;")
    a(f"setp.ge.u32 {pws}, {warp}, 4;")
    a(f"@{pw0} bra {l_prod};")
    a(f"@{pw1} bra {l_mma};")
    a(f"@{pw2} bra {l_mma1};")
    a(f"@{pws} bra {l_soft};")
    a(f"bra {l_end};")                                   # warp 3: no role

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
            if ragged and causal:
                # the causal diagonal's blocks past S hold no data (zero-filled by TMA from the f16
                # copy): flag 0, and no load past this (batch, head)'s flags
                pd = a.r("p")
                a(f"setp.lt.u32 {pd}, {bk}, {nblk};")
                a(f"and.pred {pd}, {pd}, {pk};")
                a(f"mov.u32 {fk}, 0;")
                a(f"@{pd} ld.global.nc.u32 {fk}, [{ga}];")
            else:
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
        for hb in range(D // BOXC):
            d_ = a.r()
            a(f"add.u32 {d_}, {sQ}, {Q_BYTES * i + Q_HALF * hb};")
            tma4(d_, tq, BOXC * hb, r_i, qb)
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
    a(f"shl.b32 {kvrow}, {kvrow}, 6;")
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
    for hb in range(1, D // BOXC):
        dst2 = a.r()
        a(f"add.u32 {dst2}, {dst}, {KV_HALF * hb};")
        tma4(dst2, tsel, BOXC * hb, kvrow, fb)
    pw = a.r("p")
    a(f"add.u32 {stage}, {stage}, 1;")
    a(f"setp.eq.u32 {pw}, {stage}, {STAGES};")
    a(f"@{pw} mov.u32 {stage}, 0;")
    a(f"@{pw} xor.b32 {phase}, {phase}, 1;")
    a(f"add.u32 {n_}, {n_}, 1;")
    a(f"bra {l_pl};")
    a.label(l_pdone)
    if prefetch_next:
        # the CTA that starts about when this one ends (index + prefetch_next, the SMs' worth of
        # CTAs ahead in launch order) will first read its two Q tiles and K_0 / V_0: ask L2 for them
        # now, while this CTA's last blocks run (a prefetch has no completion to wait for)
        l_nopf = a.L("nopf")
        cn, pnx = a.r(), a.r("p")
        a(f"add.u32 {cn}, {cta}, {prefetch_next};")
        a(f"setp.ge.u32 {pnx}, {cn}, {grid};")
        a(f"@{pnx} bra {l_nopf};")
        tn, bhn, bbn, hhn, rown = a.r(), a.r(), a.r(), a.r(), a.r()
        a(f"div.u32 {tn}, {cn}, {nbh};")
        a(f"sub.u32 {tn}, {nt - 1}, {tn};")
        a(f"rem.u32 {bhn}, {cn}, {nbh};")
        if bh0:
            a(f"add.u32 {bhn}, {bhn}, {bh0};")
        a(f"div.u32 {bbn}, {bhn}, {heads};")
        a(f"rem.u32 {hhn}, {bhn}, {heads};")
        a(f"shl.b32 {rown}, {tn}, 8;")
        for i in range(TILES):
            r_i = a.r()
            a(f"add.u32 {r_i}, {rown}, {BQ * i};")
            for hb in range(D // BOXC):
                a(f"cp.async.bulk.prefetch.tensor.4d.L2.global.tile [{tq}, {{{BOXC * hb}, {r_i}, {hhn}, {bbn}}}];")
        for tmn in (tk, tv16 if half else tv):
            for hb in range(D // BOXC):
                a(f"cp.async.bulk.prefetch.tensor.4d.L2.global.tile [{tmn}, {{{BOXC * hb}, 0, {hhn}, {bbn}}}];")
        a.label(l_nopf)
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
    # one issuing thread per query tile (warp 1: tile 0, warp 2: tile 1).  The tensor core's
    # instruction queue is shallow, so while one issuer waits for its P or does its bookkeeping the
    # other's MMAs keep the tensor core busy; each ring stage is released when both issuers' MMAs
    # that read it have completed (empty barriers count two arrivals).
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
        a(f"sub.u32 {lasti}, {nb}, {(3 if causal else 1) if i == 0 else 1};")

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

        # the Q operand never changes: its 8 descriptors once; every ring stage's descriptors, the
        # S/O TMEM columns and the barrier offsets are fixed, and the issue loop is unrolled over the
        # 8 ring stages (4 kv blocks), so each MMA costs at most one add
        qb_i = a.r()
        a(f"add.u32 {qb_i}, {sQ}, {Q_BYTES * i};")
        q0 = base_desc(qb_i, khi)
        qdesc = [plus(q0, (k // KPB) * Q_HALF + (k % KPB) * 32) for k in range(D // 16)]
        kd, vd = [], []
        for st_ in range(STAGES):
            sb = a.r()
            a(f"add.u32 {sb}, {sKV}, {st_ * KV_BYTES};")
            kd.append(base_desc(sb, khi))
            vd.append(base_desc(sb, vhi))
        scol_c = [a.r() for _ in range(2)]
        ocol_c = a.r()
        a(f"add.u32 {ocol_c}, {taddr}, {D * i};")
        for b_ in range(2):
            a(f"add.u32 {scol_c[b_]}, {taddr}, {S_COL0 + 2 * BKV * i + BKV * b_};")

        def ring_wait(stage_c, par):
            wait_bar(a, f"{bars}+{FULL + 8 * stage_c}", par, err, ERR_MMA, l_mdone)
            a("tcgen05.fence::after_thread_sync;")

        def qk(stage_c, buf_c):
            """S_i(j) = Q_i K_j^T into S_i[j & 1] (K_j in ring stage ``stage_c``); the buffer's previous
            P (block j-2) was read by a PV issued earlier from this thread, and the tensor core runs
            one thread's MMAs in order."""
            for k in range(D // 16):
                db = plus(kd[stage_c], (k // KPB) * KV_HALF + (k % KPB) * 32)
                a(f"tcgen05.mma.cta_group::1.kind::f16 [{scol_c[buf_c]}], {qdesc[k]}, {db}, {iqk}, "
                  f"{ptrue if k else pfalse};")
            a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bars}+{SFULL + 16 * i + 8 * buf_c}];")

        def pv(stage_c, buf_c, u, jreg, gpreg):
            """O_i += P_i(j) V_j (V_j in ring stage ``stage_c``) once the softmax has written P_i(j)
            over S_i[j & 1].  The P-full barrier of a buffer completes once per use, so block
            j = 4g + u waits for phase j >> 1, whose parity is (u >> 1) & 1.

            With the f16 path the block's flag (from the value pre-pass) picks the MMAs: f16 P (columns
            0-31, two f16 per column) times the f16 copy of V in one pass, or, when V_j did not fit
            f16, bf16 P_hi (columns 0-31) and P_lo (32-63) times V itself."""
            vds = [plus(vd[stage_c], 16 * SW * k) for k in range(BKV // 16)]      # 16 rows of SW bytes
            pacc = a.r("p")
            a(f"setp.ne.u32 {pacc}, {jreg}, 0;")
            p16 = None
            if half:
                fa_, fmt = a.r(), a.r()
                p16 = a.r("p")
                a(f"mad.lo.u32 {fa_}, {jreg}, 4, {bars};")
                a(f"ld.shared.u32 {fmt}, [{fa_}+{VFLAGS}];")
                a(f"setp.eq.u32 {p16}, {fmt}, 0;")
            wait_bar(a, f"{bars}+{PFULL + 16 * i + 8 * buf_c}", str((u >> 1) & 1), err, ERR_MMA, l_mdone)
            stamp(4 + 2 * i, jreg)
            a("tcgen05.fence::after_thread_sync;")
            l_bf, l_done = a.L("pvbf"), a.L("pvdone")
            if half:
                a(f"@!{p16} bra {l_bf};")
                for k in range(BKV // 16):
                    acc = pacc if k == 0 else ptrue
                    a(f"tcgen05.mma.cta_group::1.kind::f16 [{ocol_c}], [{scol_c[buf_c]}+{8 * k}], "
                      f"{vds[k]}, {ipv16}, {acc};")
                a(f"bra {l_done};")
            a.label(l_bf)
            for part in range(2 if precise else 1):
                for k in range(BKV // 16):
                    acc = pacc if (k == 0 and part == 0) else ptrue
                    a(f"tcgen05.mma.cta_group::1.kind::f16 [{ocol_c}], [{scol_c[buf_c]}+{(BKV // 2) * part + 8 * k}], "
                      f"{vds[k]}, {ipv}, {acc};")
            a.label(l_done)
            a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bars}+{PFREE + 16 * i + 8 * buf_c}];")
            stamp(5 + 2 * i, jreg)

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
        qk(0, 0)
        release(0, True)
        l_mg = a.L(f"mg{i}")
        a.label(l_mg)
        a(f"xor.b32 {gpn}, {gp}, 1;")
        for u in range(4):                                 # block j = 4g + u
            if i == 0:
                stamp(0, j)
            # scores of the next block first (K_{j+1} = item 2j+2, stage 2u+2 mod 8), so the softmax
            # of block j+1 can start as soon as block j's ends
            have_next = a.r("p")
            jn = a.r()
            a(f"add.u32 {jn}, {j}, 1;")
            a(f"setp.lt.u32 {have_next}, {jn}, {nb};")
            l_nok = a.L("nok")
            a(f"@!{have_next} bra {l_nok};")
            ks = (2 * u + 2) % STAGES
            ring_wait(ks, gpn if u == 3 else gp)
            if i == 0:
                stamp(1, j)
            l_qk, l_qkd = a.L("noqk"), a.L("qkd")
            pn_ = a.r("p")
            a(f"setp.gt.u32 {pn_}, {jn}, {lasti};")
            a(f"@{pn_} bra {l_qk};")
            qk(ks, (u + 1) & 1)
            release(ks, True)
            a(f"bra {l_qkd};")
            a.label(l_qk)
            release(ks, False)
            a.label(l_qkd)
            if i == 0:
                stamp(2, j)
            a.label(l_nok)
            vs = 2 * u + 1                                 # V_j = item 2j+1
            ring_wait(vs, gp)
            if i == 0:
                stamp(3, j)
            l_pv, l_pvd = a.L("nopv"), a.L("pvd")
            pj_ = a.r("p")
            a(f"setp.gt.u32 {pj_}, {j}, {lasti};")
            a(f"@{pj_} bra {l_pv};")
            pv(vs, u & 1, u, j, gp)
            release(vs, True)
            a(f"bra {l_pvd};")
            a.label(l_pv)
            release(vs, False)
            a.label(l_pvd)
            a(f"@!{have_next} bra {l_mdone};")
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
    scol0, ocol = a.r(), a.r()
    a(f"mad.lo.u32 {scol0}, {ti}, {2 * BKV}, {lanebase};")
    a(f"add.u32 {scol0}, {scol0}, {S_COL0};")              # S_ti[0]; S_ti[1] is BKV columns on
    a(f"mad.lo.u32 {ocol}, {ti}, {D}, {lanebase};")
    last, grow0 = a.r(), a.r()
    if causal:
        a(f"shl.b32 {last}, {t}, 2;")
        a(f"mad.lo.u32 {last}, {ti}, 2, {last};")
        a(f"add.u32 {last}, {last}, 1;")                   # tile i's last kv block: 4t + 2i + 1
    else:
        a(f"sub.u32 {last}, {nb}, 1;")
    a(f"mad.lo.u32 {grow0}, {ti}, {BQ}, {row0};")
    mrow = prow_m = None
    if mask:
        # M + q * S for this thread's query row q (its 64 bytes of block jj start 64 * jj further on)
        mrow, mq = a.r("rd"), a.r("rd")
        a(f"ld.param.u64 {mrow}, [p_M];")
        a(f"cvta.to.global.u64 {mrow}, {mrow};")
        growm = a.r()
        a(f"mad.lo.u32 {growm}, {ti}, {BQ}, {row0};")
        a(f"add.u32 {growm}, {growm}, {rowl};")
        a(f"mul.wide.u32 {mq}, {growm}, {seq};")
        a(f"add.s64 {mrow}, {mrow}, {mq};")
        if ragged:
            prow_m = a.r("p")
            a(f"setp.lt.u32 {prow_m}, {growm}, {seq};")   # rows past S have no mask row
    a(f"add.u32 {grow0}, {grow0}, {rowl};")                # this thread's query row
    sfb0, pfb0, pfr0 = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {sfb0}, {ti}, 16, {bars};")
    a(f"add.u32 {pfb0}, {sfb0}, {PFULL};")
    a(f"add.u32 {pfr0}, {sfb0}, {PFREE};")
    a(f"add.u32 {sfb0}, {sfb0}, {SFULL};")

    def pv_done(blk, bail, code):
        """Wait until PV_ti(blk) has completed (its buffer's PV-done barrier, phase blk >> 1)."""
        bb_, br_, pr_ = a.r(), a.r(), a.r()
        a(f"and.b32 {bb_}, {blk}, 1;")
        a(f"mad.lo.u32 {br_}, {bb_}, 8, {pfr0};")
        a(f"shr.u32 {pr_}, {blk}, 1;")
        a(f"and.b32 {pr_}, {pr_}, 1;")
        wait_bar_warp(a, br_, pr_, err, code, bail)
    ple = a.r("p")
    a(f"setp.eq.u32 {ple}, {lane}, 0;")
    ev_s, ptw = None, None
    if trace:
        ev_s = a.r()
        a(f"mad.lo.u32 {ev_s}, {ti}, 8, 8;")
        ptw = a.r("p")
        a(f"setp.eq.u32 {ptw}, {rowl}, 0;")
    jj, failed = a.r(), a.r()
    a(f"mov.u32 {jj}, 0;")
    a(f"mov.u32 {failed}, 0;")
    l_sdone = a.L("sdone")
    l_drain, l_drain_post = (a.L("drain"), a.L("drainpost")) if pingpong else (l_sdone, l_sdone)
    if pingpong:
        # The two tiles' softmax warpgroups take turns on the MUFU: tile 0's exps of block j, then
        # tile 1's, then tile 0's of block j+1, ...  Each hands the turn over with a named barrier
        # (tile 0 waits on barrier 1 and passes on barrier 2, tile 1 the reverse; 256 threads: one
        # warpgroup syncs, the other arrives), so while one tile's exps run the other loads its
        # scores, takes the row max and writes P.  Tile 1 has two blocks more than tile 0 on the
        # causal diagonal and runs those alone.  Every softmax thread executes the same sequence of
        # barrier operations whatever happens: a time-out leaves the work but not the hand-overs
        # (the drain below), so neither warpgroup can be left waiting on the other.
        last0, arr_lim = a.r(), a.r()
        tile0 = a.r("p")
        if causal:
            a(f"shl.b32 {last0}, {t}, 2;")
            a(f"add.u32 {last0}, {last0}, 1;")             # tile 0's last kv block
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

    def sstamp(k):
        """Softmax timeline stamp ``k`` (0 S ready, 1 S loaded, 2 row max, 3 format known, 7 MUFU turn
        taken, 4 exps done, 5 P stores issued, 6 P written) for this tile, from the tile's first
        thread."""
        if not trace:
            return
        ev = a.r()
        a(f"add.u32 {ev}, {ev_s}, {k};")
        stamp(ev, jj, ptw)

    l_sj = a.L("sj")
    a.label(l_sj)
    pj = a.r("p")
    a(f"setp.gt.u32 {pj}, {jj}, {last};")
    a(f"@{pj} bra {l_sdone};")
    bsel, sfb, pfb, par_s, scol = a.r(), a.r(), a.r(), a.r(), a.r()
    a(f"and.b32 {bsel}, {jj}, 1;")
    a(f"mad.lo.u32 {sfb}, {bsel}, 8, {sfb0};")
    a(f"mad.lo.u32 {pfb}, {bsel}, 8, {pfb0};")
    a(f"shr.u32 {par_s}, {jj}, 1;")
    a(f"and.b32 {par_s}, {par_s}, 1;")
    a(f"mad.lo.u32 {scol}, {bsel}, {BKV}, {scol0};")
    mw = None
    if mask:
        # this row's mask bytes for block jj, loaded before the wait for the scores so the load's
        # latency overlaps it (rows past S: every key kept)
        mw = [a.r() for _ in range(BKV // 4)]
        ma, mo = a.r("rd"), a.r("rd")
        a(f"mul.wide.u32 {mo}, {jj}, {BKV};")
        a(f"add.s64 {ma}, {mrow}, {mo};")
        partial = seq % BKV != 0            # the last block's 16-byte pieces past S are not read
        if prow_m is not None or partial:
            for w_ in mw:
                a(f"mov.u32 {w_}, 0x01010101;")   # kept; keys past S are masked by the key limit
        kv0m = None
        if partial:
            kv0m = a.r()
            a(f"shl.b32 {kv0m}, {jj}, 6;")
        for i_ in range(BKV // 16):
            g_ = ""
            if partial and seq - 16 * i_ <= 0:
                continue                        # a piece past S in every block (S < 64)
            if partial:
                pp_ = a.r("p")
                a(f"setp.lt.u32 {pp_}, {kv0m}, {seq - 16 * i_};")   # 64*jj + 16*i < S
                if prow_m is not None:
                    a(f"and.pred {pp_}, {pp_}, {prow_m};")
                g_ = f"@{pp_} "
            elif prow_m is not None:
                g_ = f"@{prow_m} "
            a(f"{g_}ld.global.nc.v4.u32 {{{', '.join(mw[4 * i_:4 * i_ + 4])}}}, [{ma}+{16 * i_}];")
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
    sstamp(0)
    a("tcgen05.fence::after_thread_sync;")
    for c in range(BKV // 32):
        src = a.r()
        a(f"add.u32 {src}, {scol}, {32 * c};")
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(s_[32 * c:32 * c + 32])}}}, [{src}];")
    a("tcgen05.wait::ld.sync.aligned;")
    sstamp(1)
    if causal:
        # kv = 64*jj + c is masked when kv > query row, i.e. c > grow0 - 64*jj; only the blocks that
        # reach the diagonal (the tile's last two) have masked columns
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
    elif seq % BKV:
        # kv = 64*jj + c past the sequence is masked: c > S - 1 - 64*jj, in the last block only
        l_nokey = a.L("nokey")
        klim, kv0k = a.r(), a.r()
        a(f"shl.b32 {kv0k}, {jj}, 6;")
        a(f"sub.s32 {klim}, {seq - 1}, {kv0k};")
        pkm = a.r("p")
        a(f"setp.ge.s32 {pkm}, {klim}, {BKV - 1};")
        a(f"@{pkm} bra {l_nokey};")                        # the same for every thread of the CTA
        for c in range(seq % BKV, BKV):
            a(f"mov.b32 {s_[c]}, 0fFF800000;")
        a.label(l_nokey)
    if mask:
        # the explicit mask: a zero byte removes its key
        for c in range(BKV):
            t_, pz = a.r(), a.r("p")
            a(f"and.b32 {t_}, {mw[c // 4]}, {0xFF << (8 * (c % 4))};")
            a(f"setp.eq.u32 {pz}, {t_}, 0;")
            a(f"@{pz} mov.b32 {s_[c]}, 0fFF800000;")
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
    sstamp(2)
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
    if mask:
        # a row whose keys are all masked so far (max still -inf) while another row of the warp
        # rescales: nothing to rescale (its O and sum are 0), and -inf - -inf must not make a NaN
        pm_inf = a.r("p")
        a(f"setp.eq.f32 {pm_inf}, {mnew}, 0fFF800000;")
        a(f"@{pm_inf} mov.b32 {alpha}, 0f3F800000;")
    a(f"mov.b32 {mref}, {mnew};")
    a(f"mul.f32 {lsum}, {lsum}, {alpha};")
    a.label(l_norescale)
    a(f"bra {l_after};")
    a.label(l_first)
    a(f"mov.b32 {mref}, {mnew};")
    a(f"setp.ne.u32 {anyneed}, {lane}, {lane};")
    a.label(l_after)
    # p = 2^(s*c - m), row sum, and P back over S's TMEM columns as bf16 pairs (hi, then lo)
    negm = a.r("f")
    a(f"neg.f32 {negm}, {mref};")
    if mask:
        # every key so far masked: the running max is -inf; exponentiate against 0 (p = 0) instead
        pninf = a.r("p")
        a(f"setp.eq.f32 {pninf}, {mref}, 0fFF800000;")
        a(f"@{pninf} mov.b32 {negm}, 0f00000000;")
    parts = [a.r("f") for _ in range(4)]
    for pp in parts:
        a(f"mov.b32 {pp}, 0f00000000;")
    def row_sum(cols):
        """parts += the row's p values over ``cols`` (pairs, on the FMA pipe)."""
        acc = [a.r("rd"), a.r("rd")]
        a(f"mov.b64 {acc[0]}, {{{parts[0]}, {parts[1]}}};")
        a(f"mov.b64 {acc[1]}, {{{parts[2]}, {parts[3]}}};")
        for k, idx in enumerate(list(cols)[::2]):
            ep = a.r("rd")
            a(f"mov.b64 {ep}, {{{s_[idx]}, {s_[idx + 1]}}};")
            a(f"add.rn.f32x2 {acc[k & 1]}, {acc[k & 1]}, {ep};")
        a(f"mov.b64 {{{parts[0]}, {parts[1]}}}, {acc[0]};")
        a(f"mov.b64 {{{parts[2]}, {parts[3]}}}, {acc[1]};")

    pconst = {}

    def pair_const(name, bits32):
        """A 64-bit register holding the f32 constant ``bits32`` in both halves (made once)."""
        if name not in pconst:
            r = a.r("rd")
            a(f"mov.b64 {r}, 0x{bits32:08X}{bits32:08X};")
            pconst[name] = r
        return pconst[name]

    def poly_pair(xp, x0, x1):
        """(x0, x1) = 2^x for the pair in ``xp`` on the FMA and integer pipes, two lanes per f32x2
        instruction: clamp at -120, split x = n + f with f in [-1/2, 1/2] by adding and taking away
        1.5 * 2^23, 2^f by the cubic ``EXP2_C`` (7.8e-5 relative, below the f16 rounding of P) in
        Horner form, then n added to the exponent field."""
        magic = pair_const("magic", 0x4B400000)
        cs = [pair_const(f"c{i}", int(EXP2_C[i][2:], 16)) for i in range(4)]
        a(f"max.f32 {x0}, {x0}, 0fC2F00000;")
        a(f"max.f32 {x1}, {x1}, 0fC2F00000;")
        tp, jp, fp, rp = a.r("rd"), a.r("rd"), a.r("rd"), a.r("rd")
        a(f"mov.b64 {xp}, {{{x0}, {x1}}};")
        a(f"add.rn.f32x2 {tp}, {xp}, {magic};")
        a(f"sub.rn.f32x2 {jp}, {tp}, {magic};")
        a(f"sub.rn.f32x2 {fp}, {xp}, {jp};")
        a(f"fma.rn.f32x2 {rp}, {fp}, {cs[3]}, {cs[2]};")
        a(f"fma.rn.f32x2 {rp}, {rp}, {fp}, {cs[1]};")
        a(f"fma.rn.f32x2 {rp}, {rp}, {fp}, {cs[0]};")
        t0, t1, r0, r1 = a.r(), a.r(), a.r(), a.r()
        a(f"mov.b64 {{{t0}, {t1}}}, {tp};")
        a(f"mov.b64 {{{r0}, {r1}}}, {rp};")
        a(f"shl.b32 {t0}, {t0}, 23;")
        a(f"shl.b32 {t1}, {t1}, 23;")
        a(f"add.s32 {r0}, {r0}, {t0};")
        a(f"add.s32 {r1}, {r1}, {t1};")
        a(f"mov.b32 {x0}, {r0};")
        a(f"mov.b32 {x1}, {r1};")

    def exp_block(poly_every, cols=range(BKV), sums=True, pairs_poly=0):
        """p = 2^(s*c - m) for the row's BKV scores, summed into ``parts``.  With ``poly_every`` = n,
        every n-th value is taken on the FMA pipe instead of the MUFU (the softmax's bottleneck):
        x is clamped at -120, split as n + f with f in [-1/2, 1/2] by the 1.5*2^23 rounding trick,
        2^f comes from a cubic (``EXP2_C``), and n is added to the exponent field.  Only the f16 path
        uses it: there P rounds 2^-120 to zero, as the MUFU's 2^-inf is zero."""
        cols = list(cols)
        if not poly_every:
            # two scores per instruction on the FMA pipe (f32x2 fma and add); the MUFU takes one each
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
                if (idx // 2) % 4 < pairs_poly:
                    poly_pair(xp, x0, x1)           # pairs_poly of every 4 pairs off the MUFU
                else:
                    a(f"ex2.approx.ftz.f32 {x0}, {x0};")
                    a(f"ex2.approx.ftz.f32 {x1}, {x1};")
                if sums:
                    ep = a.r("rd")
                    a(f"mov.b64 {ep}, {{{x0}, {x1}}};")
                    a(f"add.rn.f32x2 {acc[k & 1]}, {acc[k & 1]}, {ep};")
            a(f"mov.b64 {{{parts[0]}, {parts[1]}}}, {acc[0]};")
            a(f"mov.b64 {{{parts[2]}, {parts[3]}}}, {acc[1]};")
            return
        t_, j_, f_, r_, ti_, ri_ = (a.r("f"), a.r("f"), a.r("f"), a.r("f"), a.r(), a.r())
        for idx in cols:
            x = s_[idx]
            a(f"fma.rn.f32 {x}, {x}, {cscale}, {negm};")
            if poly_every and idx % poly_every == poly_every - 1:
                a(f"max.f32 {x}, {x}, 0fC2F00000;")
                a(f"add.f32 {t_}, {x}, 0f4B400000;")
                a(f"sub.f32 {j_}, {t_}, 0f4B400000;")
                a(f"sub.f32 {f_}, {x}, {j_};")
                a(f"fma.rn.f32 {r_}, {f_}, {EXP2_C[3]}, {EXP2_C[2]};")
                a(f"fma.rn.f32 {r_}, {r_}, {f_}, {EXP2_C[1]};")
                a(f"fma.rn.f32 {r_}, {r_}, {f_}, {EXP2_C[0]};")
                a(f"mov.b32 {ti_}, {t_};")
                a(f"shl.b32 {ti_}, {ti_}, 23;")
                a(f"mov.b32 {ri_}, {r_};")
                a(f"add.s32 {ri_}, {ri_}, {ti_};")
                a(f"mov.b32 {x}, {ri_};")
            else:
                a(f"ex2.approx.ftz.f32 {x}, {x};")
            a(f"add.f32 {parts[idx & 3]}, {parts[idx & 3]}, {x};")

    c112 = None

    def f16_pack_int(w, x0, x1):
        """w = the f16 pair (x1, x0) for 0 <= x <= 1, on the FMA and integer pipes instead of the
        conversion unit: x * 2^-112 (subnormals kept) has the f16 exponent bias, so its bits >> 13 are
        the f16 bits, normal and subnormal alike; adding 2^12 first rounds to nearest (ties away
        from zero), and a carry out of the mantissa moves into the exponent as it should."""
        nonlocal c112
        if c112 is None:
            c112 = a.r("rd")
            a(f"mov.b64 {c112}, 0x0780000007800000;")     # {2^-112, 2^-112}
        yp, y0, y1 = a.r("rd"), a.r(), a.r()
        a(f"mov.b64 {yp}, {{{x0}, {x1}}};")
        a(f"mul.rn.f32x2 {yp}, {yp}, {c112};")
        a(f"mov.b64 {{{y0}, {y1}}}, {yp};")
        a(f"add.u32 {y0}, {y0}, 4096;")
        a(f"add.u32 {y1}, {y1}, 4096;")
        a(f"shr.u32 {y0}, {y0}, 13;")
        a(f"shl.b32 {y1}, {y1}, 3;")
        a(f"lop3.b32 {w}, {y1}, {y0}, -65536, 0xEC;")     # (y1 & 0xFFFF0000) | y0

    l_pdone = a.L("pdone")
    if half:
        # the format the value pre-pass chose for this block (read once S was ready)
        sstamp(3)
    turn_wait()
    sstamp(7)
    if half:
        l_pbf = a.L("pbf")
        a(f"@!{p16} bra {l_pbf};")
        half_n = BKV // 2

        def pack_store(pairs, col):
            hw = []
            for k in pairs:
                w = a.r()
                if f16_int and k % f16_int == f16_int - 1:
                    f16_pack_int(w, s_[2 * k], s_[2 * k + 1])
                else:
                    a(f"cvt.rn.f16x2.f32 {w}, {s_[2 * k + 1]}, {s_[2 * k]};")
                hw.append(w)
            dsth = a.r()
            a(f"add.u32 {dsth}, {scol}, {col};")
            a(f"tcgen05.st.sync.aligned.32x32b.x{len(hw)}.b32 [{dsth}], {{{', '.join(hw)}}};")
        if pack_after_turn:
            # only the exps hold the MUFU turn; the f16 packing and the TMEM store of P overlap the
            # other tile's exps
            exp_block(poly_every, sums=not defer_sum, pairs_poly=pair_poly)
            sstamp(4)
            turn_pass()
            if defer_sum:
                row_sum(range(BKV))
            pack_store(range(BKV // 2), 0)
        else:
            for h in range(2):
                # each half of the row is packed and stored as soon as its exps are done; with
                # pack_in_turn the second half's packing stays inside the MUFU turn too, so no f16
                # conversion of this tile runs during the other tile's exps
                exp_block(poly_every, range(half_n * h, half_n * (h + 1)), pairs_poly=pair_poly)
                if h == 1:
                    sstamp(4)
                    if not pack_in_turn:
                        turn_pass()
                pack_store(range(half_n * h // 2, half_n * (h + 1) // 2), half_n * h // 2)
            if pack_in_turn:
                turn_pass()
        sstamp(5)
        a(f"bra {l_pdone};")
        a.label(l_pbf)
    exp_block(0)
    turn_pass()
    hi_w, lo_w = [], []
    for k in range(BKV // 2):
        i0, i1 = 2 * k, 2 * k + 1
        w = a.r()
        if precise:
            # hi = the top 16 bits of p (prmt packs two top halves into one word); lo = the top
            # 16 bits of the exact remainder p - hi
            h0, h1, wl = a.r("f"), a.r("f"), a.r()
            a(f"prmt.b32 {w}, {s_[i0]}, {s_[i1]}, 0x7632;")
            a(f"and.b32 {h0}, {s_[i0]}, -65536;")
            a(f"and.b32 {h1}, {s_[i1]}, -65536;")
            a(f"sub.f32 {h0}, {s_[i0]}, {h0};")
            a(f"sub.f32 {h1}, {s_[i1]}, {h1};")
            a(f"prmt.b32 {wl}, {h0}, {h1}, 0x7632;")
            lo_w.append(wl)
        else:
            a(f"cvt.rn.bf16x2.f32 {w}, {s_[i1]}, {s_[i0]};")
        hi_w.append(w)
    a(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{scol}], {{{', '.join(hi_w)}}};")
    if precise:
        dst2 = a.r()
        a(f"add.u32 {dst2}, {scol}, {BKV // 2};")
        a(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{dst2}], {{{', '.join(lo_w)}}};")
    sstamp(5)
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
    sstamp(6)
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
    sto = ""
    if ragged:
        prow = a.r("p")
        a(f"setp.lt.u32 {prow}, {grow0}, {seq};")         # rows past S are not stored
        sto = f"@{prow} "
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
        a(f"{sto}st.global.v8.b32 [{oaddr}+{64 * c}], {{{', '.join(words[:8])}}};")
        a(f"{sto}st.global.v8.b32 [{oaddr}+{64 * c + 32}], {{{', '.join(words[8:])}}};")
    a.label(l_noepi)

    # ---------------- teardown ---------------------------------------------------------------
    a.label(l_end)
    a("barrier.sync 0;")
    a("bar.warp.sync -1;")
    if trace:
        pt1 = a.r("p")
        a(f"setp.eq.u32 {pt1}, {tid}, 0;")
        stamp(1, TRACE_SLOTS - 1, pt1)
    l_nodealloc = a.L("nodealloc")
    a(f"@!{pw1} bra {l_nodealloc};")
    a("tcgen05.fence::after_thread_sync;")
    a(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {taddr}, {TMEM_COLS};")
    a.label(l_nodealloc)

    dyn = TILES * Q_BYTES + STAGES * KV_BYTES + BAR_BYTES + 1024
    params = ["\t.param .u64 p_Q,", "\t.param .u64 p_K,", "\t.param .u64 p_V,", "\t.param .u64 p_O,"]
    if mask:
        params.append("\t.param .u64 p_M,")
    if half:
        params += ["\t.param .u64 p_V16,", "\t.param .u64 p_vflag,"]
    params += ["\t.param .align 64 .b8 p_tmQ[128],", "\t.param .align 64 .b8 p_tmK[128],",
               "\t.param .align 64 .b8 p_tmV[128],"]
    if half:
        params.append("\t.param .align 64 .b8 p_tmV16[128],")
    params.append("\t.param .u64 p_err" + ("," if trace else ""))
    if trace:
        params.append("\t.param .u64 p_trace")
    entry = [f".visible .entry {name}("] + params + [")", f".reqntid {threads}, 1, 1",
                                                       f".maxnreg {65536 // threads // 8 * 8}", "{"]
    entry += a.decls() + a.lines + ["\tret;", "}"]
    qn, kn, vn, on = names
    dims = [D, seq, heads, batch]
    strides = [D * 2, seq * D * 2, heads * seq * D * 2]
    tmaps = [{"name": "tmQ", "tensor": qn, "dtype": "bf16", "dims": dims, "strides": strides,
              "box": [BOXC, BQ, 1, 1], "swizzle": f"{SW}B"}]
    tmaps += [{"name": f"tm{x}", "tensor": nm, "dtype": "bf16", "dims": dims, "strides": strides,
               "box": [BOXC, BKV, 1, 1], "swizzle": f"{SW}B"} for x, nm in (("K", kn), ("V", vn))]
    uparams = [qn, kn, vn, on] + ([mask_name] if mask else [])
    if half:
        v16n, vfn = scratch_names or (f"{prefix}{name}__v16", f"{prefix}{name}__vflag")
        uparams += [v16n, vfn]
        tmaps.append({"name": "tmV16", "tensor": v16n, "dtype": "f16", "dims": dims, "strides": strides,
                      "box": [BOXC, BKV, 1, 1], "swizzle": f"{SW}B"})
    extra = [{"name": "__err", "kind": "errword"}]
    if trace:
        extra.append({"name": "__trace", "kind": "buffer"})
    return {
        "name": name, "kind": "tcgen05_attention", "params": uparams,
        "raw_entry": entry, "raw_decls": [f".extern .shared .align 1024 .b8 {smem_sym}[];"],
        "grid": [grid, 1, 1], "block": [threads, 1, 1], "dyn_smem": dyn,
        "align": {qn: 16, kn: 16, vn: 16, on: 32, **({mask_name: 16} if mask else {}),
                  **({uparams[-2]: 16, uparams[-1]: 4} if half else {})},
        "zero_outputs": [], "tmaps": tmaps,
        "extra": extra,
    }


def trace_events(buf, grid: int):
    """Split a ``trace`` buffer (u64 [grid, 66, 24]) into per-CTA timelines.  For kv block j, events
    0-7 are tile 0's issuer's iteration start, K_(j+1) arrived, S(j+1) issued and V_j arrived,
    then P_0(j) ready, PV_0 issued, P_1(j) ready and PV_1 issued (each tile's issuer); 8-15 (tile 0)
    and 16-23 (tile 1) are the softmax's S(j) ready, S loaded, row max, format known, exps done,
    P stores issued, P(j) written and (last) MUFU turn taken.  Row 65 holds CTA start, end and the
    SM id."""
    import numpy as np
    return np.asarray(buf, dtype=np.uint64).reshape(grid, TRACE_SLOTS, TRACE_EVENTS)
