"""Batched bf16 GEMM on CTA pairs: ``tcgen05.mma.cta_group::2`` with 256 x 256 output tiles.

The same contraction as :mod:`.tc_gemm` (C[b] = A[b] @ B[b], A [batch, M, K] K-contiguous, B
[batch, K, N] N-contiguous, C f32), launched as clusters of two CTAs on the two SMs of a TPC.  One
MMA instruction of the pair computes a 256 x 256 x 16 product: CTA r of the pair holds rows
128r .. 128r+127 of the A tile and columns 128r .. 128r+127 of the B tile in its own shared memory,
the tensor cores of both SMs read both halves, and each CTA's tensor memory receives its own 128
rows of the 256 x 256 accumulator.  Per SM that is half the shared-memory operand traffic of the
single-CTA kernel's 128 x 256 tile for the same arithmetic (8 KiB instead of 12 KiB per 128 x 256 x
16 of work), which is what bounds that kernel's tensor pipe.

* persistent: cluster p walks tiles ``t = p, p + nclusters, ...`` (n fastest, then m, then batch);
* 192 threads per CTA: warp 0 issues TMA loads (both CTAs, each its own halves), warp 1 allocates
  tensor memory (both CTAs, ``tcgen05.alloc.cta_group::2``) and, in CTA 0 only, issues the MMAs
  from one thread; warps 2-5 of each CTA drain that CTA's 128 accumulator rows;
* a 7-stage ring of 32 KiB stages per CTA (A 128 x 64 K-major, B 64 x 128 MN-major, 128-byte
  swizzle).  Both CTAs' loads of a stage complete the transaction bytes of CTA 0's ``full`` barrier
  (``cp.async.bulk.tensor ... .cta_group::2`` with CTA 0's barrier address); CTA 0's producer
  expects both halves.  The MMA issuer's ``tcgen05.commit.cta_group::2`` arrives on the ``empty``
  barrier of each CTA (one commit per CTA, addressed through ``mapa``), so each producer refills its
  own half;
* two 256-column f32 accumulators (all 512 columns of each SM's tensor memory) so the epilogue of
  one tile overlaps the MMAs of the next: CTA 0's issuer commits ``tmem_full`` to both CTAs, and
  each epilogue warp of either CTA arrives on CTA 0's ``tmem_empty`` (8 arrivals);
* no TMA multicast: every load reads global memory into the issuing CTA's own shared memory;
* every mbarrier wait is bounded (time-out: a code in the error word, the role leaves its loop);
  all threads of both CTAs meet at a cluster barrier before tensor memory is freed, so neither CTA
  exits while its partner may still address its shared memory.

Instruction descriptor: D f32, A/B bf16, A K-major, B MN-major, M=256, N=256.  The shared-memory
descriptors describe one CTA's halves (A: 8-row groups 1024 B apart; B: 64-column atoms 8 KiB
apart, 8-row groups 1024 B apart); the pair reads the same offsets in both CTAs.
"""
from __future__ import annotations

from .ptxasm import Asm, idesc_f16, smem_desc_hi, wait_bar as _wait, wait_bar_warp as _wait_warp

BM, BN, BK = 256, 256, 64          # the pair's output tile and K block
HM, HN = BM // 2, BN // 2          # one CTA's rows of A and columns of B
STAGES = 7                         # 7 x 32 KiB + barriers fill the 227 KiB (measured 2-7 % over 6)
A_STAGE = HM * BK * 2              # 16 KiB
B_STAGE = BK * HN * 2              # 16 KiB
B_BOX = BK * 64 * 2                # one 64-column TMA box of B: 8 KiB
TX_PAIR = 2 * (A_STAGE + B_STAGE)  # bytes CTA 0's full barrier expects per stage (both halves)
THREADS = 192
TMEM_COLS = 512
EPI_ARRIVALS = 8                   # tmem_empty: the 4 epilogue warps of each CTA

ERR_PRODUCER = 61
ERR_MMA_FULL = 62
ERR_MMA_TMEM = 63
ERR_EPILOGUE = 64
ERR_DRAIN = 65

# barrier offsets from the barrier area
FULL = 0
EMPTY = 8 * STAGES
TFULL = 16 * STAGES
TEMPTY = TFULL + 16
SLOT = TEMPTY + 16


def supported(m: int, n: int, k: int) -> bool:
    """The shapes the pair kernel takes: the single-CTA kernel's (N and K multiples of 8, for TMA's
    16-byte rows and whole 32-byte stores of C)."""
    return m >= 1 and n >= 8 and k >= 8 and n % 8 == 0 and k % 8 == 0


def gemm_pair_entry(name: str, batch: int, m: int, n: int, k: int, pairs: int = 74,
                    names=("A", "B", "C"), prefix: str = "", stages: int = STAGES) -> dict:
    """The build record of the CTA-pair GEMM (``pairs`` clusters of two CTAs at most; the runtime
    may launch fewer, the tile loop strides by the launched cluster count).  Shapes that are not
    tile multiples run as edge tiles, as in the single-CTA kernel: TMA zero-fills past the tensor,
    the epilogue stores rows below M and 8-column groups below N."""
    if not supported(m, n, k):
        raise ValueError("tcgen05 GEMM needs N % 8 == 0 and K % 8 == 0")
    if not 2 <= stages <= 7:
        raise ValueError("the pair GEMM's ring holds 2-7 stages of 32 KiB (227 KiB of shared memory)")
    STAGES = stages
    EMPTY = 8 * STAGES
    TFULL = 16 * STAGES
    TEMPTY = TFULL + 16
    SLOT = TEMPTY + 16
    mt, nt, nk = -(-m // BM), -(-n // BN), -(-k // BK)
    edge_m, edge_n = m % BM != 0, n % BN != 0
    tiles = batch * mt * nt
    clusters = max(1, min(tiles, pairs))
    a = Asm()
    idesc = idesc_f16(BM, BN, False, True)
    desc_a_hi = smem_desc_hi(16, 1024)
    desc_b_hi = smem_desc_hi(B_BOX, 1024)

    tid, warp, lane, rank, clu, nclu = a.r(), a.r(), a.r(), a.r(), a.r(), a.r()
    a(f"mov.u32 {tid}, %tid.x;")
    a(f"shr.u32 {warp}, {tid}, 5;")
    a(f"and.b32 {lane}, {tid}, 31;")
    a(f"mov.u32 {rank}, %cluster_ctarank;")
    a(f"mov.u32 {clu}, %clusterid.x;")
    a(f"mov.u32 {nclu}, %nclusterid.x;")
    lead = a.r("p")
    a(f"setp.eq.u32 {lead}, {rank}, 0;")
    c_ptr, err = a.r("rd"), a.r("rd")
    a(f"ld.param.u64 {c_ptr}, [p_C];")
    a(f"cvta.to.global.u64 {c_ptr}, {c_ptr};")
    a(f"ld.param.u64 {err}, [p_err];")
    a(f"cvta.to.global.u64 {err}, {err};")
    tma, tmb = a.r("rd"), a.r("rd")
    a(f"mov.u64 {tma}, p_tmA;")
    a(f"cvta.param.u64 {tma}, {tma};")
    a(f"mov.u64 {tmb}, p_tmB;")
    a(f"cvta.param.u64 {tmb}, {tmb};")

    # shared layout (1024-aligned base, the same offsets in both CTAs): A stages, B stages, barriers
    raw, base = a.r(), a.r()
    smem_sym = f"{prefix}gemm_pair_smem"
    a(f"mov.u32 {raw}, {smem_sym};")
    a(f"add.u32 {base}, {raw}, 1023;")
    a(f"and.b32 {base}, {base}, -1024;")
    sA, sB, bars = a.r(), a.r(), a.r()
    a(f"mov.u32 {sA}, {base};")
    a(f"add.u32 {sB}, {base}, {STAGES * A_STAGE};")
    a(f"add.u32 {bars}, {base}, {STAGES * (A_STAGE + B_STAGE)};")
    # the barrier area of each CTA as a shared::cluster address (targets of the partner's arrivals)
    cbars = [a.r(), a.r()]
    for r_ in range(2):
        a(f"mapa.shared::cluster.u32 {cbars[r_]}, {bars}, {r_};")

    p0 = a.r("p")
    a(f"setp.eq.u32 {p0}, {tid}, 0;")
    l_init = a.L("noinit")
    a(f"@!{p0} bra {l_init};")
    for s in range(STAGES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{FULL + 8 * s}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{EMPTY + 8 * s}], 1;")
    for acc in range(2):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{TFULL + 8 * acc}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{TEMPTY + 8 * acc}], {EPI_ARRIVALS};")
    a("fence.mbarrier_init.release.cluster;")
    a("fence.proxy.async.shared::cta;")
    a.label(l_init)
    pw1 = a.r("p")
    a(f"setp.eq.u32 {pw1}, {warp}, 1;")
    l_noalloc = a.L("noalloc")
    a(f"@!{pw1} bra {l_noalloc};")
    # both CTAs' warp 1: one allocation at the same column in each SM's tensor memory
    a(f"tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [{bars}+{SLOT}], {TMEM_COLS};")
    a("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;")
    a("tcgen05.fence::before_thread_sync;")
    a.label(l_noalloc)
    # both CTAs' barriers are initialised (and the partner's visible) before any cross-CTA arrival
    a("barrier.cluster.arrive.release;")
    a("barrier.cluster.wait.acquire;")
    a("tcgen05.fence::after_thread_sync;")
    taddr = a.r()
    a(f"ld.shared.b32 {taddr}, [{bars}+{SLOT}];")

    l_end = a.L("end")
    l_prod, l_mma, l_epi = a.L("prod"), a.L("mma"), a.L("epi")
    pw0 = a.r("p")
    a(f"setp.eq.u32 {pw0}, {warp}, 0;")
    a(f"@{pw0} bra {l_prod};")
    a(f"@{pw1} bra {l_mma};")
    a(f"bra {l_epi};")

    def tile_coords(t):
        """(b, m0, n0) registers for tile index t (n fastest, then m, then batch)."""
        bb, rr, mm, nn = a.r(), a.r(), a.r(), a.r()
        a(f"div.u32 {bb}, {t}, {mt * nt};")
        a(f"rem.u32 {rr}, {t}, {mt * nt};")
        a(f"div.u32 {mm}, {rr}, {nt};")
        a(f"rem.u32 {nn}, {rr}, {nt};")
        a(f"mul.lo.u32 {mm}, {mm}, {BM};")
        a(f"mul.lo.u32 {nn}, {nn}, {BN};")
        return bb, mm, nn

    # ---------------- producer: warp 0, lane 0 of each CTA ------------------------------------
    # CTA r loads rows 128r.. of the A tile and columns 128r.. of the B tile into its own stage; both
    # CTAs' bytes complete CTA 0's full barrier, which CTA 0's producer arms for the pair's total
    a.label(l_prod)
    pl0 = a.r("p")
    a(f"setp.ne.u32 {pl0}, {lane}, 0;")
    a(f"@{pl0} bra {l_end};")
    stage, phase, t, kb = a.r(), a.r(), a.r(), a.r()
    armed = [a.r() for _ in range(STAGES)]          # phase of each stage's last issued round (2: none)
    for r_ in armed:
        a(f"mov.u32 {r_}, 2;")
    a(f"mov.u32 {stage}, 0;")
    a(f"mov.u32 {phase}, 0;")
    a(f"mov.u32 {t}, {clu};")
    arow, bcol = a.r(), a.r()
    a(f"mul.lo.u32 {arow}, {rank}, {HM};")
    a(f"mul.lo.u32 {bcol}, {rank}, {HN};")
    l_pt, l_pdone = a.L("pt"), a.L("pdone")
    a.label(l_pt)
    pt = a.r("p")
    a(f"setp.ge.u32 {pt}, {t}, {tiles};")
    a(f"@{pt} bra {l_pdone};")
    bb, mm, nn = tile_coords(t)
    a(f"add.u32 {mm}, {mm}, {arow};")
    a(f"add.u32 {nn}, {nn}, {bcol};")
    a(f"mov.u32 {kb}, 0;")
    l_pk = a.L("pk")
    a.label(l_pk)
    eb, fb, par = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {eb}, {stage}, 8, {bars};")
    a(f"add.u32 {eb}, {eb}, {EMPTY};")
    a(f"xor.b32 {par}, {phase}, 1;")
    _wait(a, eb, par, err, ERR_PRODUCER, l_pdone)
    a(f"mad.lo.u32 {fb}, {stage}, 8, {cbars[0]};")    # CTA 0's full barrier of this stage
    a(f"add.u32 {fb}, {fb}, {FULL};")
    lfb = a.r()
    a(f"mad.lo.u32 {lfb}, {stage}, 8, {bars};")
    a(f"add.u32 {lfb}, {lfb}, {FULL};")
    a(f"@{lead} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{lfb}], {TX_PAIR};")
    for s in range(STAGES):
        ps = a.r("p")
        a(f"setp.eq.u32 {ps}, {stage}, {s};")
        a(f"@{ps} mov.u32 {armed[s]}, {phase};")
    dA, dB, kc = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {dA}, {stage}, {A_STAGE}, {sA};")
    a(f"mad.lo.u32 {dB}, {stage}, {B_STAGE}, {sB};")
    a(f"mul.lo.u32 {kc}, {kb}, {BK};")
    a(f"cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
      f"[{dA}], [{tma}, {{{kc}, {mm}, {bb}}}], [{fb}];")
    for j in range(HN // 64):
        nj, dj = a.r(), a.r()
        a(f"add.u32 {nj}, {nn}, {64 * j};")
        a(f"add.u32 {dj}, {dB}, {B_BOX * j};")
        a(f"cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
          f"[{dj}], [{tmb}, {{{nj}, {kc}, {bb}}}], [{fb}];")
    pwrap = a.r("p")
    a(f"add.u32 {stage}, {stage}, 1;")
    a(f"setp.eq.u32 {pwrap}, {stage}, {STAGES};")
    a(f"@{pwrap} mov.u32 {stage}, 0;")
    a(f"@{pwrap} xor.b32 {phase}, {phase}, 1;")
    a(f"add.u32 {kb}, {kb}, 1;")
    pk = a.r("p")
    a(f"setp.lt.u32 {pk}, {kb}, {nk};")
    a(f"@{pk} bra {l_pk};")
    a(f"add.u32 {t}, {t}, {nclu};")
    a(f"bra {l_pt};")
    a.label(l_pdone)
    # drain, so that no load of this thread is in flight when the CTA can finish.  CTA 0 waits for the
    # full barrier of each stage's last round: it completes once both CTAs' bytes have landed, whether
    # or not the MMAs ran.  CTA 1's loads complete CTA 0's barrier, so CTA 1 waits for its empty barrier
    # instead: the MMAs that read the round are done, so its bytes had landed.  CTA 0 arrives at the
    # final cluster barrier only after its own drain.
    for s in range(STAGES):
        skip = a.L("dskip")
        pn = a.r("p")
        a(f"setp.eq.u32 {pn}, {armed[s]}, 2;")
        a(f"@{pn} bra {skip};")
        dbs = a.r()
        a(f"add.u32 {dbs}, {bars}, {EMPTY + 8 * s};")
        a(f"@{lead} add.u32 {dbs}, {bars}, {FULL + 8 * s};")
        _wait(a, dbs, armed[s], err, ERR_DRAIN, skip)
        a.label(skip)
    a(f"bra {l_end};")

    # ---------------- MMA issuer: CTA 0, warp 1, lane 0 ---------------------------------------
    a.label(l_mma)
    pl1 = a.r("p")
    a(f"setp.ne.u32 {pl1}, {lane}, 0;")
    a(f"@{pl1} bra {l_end};")
    a(f"@!{lead} bra {l_end};")                       # CTA 1's tensor core is driven by CTA 0
    mstage, mphase, acc, aphase, mt_, mkb = a.r(), a.r(), a.r(), a.r(), a.r(), a.r()
    a(f"mov.u32 {mstage}, 0;")
    a(f"mov.u32 {mphase}, 0;")
    a(f"mov.u32 {acc}, 0;")
    a(f"mov.u32 {aphase}, 0;")
    a(f"mov.u32 {mt_}, {clu};")
    idr = a.r()
    a(f"mov.u32 {idr}, {idesc};")
    dahi, dbhi = a.r("rd"), a.r("rd")
    a(f"mov.b64 {dahi}, {desc_a_hi};")
    a(f"mov.b64 {dbhi}, {desc_b_hi};")
    l_mt, l_mdone = a.L("mt"), a.L("mdone")
    a.label(l_mt)
    pm = a.r("p")
    a(f"setp.ge.u32 {pm}, {mt_}, {tiles};")
    a(f"@{pm} bra {l_mdone};")
    teb, tpar, dcol = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {teb}, {acc}, 8, {bars};")
    a(f"add.u32 {teb}, {teb}, {TEMPTY};")
    a(f"xor.b32 {tpar}, {aphase}, 1;")
    _wait(a, teb, tpar, err, ERR_MMA_TMEM, l_mdone)   # both CTAs' epilogues have drained it
    a("tcgen05.fence::after_thread_sync;")
    a(f"mad.lo.u32 {dcol}, {acc}, {BN}, {taddr};")
    a(f"mov.u32 {mkb}, 0;")
    l_mk = a.L("mk")
    a.label(l_mk)
    mfb = a.r()
    a(f"mad.lo.u32 {mfb}, {mstage}, 8, {bars};")
    a(f"add.u32 {mfb}, {mfb}, {FULL};")
    _wait(a, mfb, mphase, err, ERR_MMA_FULL, l_mdone)  # both CTAs' halves of the stage are in
    a("tcgen05.fence::after_thread_sync;")
    sa, sb = a.r(), a.r()
    a(f"mad.lo.u32 {sa}, {mstage}, {A_STAGE}, {sA};")
    a(f"mad.lo.u32 {sb}, {mstage}, {B_STAGE}, {sB};")
    for kk in range(BK // 16):
        ra, rb = a.r(), a.r()
        da, db = a.r("rd"), a.r("rd")
        a(f"add.u32 {ra}, {sa}, {32 * kk};")
        a(f"shr.u32 {ra}, {ra}, 4;")
        a(f"add.u32 {rb}, {sb}, {2048 * kk};")
        a(f"shr.u32 {rb}, {rb}, 4;")
        a(f"cvt.u64.u32 {da}, {ra};")
        a(f"cvt.u64.u32 {db}, {rb};")
        a(f"or.b64 {da}, {da}, {dahi};")
        a(f"or.b64 {db}, {db}, {dbhi};")
        pacc = a.r("p")
        if kk == 0:
            a(f"setp.ne.u32 {pacc}, {mkb}, 0;")
        else:
            a(f"setp.eq.u32 {pacc}, {mkb}, {mkb};")
        a(f"tcgen05.mma.cta_group::2.kind::f16 [{dcol}], {da}, {db}, {idr}, {pacc};")
    # the stage is free in both CTAs once these MMAs complete: one commit per CTA's empty barrier
    for r_ in range(2):
        ceb = a.r()
        a(f"mad.lo.u32 {ceb}, {mstage}, 8, {cbars[r_]};")
        a(f"add.u32 {ceb}, {ceb}, {EMPTY};")
        a(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [{ceb}];")
    pw2 = a.r("p")
    a(f"add.u32 {mstage}, {mstage}, 1;")
    a(f"setp.eq.u32 {pw2}, {mstage}, {STAGES};")
    a(f"@{pw2} mov.u32 {mstage}, 0;")
    a(f"@{pw2} xor.b32 {mphase}, {mphase}, 1;")
    a(f"add.u32 {mkb}, {mkb}, 1;")
    pk2 = a.r("p")
    a(f"setp.lt.u32 {pk2}, {mkb}, {nk};")
    a(f"@{pk2} bra {l_mk};")
    for r_ in range(2):
        ctf = a.r()
        a(f"mad.lo.u32 {ctf}, {acc}, 8, {cbars[r_]};")
        a(f"add.u32 {ctf}, {ctf}, {TFULL};")
        a(f"tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [{ctf}];")
    pa = a.r("p")
    a(f"xor.b32 {acc}, {acc}, 1;")
    a(f"setp.eq.u32 {pa}, {acc}, 0;")
    a(f"@{pa} xor.b32 {aphase}, {aphase}, 1;")
    a(f"add.u32 {mt_}, {mt_}, {nclu};")
    a(f"bra {l_mt};")
    a.label(l_mdone)
    a(f"bra {l_end};")

    # ---------------- epilogue: warps 2..5 of each CTA ------------------------------------------
    a.label(l_epi)
    q, eacc, eph, et = a.r(), a.r(), a.r(), a.r()
    a(f"and.b32 {q}, {warp}, 3;")
    lanebase = a.r()
    a(f"shl.b32 {lanebase}, {q}, 21;")                 # (32*q) << 16: this warp's TMEM lanes
    a(f"add.u32 {lanebase}, {lanebase}, {taddr};")
    a(f"mov.u32 {eacc}, 0;")
    a(f"mov.u32 {eph}, 0;")
    a(f"mov.u32 {et}, {clu};")
    erow0 = a.r()
    a(f"mad.lo.u32 {erow0}, {rank}, {HM}, {lane};")    # this CTA's half of the tile, this lane
    a(f"mad.lo.u32 {erow0}, {q}, 32, {erow0};")
    l_et, l_edone = a.L("et"), a.L("edone")
    a.label(l_et)
    pe = a.r("p")
    a(f"setp.ge.u32 {pe}, {et}, {tiles};")
    a(f"@{pe} bra {l_edone};")
    ebb, emm, enn = tile_coords(et)
    efb = a.r()
    a(f"mad.lo.u32 {efb}, {eacc}, 8, {bars};")
    a(f"add.u32 {efb}, {efb}, {TFULL};")
    _wait_warp(a, efb, eph, err, ERR_EPILOGUE, l_edone)
    a("tcgen05.fence::after_thread_sync;")
    # this thread's output row: C + ((b*M + m0 + 128*rank + 32q + lane) * N + n0) * 4
    row, rowaddr, rin = a.r(), a.r("rd"), a.r()
    a(f"add.u32 {rin}, {emm}, {erow0};")              # row within the batch
    prow = None
    if edge_m:
        prow = a.r("p")
        a(f"setp.lt.u32 {prow}, {rin}, {m};")          # rows past M belong to no output
    a(f"mad.lo.u32 {row}, {ebb}, {m}, {rin};")
    tmp64 = a.r("rd")
    a(f"mul.wide.u32 {rowaddr}, {row}, {n * 4};")
    a(f"mul.wide.u32 {tmp64}, {enn}, 4;")
    a(f"add.s64 {rowaddr}, {rowaddr}, {tmp64};")
    a(f"add.s64 {rowaddr}, {rowaddr}, {c_ptr};")
    tcol = a.r()
    a(f"mad.lo.u32 {tcol}, {eacc}, {BN}, {lanebase};")
    for ch in range(BN // 32):
        regs = [a.r("f") for _ in range(32)]
        src = a.r()
        a(f"add.u32 {src}, {tcol}, {32 * ch};")
        a(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(regs)}}}, [{src}];")
        a("tcgen05.wait::ld.sync.aligned;")
        for v in range(4):
            guard = prow
            if edge_n:
                # the 8 columns n0 + 32ch + 8v .. +7 are all below N or all past it (N % 8 == 0)
                lim = n - (32 * ch + 8 * v)
                if lim <= 0:
                    continue
                pc = a.r("p")
                a(f"setp.lt.u32 {pc}, {enn}, {lim};")
                if prow is not None:
                    a(f"and.pred {pc}, {pc}, {prow};")
                guard = pc
            g = f"@{guard} " if guard else ""
            a(f"{g}st.global.v8.f32 [{rowaddr}+{128 * ch + 32 * v}], {{{', '.join(regs[8 * v:8 * v + 8])}}};")
    a("tcgen05.fence::before_thread_sync;")
    a("bar.warp.sync -1;")
    pl = a.r("p")
    a(f"setp.eq.u32 {pl}, {lane}, 0;")
    teb2 = a.r()
    a(f"mad.lo.u32 {teb2}, {eacc}, 8, {cbars[0]};")    # CTA 0's tmem_empty: its issuer waits on it
    a(f"add.u32 {teb2}, {teb2}, {TEMPTY};")
    a(f"@{pl} mbarrier.arrive.release.cluster.shared::cluster.b64 _, [{teb2}];")
    pa2 = a.r("p")
    a(f"xor.b32 {eacc}, {eacc}, 1;")
    a(f"setp.eq.u32 {pa2}, {eacc}, 0;")
    a(f"@{pa2} xor.b32 {eph}, {eph}, 1;")
    a(f"add.u32 {et}, {et}, {nclu};")
    a(f"bra {l_et};")
    a.label(l_edone)

    # ---------------- teardown -------------------------------------------------------------
    # every thread of both CTAs: nothing of the partner's addresses this CTA's shared memory or
    # tensor memory any more once both have arrived
    a.label(l_end)
    a("barrier.cluster.arrive.release;")
    a("barrier.cluster.wait.acquire;")
    a("bar.warp.sync -1;")
    l_nodealloc = a.L("nodealloc")
    a(f"@!{pw1} bra {l_nodealloc};")
    a("tcgen05.fence::after_thread_sync;")
    a(f"tcgen05.dealloc.cta_group::2.sync.aligned.b32 {taddr}, {TMEM_COLS};")
    a.label(l_nodealloc)

    dyn = STAGES * (A_STAGE + B_STAGE) + 1024 + 1024
    entry = [f".visible .entry {name}(",
             "\t.param .u64 p_A,", "\t.param .u64 p_B,", "\t.param .u64 p_C,",
             "\t.param .align 64 .b8 p_tmA[128],", "\t.param .align 64 .b8 p_tmB[128],",
             "\t.param .u64 p_err", ")",
             f".reqntid {THREADS}, 1, 1", ".reqnctapercluster 2, 1, 1", ".maxnreg 168", "{"]
    entry += a.decls() + a.lines + ["\tret;", "}"]
    xn, yn, cn = names
    tmaps = [
        {"name": "tmA", "tensor": xn, "dtype": "bf16", "dims": [k, m, batch], "strides": [k * 2, m * k * 2],
         "box": [BK, HM, 1], "swizzle": "128B"},
        {"name": "tmB", "tensor": yn, "dtype": "bf16", "dims": [n, k, batch], "strides": [n * 2, k * n * 2],
         "box": [64, BK, 1], "swizzle": "128B"},
    ]
    return {
        "name": name, "kind": "tcgen05_gemm_pair", "params": [xn, yn, cn],
        "raw_entry": entry, "raw_decls": [f".extern .shared .align 1024 .b8 {smem_sym}[];"],
        "grid": [2 * clusters, 1, 1], "block": [THREADS, 1, 1], "cluster": [2, 1, 1], "dyn_smem": dyn,
        "align": {xn: 16, yn: 16, cn: 32}, "zero_outputs": [], "tmaps": tmaps,
        "extra": [{"name": "__err", "kind": "errword"}], "tiles": tiles,
    }
