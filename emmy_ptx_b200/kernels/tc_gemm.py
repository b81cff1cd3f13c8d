"""Batched bf16 GEMM with f32 accumulation on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).

C[b] = A[b] @ B[b] with A [batch, M, K] (K contiguous), B [batch, K, N] (N contiguous) and
C [batch, M, N] f32 — the dense contraction a matmul Accum loop nest computes (the bmm IR of
config 4).  The kernel is written here as PTX text, instruction by instruction:

* persistent: one CTA per SM walks output tiles ``t = ctaid, ctaid + nctaid, ...``, n fastest, so
  the CTAs in flight share A row panels and the whole B matrix through L2;
* warp-specialised, 192 threads: warp 0 issues TMA loads, warp 1 owns TMEM and issues
  ``tcgen05.mma`` from one thread, warps 2-5 drain the accumulator (each reads the 32 TMEM lanes
  its warp is allowed to address) and store f32 rows with 256-bit stores;
* a 4-stage ring of 48 KiB stages (A 128x64, B 64x256, 128-byte swizzle) synchronised by
  mbarriers: ``full`` (TMA transaction bytes) and ``empty`` (``tcgen05.commit`` of the MMAs that
  read the stage);
* two 128x256 f32 accumulators in TMEM (all 512 columns), so the epilogue of one tile overlaps
  the MMAs of the next (``tmem_full`` / ``tmem_empty`` barriers);
* branches are plain ``bra``: several depend on the lane (one elected thread per role), and a
  ``bra.uni`` there would promise a warp-uniform branch that is not;
* every mbarrier wait is bounded: on time-out the thread writes a code to the error word and
  leaves its loop; the producer then waits (bounded) for its own loads in flight, all threads meet
  at the final barrier and warp 1 frees TMEM, so the kernel always returns.

Instruction descriptor (kind::f16): D f32, A/B bf16, A K-major, B MN-major, M=128, N=256.
Shared-memory matrix descriptors: SWIZZLE_128B; A canonical K-major (8-row groups 1024 B apart);
B canonical MN-major (64-column atoms 8 KiB apart = leading offset, 8-row groups 1024 B apart =
stride offset).  One MMA consumes K=16: A's start address advances 32 B, B's 16 rows = 2 KiB.
"""
from __future__ import annotations

BM, BN, BK = 128, 256, 64
STAGES = 4
A_STAGE = BM * BK * 2            # 16 KiB
B_STAGE = BK * BN * 2            # 32 KiB
B_BOX = BK * 64 * 2              # one 64-column TMA box of B: 8 KiB
TX_BYTES = A_STAGE + B_STAGE
THREADS = 192
TMEM_COLS = 512

# error codes written to the error word
ERR_PRODUCER = 1
ERR_MMA_FULL = 2
ERR_MMA_TMEM = 3
ERR_EPILOGUE = 4
ERR_DRAIN = 5


from .ptxasm import Asm, idesc_f16, smem_desc_hi, wait_bar as _wait, wait_bar_warp as _wait_warp


def supported(m: int, n: int, k: int) -> bool:
    """Whether the tcgen05 GEMM takes these shapes: any M; N and K multiples of 8, so that the
    row strides of A (K bf16) and B (N bf16) are whole 16-byte units as TMA requires, and C's f32
    rows split into whole 32-byte stores."""
    return m >= 1 and n >= 8 and k >= 8 and n % 8 == 0 and k % 8 == 0


def gemm_entry(name: str, batch: int, m: int, n: int, k: int, sms: int = 148,
               names=("A", "B", "C"), prefix: str = "") -> dict:
    """The build record (module writer format) of the tcgen05 GEMM for these shapes; ``names`` are
    the IR buffer names of X, Y and the output (the kernel's parameters, in that order).

    Shapes that are not tile multiples run as edge tiles: TMA fills the parts of an A or B box past
    the tensor's end with zeros (their products add nothing, in K too), and the epilogue stores only
    the rows below M and the 8-column groups below N."""
    if not supported(m, n, k):
        raise ValueError("tcgen05 GEMM needs N % 8 == 0 and K % 8 == 0")
    mt, nt, nk = -(-m // BM), -(-n // BN), -(-k // BK)
    edge_m, edge_n = m % BM != 0, n % BN != 0
    tiles = batch * mt * nt
    grid = min(tiles, sms)
    a = Asm()
    idesc = idesc_f16(BM, BN, False, True)
    desc_a_hi = smem_desc_hi(16, 1024)
    desc_b_hi = smem_desc_hi(B_BOX, 1024)

    tid, warp, lane, cta, ncta = a.r(), a.r(), a.r(), a.r(), a.r()
    a(f"mov.u32 {tid}, %tid.x;")
    a(f"shr.u32 {warp}, {tid}, 5;")
    a(f"and.b32 {lane}, {tid}, 31;")
    a(f"mov.u32 {cta}, %ctaid.x;")
    a(f"mov.u32 {ncta}, %nctaid.x;")
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

    # shared layout (1024-aligned base): A stages, B stages, then barriers and the TMEM slot
    raw, base = a.r(), a.r()
    smem_sym = f"{prefix}gemm_smem"
    a(f"mov.u32 {raw}, {smem_sym};")
    a(f"add.u32 {base}, {raw}, 1023;")
    a(f"and.b32 {base}, {base}, -1024;")
    sA, sB, bars = a.r(), a.r(), a.r()
    a(f"mov.u32 {sA}, {base};")
    a(f"add.u32 {sB}, {base}, {STAGES * A_STAGE};")
    a(f"add.u32 {bars}, {base}, {STAGES * (A_STAGE + B_STAGE)};")
    # barrier offsets from `bars`
    FULL, EMPTY, TFULL, TEMPTY, SLOT = 0, 8 * STAGES, 16 * STAGES, 16 * STAGES + 16, 16 * STAGES + 32

    p0 = a.r("p")
    a(f"setp.eq.u32 {p0}, {tid}, 0;")
    l_init = a.L("noinit")
    a(f"@!{p0} bra {l_init};")
    for s in range(STAGES):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{FULL + 8 * s}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{EMPTY + 8 * s}], 1;")
    for acc in range(2):
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{TFULL + 8 * acc}], 1;")
        a(f"mbarrier.init.shared::cta.b64 [{bars}+{TEMPTY + 8 * acc}], 4;")
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

    # ---------------- producer: warp 0, lane 0 ------------------------------------------
    a.label(l_prod)
    pl0 = a.r("p")
    a(f"setp.ne.u32 {pl0}, {lane}, 0;")
    a(f"@{pl0} bra {l_end};")
    stage, phase, t, kb = a.r(), a.r(), a.r(), a.r()
    armed = [a.r() for _ in range(STAGES)]          # parity each stage's full barrier must reach
    for r_ in armed:
        a(f"mov.u32 {r_}, 2;")
    a(f"mov.u32 {stage}, 0;")
    a(f"mov.u32 {phase}, 0;")
    a(f"mov.u32 {t}, {cta};")
    l_pt, l_pdone, l_pbail = a.L("pt"), a.L("pdone"), a.L("pbail")
    a.label(l_pt)
    pt = a.r("p")
    a(f"setp.ge.u32 {pt}, {t}, {tiles};")
    a(f"@{pt} bra {l_pdone};")
    bb, mm, nn = tile_coords(t)
    a(f"mov.u32 {kb}, 0;")
    l_pk = a.L("pk")
    a.label(l_pk)
    eb, fb, par = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {eb}, {stage}, 8, {bars};")
    a(f"add.u32 {fb}, {eb}, {FULL}];".replace("];", ";"))
    a(f"add.u32 {eb}, {eb}, {EMPTY};")
    a(f"xor.b32 {par}, {phase}, 1;")
    _wait(a, eb, par, err, ERR_PRODUCER, l_pbail)
    a(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {TX_BYTES};")
    # remember which parity this stage's full barrier will complete
    for s in range(STAGES):
        ps = a.r("p")
        a(f"setp.eq.u32 {ps}, {stage}, {s};")
        a(f"@{ps} mov.u32 {armed[s]}, {phase};")
    dA, dB, kc = a.r(), a.r(), a.r()
    a(f"mad.lo.u32 {dA}, {stage}, {A_STAGE}, {sA};")
    a(f"mad.lo.u32 {dB}, {stage}, {B_STAGE}, {sB};")
    a(f"mul.lo.u32 {kc}, {kb}, {BK};")
    a(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      f"[{dA}], [{tma}, {{{kc}, {mm}, {bb}}}], [{fb}];")
    for j in range(BN // 64):
        nj, dj = a.r(), a.r()
        a(f"add.u32 {nj}, {nn}, {64 * j};")
        a(f"add.u32 {dj}, {dB}, {B_BOX * j};")
        a(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
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
    a(f"add.u32 {t}, {t}, {ncta};")
    a(f"bra {l_pt};")
    a.label(l_pbail)
    a.label(l_pdone)
    # drain: every load this thread issued has landed before the CTA can finish
    for s in range(STAGES):
        skip = a.L("dskip")
        pn = a.r("p")
        a(f"setp.eq.u32 {pn}, {armed[s]}, 2;")
        a(f"@{pn} bra {skip};")
        fbs = a.r()
        a(f"add.u32 {fbs}, {bars}, {FULL + 8 * s};")
        _wait(a, fbs, armed[s], err, ERR_DRAIN, skip)
        a.label(skip)
    a(f"bra {l_end};")

    # ---------------- MMA issuer: warp 1, lane 0 -----------------------------------------
    a.label(l_mma)
    pl1 = a.r("p")
    a(f"setp.ne.u32 {pl1}, {lane}, 0;")
    a(f"@{pl1} bra {l_end};")
    mstage, mphase, acc, aphase, mt_, mkb = a.r(), a.r(), a.r(), a.r(), a.r(), a.r()
    a(f"mov.u32 {mstage}, 0;")
    a(f"mov.u32 {mphase}, 0;")
    a(f"mov.u32 {acc}, 0;")
    a(f"mov.u32 {aphase}, 0;")
    a(f"mov.u32 {mt_}, {cta};")
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
    _wait(a, teb, tpar, err, ERR_MMA_TMEM, l_mdone)
    a("tcgen05.fence::after_thread_sync;")
    a(f"mad.lo.u32 {dcol}, {acc}, {BN}, {taddr};")
    a(f"mov.u32 {mkb}, 0;")
    l_mk = a.L("mk")
    a.label(l_mk)
    mfb = a.r()
    a(f"mad.lo.u32 {mfb}, {mstage}, 8, {bars};")
    a(f"add.u32 {mfb}, {mfb}, {FULL};")
    _wait(a, mfb, mphase, err, ERR_MMA_FULL, l_mdone)
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
        a(f"tcgen05.mma.cta_group::1.kind::f16 [{dcol}], {da}, {db}, {idr}, {pacc};")
    meb = a.r()
    a(f"mad.lo.u32 {meb}, {mstage}, 8, {bars};")
    a(f"add.u32 {meb}, {meb}, {EMPTY};")
    a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{meb}];")
    pw2 = a.r("p")
    a(f"add.u32 {mstage}, {mstage}, 1;")
    a(f"setp.eq.u32 {pw2}, {mstage}, {STAGES};")
    a(f"@{pw2} mov.u32 {mstage}, 0;")
    a(f"@{pw2} xor.b32 {mphase}, {mphase}, 1;")
    a(f"add.u32 {mkb}, {mkb}, 1;")
    pk2 = a.r("p")
    a(f"setp.lt.u32 {pk2}, {mkb}, {nk};")
    a(f"@{pk2} bra {l_mk};")
    tfb = a.r()
    a(f"mad.lo.u32 {tfb}, {acc}, 8, {bars};")
    a(f"add.u32 {tfb}, {tfb}, {TFULL};")
    a(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{tfb}];")
    pa = a.r("p")
    a(f"xor.b32 {acc}, {acc}, 1;")
    a(f"setp.eq.u32 {pa}, {acc}, 0;")
    a(f"@{pa} xor.b32 {aphase}, {aphase}, 1;")
    a(f"add.u32 {mt_}, {mt_}, {ncta};")
    a(f"bra {l_mt};")
    a.label(l_mdone)
    a(f"bra {l_end};")

    # ---------------- epilogue: warps 2..5 -------------------------------------------------
    a.label(l_epi)
    q, eacc, eph, et = a.r(), a.r(), a.r(), a.r()
    a(f"and.b32 {q}, {warp}, 3;")
    lanebase = a.r()
    a(f"shl.b32 {lanebase}, {q}, 21;")                 # (32*q) << 16: this warp's TMEM lanes
    a(f"add.u32 {lanebase}, {lanebase}, {taddr};")
    a(f"mov.u32 {eacc}, 0;")
    a(f"mov.u32 {eph}, 0;")
    a(f"mov.u32 {et}, {cta};")
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
    # this thread's output row: C + ((b*M + m0 + 32q + lane) * N + n0) * 4
    row, rowaddr = a.r(), a.r("rd")
    rin = a.r()
    a(f"mad.lo.u32 {rin}, {q}, 32, {emm};")
    a(f"add.u32 {rin}, {rin}, {lane};")                # row within the batch
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
                # the 8 columns n0 + 32ch + 8v .. +7 are all below N or all past it (N % 8 == 0);
                # a group past N in the first tile is past N in every tile
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
    a(f"mad.lo.u32 {teb2}, {eacc}, 8, {bars};")
    a(f"add.u32 {teb2}, {teb2}, {TEMPTY};")
    a(f"@{pl} mbarrier.arrive.shared::cta.b64 _, [{teb2}];")
    pa2 = a.r("p")
    a(f"xor.b32 {eacc}, {eacc}, 1;")
    a(f"setp.eq.u32 {pa2}, {eacc}, 0;")
    a(f"@{pa2} xor.b32 {eph}, {eph}, 1;")
    a(f"add.u32 {et}, {et}, {ncta};")
    a(f"bra {l_et};")
    a.label(l_edone)

    # ---------------- teardown -------------------------------------------------------------
    a.label(l_end)
    a("barrier.sync 0;")
    a("bar.warp.sync -1;")
    l_nodealloc = a.L("nodealloc")
    a(f"@!{pw1} bra {l_nodealloc};")
    a("tcgen05.fence::after_thread_sync;")
    a(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {taddr}, {TMEM_COLS};")
    a.label(l_nodealloc)

    dyn = STAGES * (A_STAGE + B_STAGE) + 1024 + 1024
    entry = [f".visible .entry {name}(",
             "\t.param .u64 p_A,", "\t.param .u64 p_B,", "\t.param .u64 p_C,",
             "\t.param .align 64 .b8 p_tmA[128],", "\t.param .align 64 .b8 p_tmB[128],",
             "\t.param .u64 p_err", ")",
             f".reqntid {THREADS}, 1, 1", ".maxnreg 168", "{"]
    entry += a.decls() + a.lines + ["\tret;", "}"]
    xn, yn, cn = names
    tmaps = [
        {"name": "tmA", "tensor": xn, "dtype": "bf16", "dims": [k, m, batch], "strides": [k * 2, m * k * 2],
         "box": [BK, BM, 1], "swizzle": "128B"},
        {"name": "tmB", "tensor": yn, "dtype": "bf16", "dims": [n, k, batch], "strides": [n * 2, k * n * 2],
         "box": [64, BK, 1], "swizzle": "128B"},
    ]
    return {
        "name": name, "kind": "tcgen05_gemm", "params": [xn, yn, cn],
        "raw_entry": entry, "raw_decls": [f".extern .shared .align 1024 .b8 {smem_sym}[];"],
        "grid": [grid, 1, 1], "block": [THREADS, 1, 1], "dyn_smem": dyn, "align": {xn: 16, yn: 16, cn: 32},
        "zero_outputs": [], "tmaps": tmaps, "extra": [{"name": "__err", "kind": "errword"}],
        "tiles": tiles,
    }
