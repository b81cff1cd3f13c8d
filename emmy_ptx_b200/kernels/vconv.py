"""The attention kernel's value pre-pass: V bf16 -> f16 once per launch, with a per-block range flag.

The tensor core multiplies operands of one type, so the f16 P of the attention kernel needs V in f16.
Every 64-row key/value block of V [batch, heads, S, 128] is converted here (one CTA per block, 16-byte
loads and stores, 256 threads) into a scratch tensor of the same shape, and the block's flag records
whether it fits: 0 when every |v| is at most 65,280 (the largest bf16 value below the f16 overflow
threshold), 1 otherwise.  The attention kernel then loads each block from the f16 copy or, for a
flagged block, from V itself with P as two bf16 parts.  Each CTA writes its own flag, so nothing needs
zeroing first.  When S is no multiple of 64 each (batch, head) ends with a partial block: its rows past
S are neither read nor written, and its flag covers the rows it has.
"""
from __future__ import annotations

from .ptxasm import Asm

THREADS = 256
BLOCK_ROWS = 64
D = 128
BLOCK_BYTES = BLOCK_ROWS * D * 2          # 16 KiB of bf16 in, the same of f16 out
F16_MAX_BF16_BITS = 0x477F


def vconv_entry(name: str, batch: int, heads: int, seq: int, names=("V", "__v16", "__vflag"),
                bh_range: tuple[int, int] | None = None, ctas: int | None = None,
                block_rows: int = BLOCK_ROWS, dim: int = D) -> dict:
    """The pre-pass entry; ``bh_range`` = (first, count) converts only those flattened (batch, head)
    pairs (their blocks and flags sit at the same places as in a whole-tensor launch).  ``ctas``
    caps the grid: each CTA then strides over the blocks, which keeps the launch to one CTA per SM
    when it shares the GPU with a concurrent kernel.  ``block_rows`` is the attention kernel's key /
    value block (64, or 128 for the 128-row kernel): one CTA and one flag per block."""
    if block_rows not in (64, 128):
        raise ValueError("the value pre-pass converts 64- or 128-row blocks")
    ragged = seq % block_rows != 0
    if ragged and block_rows != BLOCK_ROWS:
        raise ValueError(f"the {block_rows}-row value pre-pass needs S % {block_rows} == 0")
    if dim not in (32, 64, 128):
        raise ValueError("the value pre-pass converts head dim 32, 64 or 128")
    block_bytes = block_rows * dim * 2
    bh0, nbh = bh_range if bh_range is not None else (0, batch * heads)
    if not (0 <= bh0 and nbh > 0 and bh0 + nbh <= batch * heads):
        raise ValueError(f"bh_range {bh_range} outside the {batch * heads} (batch, head) pairs")
    per_bh = -(-seq // block_rows)          # blocks per (batch, head); the last one partial when ragged
    blocks = nbh * per_bh
    first = bh0 * per_bh
    vec = block_bytes // 16 // THREADS      # 16-byte vectors per thread
    grid = blocks if not ctas else min(blocks, int(ctas))
    a = Asm()
    tid, blk = a.r(), a.r()
    a(f"mov.u32 {tid}, %tid.x;")
    a(f"mov.u32 {blk}, %ctaid.x;")
    if first:
        a(f"add.u32 {blk}, {blk}, {first};")
    pv, p16, pf = a.r("rd"), a.r("rd"), a.r("rd")
    for reg, pname in ((pv, "p_V"), (p16, "p_V16"), (pf, "p_flag")):
        a(f"ld.param.u64 {reg}, [{pname}];")
        a(f"cvta.to.global.u64 {reg}, {reg};")
    l_top, l_done = a.L("blk"), a.L("alldone")
    if grid < blocks:
        a.label(l_top)
        pend = a.r("p")
        a(f"setp.ge.u32 {pend}, {blk}, {first + blocks};")
        a(f"@{pend} bra {l_done};")
    off = a.r("rd")
    lim = None
    if ragged:
        # block j of pair bh starts at row bh*S + 64*j; its rows past S are neither read nor written
        # (lim = the block's valid bytes, compared with each 16-byte vector's offset in the block)
        bhr, jr, rows_, lim = a.r(), a.r(), a.r(), a.r()
        a(f"div.u32 {bhr}, {blk}, {per_bh};")
        a(f"rem.u32 {jr}, {blk}, {per_bh};")
        a(f"mul.lo.u32 {rows_}, {jr}, {block_rows};")
        a(f"sub.u32 {lim}, {seq}, {rows_};")
        a(f"min.u32 {lim}, {lim}, {block_rows};")
        a(f"mul.lo.u32 {lim}, {lim}, {dim * 2};")
        a(f"mad.lo.u32 {rows_}, {bhr}, {seq}, {rows_};")
        a(f"mul.wide.u32 {off}, {rows_}, {dim * 2};")
    else:
        a(f"mul.wide.u32 {off}, {blk}, {block_bytes};")
    t16 = a.r("rd")
    a(f"mul.wide.u32 {t16}, {tid}, 16;")
    a(f"add.s64 {off}, {off}, {t16};")
    src, dst = a.r("rd"), a.r("rd")
    a(f"add.s64 {src}, {pv}, {off};")
    a(f"add.s64 {dst}, {p16}, {off};")
    m = a.r()
    a(f"mov.u32 {m}, 0;")
    ws_all, preds = [], []
    for v in range(vec):
        ws = [a.r() for _ in range(4)]
        g = ""
        if ragged:
            pin, boff = a.r("p"), a.r()
            a(f"mad.lo.u32 {boff}, {tid}, 16, {v * THREADS * 16};")
            a(f"setp.lt.u32 {pin}, {boff}, {lim};")
            for w in ws:
                a(f"mov.u32 {w}, 0;")
            g = f"@{pin} "
        preds.append(g)
        a(f"{g}ld.global.nc.v4.b32 {{{', '.join(ws)}}}, [{src}+{v * THREADS * 16}];")
        ws_all.append(ws)
    for v, ws in enumerate(ws_all):
        out = []
        for w in ws:
            t_, lo_, hi_, f_ = a.r(), a.r("f"), a.r("f"), a.r()
            a(f"and.b32 {t_}, {w}, 0x7FFF7FFF;")
            a(f"max.u16x2 {m}, {m}, {t_};")
            a(f"shl.b32 {lo_}, {w}, 16;")
            a(f"and.b32 {hi_}, {w}, -65536;")
            a(f"cvt.rn.f16x2.f32 {f_}, {hi_}, {lo_};")
            out.append(f_)
        a(f"{preds[v]}st.global.v4.b32 [{dst}+{v * THREADS * 16}], {{{', '.join(out)}}};")
    mlo, mhi, p1, p2, ovf = a.r(), a.r(), a.r("p"), a.r("p"), a.r("p")
    a(f"and.b32 {mlo}, {m}, 65535;")
    a(f"shr.u32 {mhi}, {m}, 16;")
    a(f"setp.gt.u32 {p1}, {mlo}, {F16_MAX_BF16_BITS};")
    a(f"setp.gt.u32 {p2}, {mhi}, {F16_MAX_BF16_BITS};")
    a(f"or.pred {p1}, {p1}, {p2};")
    # the whole block's verdict (every thread of the CTA takes part; no wait on anything outside it)
    a(f"bar.red.or.pred {ovf}, 0, {p1};")
    p0 = a.r("p")
    a(f"setp.eq.u32 {p0}, {tid}, 0;")
    fv, fa = a.r(), a.r("rd")
    a(f"selp.u32 {fv}, 1, 0, {ovf};")
    a(f"mul.wide.u32 {fa}, {blk}, 4;")
    a(f"add.s64 {fa}, {fa}, {pf};")
    a(f"@{p0} st.global.u32 [{fa}], {fv};")
    if grid < blocks:
        a(f"add.u32 {blk}, {blk}, {grid};")
        a(f"bra {l_top};")
        a.label(l_done)
    entry = [f".visible .entry {name}(", "\t.param .u64 p_V,", "\t.param .u64 p_V16,", "\t.param .u64 p_flag", ")",
             f".reqntid {THREADS}, 1, 1", "{"] + a.decls() + a.lines + ["\tret;", "}"]
    vn, v16n, fn = names
    return {
        "name": name, "kind": "value_prepass", "params": [vn, v16n, fn], "raw_entry": entry,
        "grid": [grid, 1, 1], "block": [THREADS, 1, 1], "dyn_smem": 0,
        "align": {vn: 16, v16n: 16, fn: 4}, "zero_outputs": [],
        "scratch": [{"name": v16n, "dtype": "f16", "shape": [batch, heads, seq, dim]},
                    {"name": fn, "dtype": "i32", "shape": [batch * heads * per_bh]}],
    }
