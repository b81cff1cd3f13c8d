"""The multi-GPU sum's exchange step over NVLink peer memory: a one-warp kernel, or the reduction's epilogue.

Config 2 at N GPUs: each rank reduces its shard into a one-element partial, then every rank needs the
total.  Instead of a one-element ``ncclAllReduce`` the partials go through an exchange buffer that every
rank allocates and maps into every other rank's process (CUDA IPC, ``dist.PeerAllReduce``):

* the buffer of rank q holds a step counter (only rank q touches it), two slots per source rank
  (``DATA``, double-buffered by the step's parity) and one flag per source rank (``FLAGS``);
* one warp per rank: lane 0 advances the step counter to e; lane r (< N) writes this rank's partial into
  slot [e & 1][rank] of rank r's buffer and then, with a release store at system scope, e into flag
  [rank] of that buffer;
* lane k (< N) waits with acquire loads for flag [k] of its own buffer to reach e (bounded by
  %globaltimer: after ``WAIT_NS`` it writes status code 51 and goes on), then reads slot [e & 1][k];
* the partials are added in rank order 0..N-1, so every rank computes the same bits, and lane 0 writes
  the total over the partial.

The parity slots make reuse safe: rank p writes slot [e & 1][p] of rank q's buffer again only at step
e + 2, and it gets there only after seeing rank q's flag for step e + 1, which rank q writes after it has
read step e's slots.  All loads and stores are plain peer accesses; no multicast object is used.

:func:`peer_sum_entry` is the exchange as its own kernel, launched right after the reduction.
:func:`emit_exchange` writes the same steps into another kernel: the generic emitter's ``exchange``
option appends them to the reduction kernel, run by warp 0 of the block that finishes last (the ticket
of the reduction's self-zeroing accumulator scratch picks it), so the reduction and the exchange are one
launch and the partial needs no zeroing before it.
"""
from __future__ import annotations

STEP = 0                 # u32 step counter (written by the owning rank only)
DATA = 256               # u64 slots [2][MAX_RANKS]
FLAGS = 1024             # u32 flags [MAX_RANKS]
MAX_RANKS = 32
BUF_BYTES = 2048
WAIT_NS = 2_000_000_000  # 2 s
ERR_PEER_WAIT = 51


def emit_exchange(emit, reg, label, lane: str, out: str, xch: str, peers: str, err: str,
                  rank: int, world: int, dtype: str) -> None:
    """The exchange, executed by one whole warp: ``lane`` its lane index (b32 register); ``out``,
    ``xch``, ``peers`` and ``err`` global addresses (b64 registers) of the one-element partial, this
    rank's exchange buffer, the table of every rank's buffer and the status word.  ``emit(line)``
    appends an instruction or label (``name:``); ``reg(cls)`` returns a fresh register of class
    ``"b32"``, ``"b64"``, ``"pred"`` or ``"f32"``; ``label(tag)`` a fresh label."""
    if dtype not in ("f32", "i32"):
        raise ValueError("the peer exchange sums f32 or i32")
    if not 1 <= world <= MAX_RANKS or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world} outside 1..{MAX_RANKS} ranks")
    r = lambda: reg("b32")                     # noqa: E731
    rd = lambda: reg("b64")                    # noqa: E731
    pr = lambda: reg("pred")                   # noqa: E731
    p_first, e, v, par, slot, val = pr(), r(), r(), r(), r(), r()
    emit(f"setp.eq.u32 {p_first}, {lane}, 0;")
    # step e = counter + 1 (every lane reads it before lane 0 writes it back)
    emit(f"ld.global.u32 {e}, [{xch}+{STEP}];")
    emit(f"add.u32 {e}, {e}, 1;")
    emit("bar.warp.sync -1;")
    emit(f"@{p_first} st.global.u32 [{xch}+{STEP}], {e};")
    emit(f"ld.global.b32 {v}, [{out}];")                     # this rank's partial (bits)
    emit(f"and.b32 {par}, {e}, 1;")                          # parity of the step
    emit(f"mul.lo.u32 {slot}, {par}, {8 * world};")
    emit(f"add.u32 {slot}, {slot}, {DATA + 8 * rank};")      # slot [e & 1][rank] in a buffer
    emit(f"mov.b32 {val}, 0;")                               # partial of rank `lane` (read below)
    p_in, done, top, got = pr(), label("xdone"), label("xwait"), label("xgot")
    emit(f"setp.lt.u32 {p_in}, {lane}, {world};")
    emit(f"@!{p_in} bra {done};")
    # lane r: publish to rank r
    ta, peer, dst = rd(), rd(), rd()
    emit(f"mul.wide.u32 {ta}, {lane}, 8;")
    emit(f"add.s64 {ta}, {ta}, {peers};")
    emit(f"ld.global.u64 {peer}, [{ta}];")                   # rank r's buffer, mapped here
    emit(f"cvt.u64.u32 {dst}, {slot};")
    emit(f"add.s64 {dst}, {dst}, {peer};")
    emit(f"st.global.b32 [{dst}], {v};")
    emit(f"st.release.sys.global.u32 [{peer}+{FLAGS + 4 * rank}], {e};")
    # lane k: wait for rank k's flag in this rank's buffer, then read its slot
    fa, t0, t1 = rd(), rd(), rd()
    f, p_ok, p_more = r(), pr(), pr()
    emit(f"mul.wide.u32 {fa}, {lane}, 4;")
    emit(f"add.s64 {fa}, {fa}, {xch};")
    emit(f"mov.u64 {t0}, %globaltimer;")
    emit(f"{top}:")
    emit(f"ld.acquire.sys.global.u32 {f}, [{fa}+{FLAGS}];")
    emit(f"setp.ge.u32 {p_ok}, {f}, {e};")
    emit(f"@{p_ok} bra {got};")
    emit(f"mov.u64 {t1}, %globaltimer;")
    emit(f"sub.s64 {t1}, {t1}, {t0};")
    emit(f"setp.lt.s64 {p_more}, {t1}, {WAIT_NS};")
    emit(f"@{p_more} bra {top};")
    emit(f"st.global.u32 [{err}], {ERR_PEER_WAIT};")
    emit(f"{got}:")
    so, sa = r(), rd()
    emit(f"mul.lo.u32 {so}, {par}, {8 * world};")
    emit(f"mad.lo.u32 {so}, {lane}, 8, {so};")
    emit(f"cvt.u64.u32 {sa}, {so};")
    emit(f"add.s64 {sa}, {sa}, {xch};")
    emit(f"ld.global.b32 {val}, [{sa}+{DATA}];")
    emit(f"{done}:")
    emit("bar.warp.sync -1;")
    # the total in rank order (the same bits on every rank)
    x = r()
    if dtype == "f32":
        tot, xf = reg("f32"), reg("f32")
        emit(f"mov.b32 {tot}, 0f00000000;")
    else:
        tot = r()
        emit(f"mov.u32 {tot}, 0;")
    for k in range(world):
        emit(f"shfl.sync.idx.b32 {x}, {val}, {k}, 31, -1;")
        if dtype == "f32":
            emit(f"mov.b32 {xf}, {x};")
            emit(f"add.rn.f32 {tot}, {tot}, {xf};")
        else:
            emit(f"add.s32 {tot}, {tot}, {x};")
    emit(f"@{p_first} st.global.{'f32' if dtype == 'f32' else 's32'} [{out}], {tot};")


class _Regs:
    """Numbered registers per class for the standalone kernel."""

    PREFIX = {"b32": "%r", "b64": "%rd", "pred": "%p", "f32": "%f"}

    def __init__(self):
        self.n = {k: 0 for k in self.PREFIX}
        self.labels = 0

    def __call__(self, cls):
        self.n[cls] += 1
        return f"{self.PREFIX[cls]}{self.n[cls]}"

    def label(self, tag):
        self.labels += 1
        return f"$X{self.labels}_{tag}"

    def decls(self):
        ty = {"b32": ".b32", "b64": ".b64", "pred": ".pred", "f32": ".f32"}
        return [f"\t.reg {ty[c]} {self.PREFIX[c]}<{k + 1}>;" for c, k in self.n.items() if k]


def peer_sum_entry(name: str, rank: int, world: int, dtype: str) -> dict:
    """The exchange kernel for ``rank`` of ``world`` (one warp) as a raw-entry build record; parameters
    ``out`` (the one-element partial, replaced by the total), ``xch`` (this rank's exchange buffer),
    ``peers`` (``world`` u64: every rank's exchange buffer as mapped in this process) and ``err``."""
    regs = _Regs()
    lines = []

    def emit(line):
        lines.append(line if line.endswith(":") else "\t" + line)

    lane = regs("b32")
    emit(f"mov.u32 {lane}, %tid.x;")
    ptrs = {}
    for nm in ("out", "xch", "peers", "err"):
        ptrs[nm] = regs("b64")
        emit(f"ld.param.u64 {ptrs[nm]}, [p_{nm}];")
        emit(f"cvta.to.global.u64 {ptrs[nm]}, {ptrs[nm]};")
    emit_exchange(emit, regs, regs.label, lane, ptrs["out"], ptrs["xch"], ptrs["peers"], ptrs["err"],
                  rank, world, dtype)
    entry = [f".visible .entry {name}(", "\t.param .u64 p_out,", "\t.param .u64 p_xch,", "\t.param .u64 p_peers,",
             "\t.param .u64 p_err", ")", ".reqntid 32, 1, 1", "{"] + regs.decls() + lines + ["\tret;", "}"]
    return {"name": name, "kind": "peer_exchange", "params": ["out", "xch", "peers"], "raw_entry": entry,
            "raw_decls": [], "grid": [1, 1, 1], "block": [32, 1, 1], "dyn_smem": 0,
            "align": {"out": 4, "xch": 256, "peers": 8}, "zero_outputs": [],
            "extra": [{"name": "__err", "kind": "errword"}]}
