"""The multi-GPU sum's exchange step as one small kernel over NVLink peer memory.

Config 2 at N GPUs: each rank reduces its shard into a one-element partial, then every rank needs the
total.  Instead of a one-element ``ncclAllReduce`` this kernel, launched right after the reduction on
the same stream, exchanges the partials through an exchange buffer that every rank allocates and maps
into every other rank's process (CUDA IPC, ``dist.PeerAllReduce``):

* the buffer of rank q holds a step counter (only rank q writes it), two slots per source rank
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
read step e's slots.  No step holds an NCCL call, so a multi-GPU step (zeroing, reduction, exchange) can
replay from a CUDA graph.  All loads and stores are plain peer accesses; no multicast object is used.
"""
from __future__ import annotations

STEP = 0                 # u32 step counter (written by the owning rank only)
DATA = 256               # u64 slots [2][MAX_RANKS]
FLAGS = 1024             # u32 flags [MAX_RANKS]
MAX_RANKS = 32
BUF_BYTES = 2048
WAIT_NS = 2_000_000_000  # 2 s
ERR_PEER_WAIT = 51


def peer_sum_entry(name: str, rank: int, world: int, dtype: str) -> dict:
    """The exchange kernel for ``rank`` of ``world`` (one warp) as a raw-entry build record; parameters
    ``out`` (the one-element partial, replaced by the total), ``xch`` (this rank's exchange buffer),
    ``peers`` (``world`` u64: every rank's exchange buffer as mapped in this process) and ``err``."""
    if dtype not in ("f32", "i32"):
        raise ValueError("the peer exchange sums f32 or i32")
    if not 1 <= world <= MAX_RANKS or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world} outside 1..{MAX_RANKS} ranks")
    ty = "f32" if dtype == "f32" else "s32"
    L = []

    def a(line):
        L.append(line if line.endswith(":") else "\t" + line)

    a("mov.u32 %r1, %tid.x;")                                   # lane
    for i, nm in enumerate(("out", "xch", "peers", "err")):
        a(f"ld.param.u64 %rd{i + 1}, [p_{nm}];")
        a(f"cvta.to.global.u64 %rd{i + 1}, %rd{i + 1};")
    a("setp.eq.u32 %p1, %r1, 0;")
    # step e = counter + 1 (every lane reads it before lane 0 writes it back)
    a(f"ld.global.u32 %r2, [%rd2+{STEP}];")
    a("add.u32 %r2, %r2, 1;")
    a("bar.warp.sync -1;")
    a(f"@%p1 st.global.u32 [%rd2+{STEP}], %r2;")
    a("ld.global.b32 %r3, [%rd1];")                             # this rank's partial (bits)
    a("and.b32 %r4, %r2, 1;")                                   # parity of the step
    a(f"mul.lo.u32 %r5, %r4, {8 * world};")
    a(f"add.u32 %r5, %r5, {DATA + 8 * rank};")                  # slot [e & 1][rank] in a buffer
    a("mov.b32 %r9, 0;")                                        # partial of rank `lane` (read below)
    a(f"setp.lt.u32 %p2, %r1, {world};")
    a("@!%p2 bra $PUBDONE;")
    # lane r: publish to rank r
    a("mul.wide.u32 %rd5, %r1, 8;")
    a("add.s64 %rd5, %rd5, %rd3;")
    a("ld.global.u64 %rd6, [%rd5];")                            # rank r's buffer, mapped here
    a("cvt.u64.u32 %rd7, %r5;")
    a("add.s64 %rd7, %rd7, %rd6;")
    a("st.global.b32 [%rd7], %r3;")
    a(f"st.release.sys.global.u32 [%rd6+{FLAGS + 4 * rank}], %r2;")
    # lane k: wait for rank k's flag in this rank's buffer, then read its slot
    a("mul.wide.u32 %rd8, %r1, 4;")
    a("add.s64 %rd8, %rd8, %rd2;")
    a("mov.u64 %rd9, %globaltimer;")
    a("$WAIT:")
    a(f"ld.acquire.sys.global.u32 %r6, [%rd8+{FLAGS}];")
    a("setp.ge.u32 %p3, %r6, %r2;")
    a("@%p3 bra $GOT;")
    a("mov.u64 %rd10, %globaltimer;")
    a("sub.s64 %rd10, %rd10, %rd9;")
    a(f"setp.lt.s64 %p4, %rd10, {WAIT_NS};")
    a("@%p4 bra $WAIT;")
    a(f"st.global.u32 [%rd4], {ERR_PEER_WAIT};")
    a("$GOT:")
    a(f"mul.lo.u32 %r7, %r4, {8 * world};")
    a("mad.lo.u32 %r7, %r1, 8, %r7;")
    a("cvt.u64.u32 %rd11, %r7;")
    a("add.s64 %rd11, %rd11, %rd2;")
    a(f"ld.global.b32 %r9, [%rd11+{DATA}];")
    a("$PUBDONE:")
    a("bar.warp.sync -1;")
    # the total in rank order (the same bits on every rank)
    if dtype == "f32":
        a("mov.b32 %f1, 0f00000000;")
    else:
        a("mov.u32 %r10, 0;")
    for k in range(world):
        a(f"shfl.sync.idx.b32 %r8, %r9, {k}, 31, -1;")
        if dtype == "f32":
            a("mov.b32 %f2, %r8;")
            a("add.rn.f32 %f1, %f1, %f2;")
        else:
            a("add.s32 %r10, %r10, %r8;")
    total = "%f1" if dtype == "f32" else "%r10"
    a(f"@%p1 st.global.{ty} [%rd1], {total};")
    entry = [f".visible .entry {name}(", "\t.param .u64 p_out,", "\t.param .u64 p_xch,", "\t.param .u64 p_peers,",
             "\t.param .u64 p_err", ")", ".reqntid 32, 1, 1", "{",
             "\t.reg .b32 %r<11>;", "\t.reg .b64 %rd<12>;", "\t.reg .pred %p<5>;", "\t.reg .f32 %f<3>;"]
    entry += L + ["\tret;", "}"]
    return {"name": name, "kind": "peer_exchange", "params": ["out", "xch", "peers"], "raw_entry": entry,
            "raw_decls": [], "grid": [1, 1, 1], "block": [32, 1, 1], "dyn_smem": 0,
            "align": {"out": 4, "xch": 256, "peers": 8}, "zero_outputs": [],
            "extra": [{"name": "__err", "kind": "errword"}]}
