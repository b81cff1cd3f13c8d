"""Kernel-IR for the five benchmark configurations, authored in Emmy's lowered form.

Emmy (the producer of the IR) is not installed, so the IR for each configuration is built
here, in the statement vocabulary the reference consumes (compile.py:1113-1711) and with the
schedules Emmy's lowering uses for each kernel family (README.md:17-18, 63-64, 101-117):

* ``softmax_ir``   — one block per row, per-thread vector load, WarpShuffle + TreeHalve for the
                     row max and the row sum (config 1).
* ``sum_ir``       — grid-stride Accum over 4-wide vectors, WarpShuffle + TreeHalve per block,
                     one atomic Write of the block partial (config 2; f32 or i32).
* ``fused_ir``     — Tile over 8-element bf16 vectors, fp32 math, one narrowing at the store
                     (config 3).
* ``bmm_ir``       — 64x64 block tiles, cp.async double-buffered K stripes into shared memory,
                     4x4 register micro-tile of Accums (config 4).
* ``attention_ir`` — one warp per query row, QK dot via WarpShuffle, causal Select, online
                     softmax with Accum ``base`` for the running max / sum, PV Accum (config 5).

Every builder returns a :class:`Problem`: the IR graph dict, its ``meta.json`` record
(localrun.py:148-184 format) and the input specification used to make seeded inputs.
"""
from __future__ import annotations

import math
import zlib
from dataclasses import dataclass, field

LOG2E = 1.4426950408889634

# ---- tiny constructors for the wire dicts -------------------------------------------------


def V(name):
    return {"kind": "Var", "name": name}


def Lit(value, dtype="f32"):
    return {"kind": "Literal", "value": value, "dtype": dtype}


def Bin(op, left, right):
    return {"kind": "BinaryExpr", "op": op, "left": left, "right": right}


def Builtin(name):
    return {"kind": "Builtin", "name": name}


def Axis(name, extent):
    return {"kind": "Axis", "name": name, "extent": int(extent)}


def Tile(axes, body):
    return {"kind": "Tile", "axes": axes, "body": body}


def Load(names, buf, index, dtype=None):
    d = {"kind": "Load", "names": list(names), "input": buf, "index": index}
    if dtype is not None:
        d["dtype"] = dtype
    return d


def Write(buf, values, index, dtype, atomic=False):
    return {"kind": "Write", "output": buf, "values": list(values), "index": index,
            "value_dtype": dtype, "atomic": atomic}


def Op(name):
    return {"kind": "ElementwiseImpl", "name": name}


_IDENT = {"add": 0.0, "multiply": 1.0, "maximum": -math.inf, "minimum": math.inf}


def Red(name):
    return {"kind": "ReduceOp", "name": name, "identity": _IDENT[name], "has_identity": True}


def Assign(name, op, args, dtype="f32"):
    return {"kind": "Assign", "name": name, "op": Op(op), "args": list(args), "dtype": dtype}


def Let(name, value, dtype="i32"):
    return {"kind": "Let", "name": name, "value": value, "dtype": dtype}


def Init(name, dtype, identity):
    return {"kind": "Init", "name": name, "dtype": dtype, "identity": identity}


def Accum(name, op, value, dtype="f32", base=None):
    d = {"kind": "Accum", "name": name, "op": Red(op), "value": value, "dtype": dtype}
    if base is not None:
        d["base"] = base
    return d


def Select(name, branches):
    return {"kind": "Select", "name": name,
            "branches": [{"kind": "SelectBranch", "select": s, "value": v} for s, v in branches]}


def Cond(cond, body, else_body=None):
    d = {"kind": "Cond", "cond": cond, "body": body}
    if else_body:
        d["else_body"] = else_body
    return d


def Loop(name, extent, body, unroll=False):
    return {"kind": "Loop", "axis": Axis(name, extent), "body": body, "unroll": unroll}


def StridedLoop(name, extent, start, step, body, end=None):
    d = {"kind": "StridedLoop", "axis": Axis(name, extent), "start": start, "step": step, "body": body}
    if end is not None:
        d["end"] = end
    return d


def WarpShuffle(state, state_b, combine, length=32):
    return {"kind": "WarpShuffle", "state": list(state), "state_b": list(state_b),
            "combine_states": combine, "length": length}


def TreeHalve(bufs, state, state_b, combine, length, tid_var):
    return {"kind": "TreeHalve", "bufs": list(bufs), "state": list(state), "state_b": list(state_b),
            "combine_states": combine, "length": length, "tid_var": tid_var}


def Smem(name, extents, dtype, align=0):
    return {"kind": "Smem", "name": name, "extents": list(extents), "dtype": dtype, "align": align}


def Sync():
    return {"kind": "Sync"}


def CpAsyncCopy(smem, smem_index, lane_index, src, src_index, nbytes=16):
    return {"kind": "CpAsyncCopy", "smem": smem, "smem_index": smem_index, "lane_index": lane_index,
            "src": src, "src_index": src_index, "nbytes": nbytes}


def CpAsyncCommit():
    return {"kind": "CpAsyncCommit"}


def CpAsyncWait(group):
    return {"kind": "CpAsyncWait", "group": group}


# ---- problems -------------------------------------------------------------------------------


@dataclass
class TensorSpec:
    """A kernel argument: shape, dtype, and for inputs the seeded distribution it is drawn from."""

    name: str
    shape: tuple
    dtype: str
    dist: tuple = ("zeros",)      # ("normal", std) | ("uniform", lo, hi) | ("randint", lo, hi_excl) | ("zeros",)
    output: bool = False

    @property
    def seed(self) -> int:
        """``crc32(name) ^ 1234``, the per-tensor seed rule of oracle.py:191."""
        return zlib.crc32(self.name.encode()) ^ 1234

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n


@dataclass
class Problem:
    """One kernel IR plus everything a runner needs: meta record, argument specs, tolerances."""

    name: str
    family: str
    entry: str
    graph: dict
    args: list[TensorSpec]
    grid: int
    block: int
    smem_bytes: int = 0
    zero_outputs: list[str] = field(default_factory=list)
    rtol: float = 1e-5
    atol: float = 1e-6
    params: dict = field(default_factory=dict)

    @property
    def arg_order(self) -> list[str]:
        return [a.name for a in self.args]

    def spec(self, name: str) -> TensorSpec:
        return next(a for a in self.args if a.name == name)

    @property
    def inputs(self) -> list[TensorSpec]:
        return [a for a in self.args if not a.output]

    @property
    def outputs(self) -> list[TensorSpec]:
        return [a for a in self.args if a.output]

    def meta(self) -> dict:
        """The ``meta.json`` document (localrun.py:148-184 format), with ``arg_order`` (compile.py:488)."""
        args = []
        for a in self.args:
            rec = {"name": a.name, "dtype": a.dtype, "shape": list(a.shape)}
            if a.output:
                rec["output"] = True
            args.append(rec)
        return {
            "kernels": [{
                "entry": self.entry, "arg_order": self.arg_order, "args": args,
                "grid": [self.grid, 1, 1], "block": [self.block, 1, 1], "smem_bytes": self.smem_bytes,
                "zero_outputs": list(self.zero_outputs),
            }],
            "rtol": self.rtol, "atol": self.atol,
        }


def _graph(entry: str, args: list[TensorSpec], body: list) -> dict:
    nodes = {}
    for a in args:
        if not a.output:
            nodes[a.name] = {"op": "InputOp", "op_fields": {}, "inputs": [],
                             "outputs": [{"name": a.name, "shape": list(a.shape), "dtype": a.dtype}]}
    outs = [a for a in args if a.output]
    nodes[entry] = {
        "op": "KernelOp",
        "op_fields": {"name": entry, "body": body},
        "inputs": [a.name for a in args if not a.output],
        "outputs": [{"name": a.name, "shape": list(a.shape), "dtype": a.dtype} for a in outs],
    }
    return {"nodes": nodes, "inputs": [a.name for a in args if not a.output],
            "outputs": [a.name for a in outs]}


def _combine(name, other, op, dtype):
    return [Assign(name, op, [name, other], dtype)]


# ---- config 1: row softmax ------------------------------------------------------------------


def softmax_ir(rows: int = 4096, cols: int = 1024, schedule: str | None = None, recip: bool = False,
               threads: int = 128) -> Problem:
    """y = softmax(x, -1) for x f32 [rows, cols].

    ``schedule="warp"`` (the default up to 1024 columns): one warp per row, each lane holding cols/32
    values from cols/128 coalesced 16-byte loads issued back to back, both reductions inside the warp.
    ``schedule="block"``: one block of cols/4 threads per row, WarpShuffle then TreeHalve across warps.
    ``recip`` (warp schedule): y = e * (1 / s) with one division per row instead of one per element.
    ``threads`` (warp schedule): the block size, ``threads // 32`` rows a block.
    """
    if schedule is None:
        schedule = "warp" if cols <= 1024 else "block"
    if schedule == "warp":
        return _softmax_warp_ir(rows, cols, recip, threads)
    if cols % 128 or cols // 4 > 1024:
        raise ValueError("softmax_ir needs cols % 128 == 0 and cols <= 4096")
    t = cols // 4
    w = t // 32
    xs = [f"x{k}" for k in range(4)]
    es = [f"e{k}" for k in range(4)]
    ys = [f"y{k}" for k in range(4)]
    body = [
        Smem("red_m", [w], "f32", 16),
        Smem("red_s", [w], "f32", 16),
        Tile([Axis("row", rows), Axis("t", t)], [
            Let("c", Bin("*", V("t"), 4)),
            Load(xs, "x", [V("row"), V("c")], "f32"),
            Assign("m01", "maximum", ["x0", "x1"]),
            Assign("m23", "maximum", ["x2", "x3"]),
            Assign("m", "maximum", ["m01", "m23"]),
            WarpShuffle(["m"], ["m_o"], _combine("m", "m_o", "maximum", "f32")),
            Cond(Bin("==", V("lane"), 0), [Write("red_m", ["m"], [V("warp")], "f32")]),
            Sync(),
            TreeHalve(["red_m"], ["m"], ["m_b"], _combine("m", "m_b", "maximum", "f32"), w, "t"),
            *[Assign(f"z{k}", "subtract", [xs[k], "m"]) for k in range(4)],
            *[Assign(es[k], "exp", [f"z{k}"]) for k in range(4)],
            Assign("s01", "add", ["e0", "e1"]),
            Assign("s23", "add", ["e2", "e3"]),
            Assign("s", "add", ["s01", "s23"]),
            WarpShuffle(["s"], ["s_o"], _combine("s", "s_o", "add", "f32")),
            Cond(Bin("==", V("lane"), 0), [Write("red_s", ["s"], [V("warp")], "f32")]),
            Sync(),
            TreeHalve(["red_s"], ["s"], ["s_b"], _combine("s", "s_b", "add", "f32"), w, "t"),
            *[Assign(ys[k], "divide", [es[k], "s"]) for k in range(4)],
            Write("y", ys, [V("row"), V("c")], "f32"),
        ]),
    ]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)),
            TensorSpec("y", (rows, cols), "f32", output=True)]
    return Problem(f"softmax_{rows}x{cols}", "softmax", "row_softmax", _graph("row_softmax", args, body),
                   args, grid=rows, block=t, rtol=1e-5, atol=1e-7, params={"rows": rows, "cols": cols})


def _tree(op: str, names: list, prefix: str, final: str) -> list:
    """Pairwise Assigns combining ``names`` (at least two) with ``op``; the last one is named ``final``."""
    stmts, lvl, k = [], list(names), 0
    while len(lvl) > 1:
        nxt = []
        for j in range(0, len(lvl) - 1, 2):
            nm = final if len(lvl) == 2 else f"{prefix}{k}_{j // 2}"
            stmts.append(Assign(nm, op, [lvl[j], lvl[j + 1]]))
            nxt.append(nm)
        if len(lvl) % 2:
            nxt.append(lvl[-1])
        lvl, k = nxt, k + 1
    return stmts


def _softmax_warp_ir(rows: int, cols: int, recip: bool = False, threads: int = 128) -> Problem:
    if cols % 128 or cols > 1024:
        raise ValueError("the warp-per-row softmax needs cols % 128 == 0 and cols <= 1024")
    if threads % 32 or not 32 <= threads <= 1024:
        raise ValueError("the warp-per-row softmax needs a block of 32..1024 threads, a multiple of 32")
    chunks = cols // 128
    xs = [[f"x{c}_{k}" for k in range(4)] for c in range(chunks)]
    flat = [n for ch in xs for n in ch]
    loads = []
    for c in range(chunks):
        loads.append(Let(f"col{c}", Bin("+", Bin("*", V("ln"), 4), 128 * c)))
        loads.append(Load(xs[c], "x", [V("row"), V(f"col{c}")], "f32"))
    es = [f"e_{n}" for n in flat]
    body = [Tile([Axis("row", rows), Axis("ln", 32)], [
        *loads,
        *_tree("maximum", flat, "mx", "m"),
        WarpShuffle(["m"], ["m_o"], _combine("m", "m_o", "maximum", "f32")),
        *[Assign(f"z_{n}", "subtract", [n, "m"]) for n in flat],
        *[Assign(f"e_{n}", "exp", [f"z_{n}"]) for n in flat],
        *_tree("add", es, "sm", "s"),
        WarpShuffle(["s"], ["s_o"], _combine("s", "s_o", "add", "f32")),
        *([Assign("rs", "divide", [Lit(1.0), "s"]), *[Assign(f"y_{n}", "multiply", [f"e_{n}", "rs"]) for n in flat]]
          if recip else [Assign(f"y_{n}", "divide", [f"e_{n}", "s"]) for n in flat]),
        *[Write("y", [f"y_{n}" for n in xs[c]], [V("row"), V(f"col{c}")], "f32") for c in range(chunks)],
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)),
            TensorSpec("y", (rows, cols), "f32", output=True)]
    return Problem(f"softmax_{rows}x{cols}", "softmax", "row_softmax", _graph("row_softmax", args, body),
                   args, grid=(rows * 32 + threads - 1) // threads, block=threads, rtol=1e-5, atol=1e-7,
                   params={"rows": rows, "cols": cols, "schedule": "warp", **({"recip": True} if recip else {}),
                           **({"threads": threads} if threads != 128 else {})})


# ---- config 2: full-array sum ---------------------------------------------------------------


def sum_ir(n: int = 1 << 28, dtype: str = "f32", blocks: int = 592, threads: int = 512) -> Problem:
    """out[0] = sum(x) for x [n] (f32 or i32): grid-stride vector Accum, warp + block tree, one
    atomic add per block into a zeroed scalar."""
    if dtype not in ("f32", "i32"):
        raise ValueError("sum_ir dtype must be f32 or i32")
    if threads % 32 or threads > 1024:
        raise ValueError("threads must be a multiple of 32, at most 1024")
    total = blocks * threads
    nv = n // 4
    w = threads // 32
    xs = [f"x{k}" for k in range(4)]
    body = [
        Smem("red", [w], dtype, 16),
        Tile([Axis("g", total)], [
            Let("t", Builtin("threadIdx.x")),
            StridedLoop("v", nv, V("g"), total, [
                Let("e", Bin("*", V("v"), 4)),
                Load(xs, "x", [V("e")], dtype),
                *[Accum("acc", "add", xs[k], dtype) for k in range(4)],
            ], end=nv),
        ]),
    ]
    tile_body = body[1]["body"]
    if n % 4:
        tile_body.append(StridedLoop("r", n, Bin("+", V("g"), 4 * nv), total, [
            Load(["xt"], "x", [V("r")], dtype),
            Accum("acc", "add", "xt", dtype),
        ], end=n))
    tile_body.extend([
        WarpShuffle(["acc"], ["acc_o"], _combine("acc", "acc_o", "add", dtype)),
        Cond(Bin("==", V("lane"), 0), [Write("red", ["acc"], [V("warp")], dtype)]),
        Sync(),
        TreeHalve(["red"], ["acc"], ["acc_b"], _combine("acc", "acc_b", "add", dtype), w, "t"),
        Cond(Bin("==", V("t"), 0), [Write("out", ["acc"], [0], dtype, atomic=True)]),
    ])
    dist = ("uniform", -1.0, 1.0) if dtype == "f32" else ("randint", -1000, 1001)
    args = [TensorSpec("x", (n,), dtype, dist), TensorSpec("out", (1,), dtype, output=True)]
    return Problem(f"sum_{dtype}_{n}", "sum", f"array_sum_{dtype}", _graph(f"array_sum_{dtype}", args, body),
                   args, grid=blocks, block=threads, zero_outputs=["out"],
                   rtol=1e-5 if dtype == "f32" else 0.0, atol=0.0,
                   params={"n": n, "dtype": dtype, "blocks": blocks, "threads": threads})


# ---- config 3: fused broadcast elementwise -------------------------------------------------


def fused_ir(rows: int = 8192, cols: int = 8192, out_dtype: str = "bf16") -> Problem:
    """y = relu(a*b + c) * exp(d): a, b, d bf16 [rows, cols], c f32 [cols] broadcast over rows."""
    if cols % 8:
        raise ValueError("fused_ir needs cols % 8 == 0")
    threads = 256
    cells = rows * (cols // 8)
    ks = range(8)
    body = [Tile([Axis("i", rows), Axis("j8", cols // 8)], [
        Let("j", Bin("*", V("j8"), 8)),
        Let("j4", Bin("+", V("j"), 4)),
        Load([f"a{k}" for k in ks], "a", [V("i"), V("j")], "bf16"),
        Load([f"b{k}" for k in ks], "b", [V("i"), V("j")], "bf16"),
        Load([f"d{k}" for k in ks], "d", [V("i"), V("j")], "bf16"),
        Load([f"c{k}" for k in range(4)], "c", [V("j")], "f32"),
        Load([f"c{k}" for k in range(4, 8)], "c", [V("j4")], "f32"),
        *[Assign(f"p{k}", "multiply", [f"a{k}", f"b{k}"]) for k in ks],
        *[Assign(f"q{k}", "add", [f"p{k}", f"c{k}"]) for k in ks],
        *[Assign(f"r{k}", "relu", [f"q{k}"]) for k in ks],
        *[Assign(f"x{k}", "exp", [f"d{k}"]) for k in ks],
        *[Assign(f"y{k}", "multiply", [f"r{k}", f"x{k}"], out_dtype) for k in ks],
        Write("y", [f"y{k}" for k in ks], [V("i"), V("j")], out_dtype),
    ])]
    args = [TensorSpec("a", (rows, cols), "bf16", ("normal", 1.0)),
            TensorSpec("b", (rows, cols), "bf16", ("normal", 1.0)),
            TensorSpec("c", (cols,), "f32", ("normal", 0.1)),
            TensorSpec("d", (rows, cols), "bf16", ("normal", 1.0)),
            TensorSpec("y", (rows, cols), out_dtype, output=True)]
    grid = (cells + threads - 1) // threads
    return Problem(f"fused_{rows}x{cols}", "fused", "fused_relu_exp", _graph("fused_relu_exp", args, body),
                   args, grid=grid, block=threads, rtol=1e-5, atol=1e-6,
                   params={"rows": rows, "cols": cols, "out_dtype": out_dtype})


# ---- config 4: batched matmul ---------------------------------------------------------------


def bmm_ir(batch: int = 16, m: int = 4096, n: int = 4096, k: int = 4096) -> Problem:
    """C[b] = A[b] @ B[b], bf16 inputs, f32 accumulation and output.

    64x64 output tile per 256-thread block, K in 32-wide stripes double-buffered in shared
    memory by cp.async (one 16-byte copy per thread per operand per stripe), each thread a 4x4
    register micro-tile.
    """
    if m % 64 or n % 64 or k % 32:
        raise ValueError("bmm_ir needs m, n % 64 == 0 and k % 32 == 0")
    bm = bn = 64
    bk = 32
    nk = k // bk
    R = range(4)
    inner = [
        *[Load([f"a{i}"], "sA", [V("s"), Bin("+", V("r4"), i), V("kk")], "bf16") for i in R],
        Load([f"b{j}" for j in R], "sB", [V("s"), V("kk"), V("c4")], "bf16"),
        *[Assign(f"p{i}{j}", "multiply", [f"a{i}", f"b{j}"]) for i in R for j in R],
        *[Accum(f"c{i}{j}", "add", f"p{i}{j}") for i in R for j in R],
    ]
    kloop = StridedLoop("kb", nk, 0, 1, [
        Let("s", Bin("%", V("kb"), 2)),
        Let("s1", Bin("-", 1, V("s"))),
        Let("kn", Bin("*", Bin("+", V("kb"), 1), bk)),
        Cond(Bin("<", Bin("+", V("kb"), 1), nk), [
            CpAsyncCopy("sA", [V("s1"), 0, 0], [V("ar"), V("ac")], "A",
                        [V("b"), V("arow"), Bin("+", V("kn"), V("ac"))]),
            CpAsyncCopy("sB", [V("s1"), 0, 0], [V("br"), V("bc")], "B",
                        [V("b"), Bin("+", V("kn"), V("br")), V("bcol")]),
        ]),
        CpAsyncCommit(),
        CpAsyncWait(1),
        Sync(),
        Loop("kk", bk, inner, unroll=True),
        Sync(),
    ], end=nk)
    body = [
        Smem("sA", [2, bm, bk], "bf16", 16),
        Smem("sB", [2, bk, bn], "bf16", 16),
        Tile([Axis("b", batch), Axis("tm", m // bm), Axis("tn", n // bn), Axis("t", 256)], [
            Let("ar", Bin("/", V("t"), 4)),
            Let("ac", Bin("*", Bin("%", V("t"), 4), 8)),
            Let("br", Bin("/", V("t"), 8)),
            Let("bc", Bin("*", Bin("%", V("t"), 8), 8)),
            Let("r4", Bin("*", Bin("/", V("t"), 16), 4)),
            Let("c4", Bin("*", Bin("%", V("t"), 16), 4)),
            Let("arow", Bin("+", Bin("*", V("tm"), bm), V("ar"))),
            Let("bcol", Bin("+", Bin("*", V("tn"), bn), V("bc"))),
            Let("orow", Bin("+", Bin("*", V("tm"), bm), V("r4"))),
            Let("ocol", Bin("+", Bin("*", V("tn"), bn), V("c4"))),
            *[Init(f"c{i}{j}", "f32", 0.0) for i in R for j in R],
            CpAsyncCopy("sA", [0, 0, 0], [V("ar"), V("ac")], "A", [V("b"), V("arow"), V("ac")]),
            CpAsyncCopy("sB", [0, 0, 0], [V("br"), V("bc")], "B", [V("b"), V("br"), V("bcol")]),
            CpAsyncCommit(),
            kloop,
            *[Write("C", [f"c{i}{j}" for j in R], [V("b"), Bin("+", V("orow"), i), V("ocol")], "f32")
              for i in R],
        ]),
    ]
    args = [TensorSpec("A", (batch, m, k), "bf16", ("normal", 0.02)),
            TensorSpec("B", (batch, k, n), "bf16", ("normal", 0.02)),
            TensorSpec("C", (batch, m, n), "f32", output=True)]
    grid = batch * (m // bm) * (n // bn)
    return Problem(f"bmm_{batch}x{m}x{n}x{k}", "bmm", "bmm_bf16", _graph("bmm_bf16", args, body), args,
                   grid=grid, block=256, rtol=1e-4, atol=1e-6,
                   params={"batch": batch, "m": m, "n": n, "k": k})


def bmm_naive_ir(batch: int, m: int, n: int, k: int, threads: int = 256) -> Problem:
    """The same batched matmul in its unscheduled form: a thread per output element, a rolled Loop
    over k accumulating bf16 products in f32 (what a lowering emits before any tiling)."""
    body = [Tile([Axis("b", batch), Axis("i", m), Axis("j", n)], [
        Loop("kk", k, [
            Load(["a"], "A", [V("b"), V("i"), V("kk")], "bf16"),
            Load(["w"], "B", [V("b"), V("kk"), V("j")], "bf16"),
            Assign("p", "multiply", ["a", "w"]),
            Accum("acc", "add", "p"),
        ]),
        Write("C", ["acc"], [V("b"), V("i"), V("j")], "f32"),
    ])]
    args = [TensorSpec("A", (batch, m, k), "bf16", ("normal", 0.02)),
            TensorSpec("B", (batch, k, n), "bf16", ("normal", 0.02)),
            TensorSpec("C", (batch, m, n), "f32", output=True)]
    return Problem(f"bmm_naive_{batch}x{m}x{n}x{k}", "bmm", "bmm_naive", _graph("bmm_naive", args, body), args,
                   grid=(batch * m * n + threads - 1) // threads, block=threads, rtol=1e-4, atol=1e-6,
                   params={"batch": batch, "m": m, "n": n, "k": k})


# ---- config 5: causal attention -------------------------------------------------------------


def attention_ir(batch: int = 8, heads: int = 32, seq: int = 4096, dim: int = 128,
                 causal: bool = True, scale: float | None = None, mask: bool = False) -> Problem:
    """O = softmax(Q K^T / sqrt(D) + causal mask) V, bf16 in and out, f32 math.

    One warp per query row; each lane holds D/32 contiguous dims.  Scores come from a lane dot
    plus a WarpShuffle sum, the causal mask is a Select, and the online softmax keeps the running
    max / sum / output as Accums whose ``base`` is the rescaled previous value.

    ``mask`` adds an explicit boolean mask M [seq, seq] (u8; nonzero = the key takes part, torch's
    ``attn_mask`` convention): a masked score is -inf.  Since any key may then be masked, the
    exponents use a safe maximum (0 while every key so far is masked), so a masked first key cannot
    turn the running sum into NaN; a row with every key masked ends as 0 / 0 = NaN, as in torch.
    """
    if dim % 32 or dim // 32 not in (1, 2, 4, 8):
        raise ValueError("attention_ir needs dim in {32, 64, 128, 256}")
    per = dim // 32
    P = range(per)
    scale = 1.0 / math.sqrt(dim) if scale is None else float(scale)
    qs = [f"q{i}" for i in P]
    ks = [f"k{i}" for i in P]
    vs = [f"v{i}" for i in P]
    os_ = [f"o{i}" for i in P]
    # this lane's partial dot product, summed pairwise over its dims; the last sum is "dp"
    if per == 1:
        dot = [Assign("dp", "multiply", [qs[0], ks[0]])]
    else:
        dot = [Assign(f"pp{i}", "multiply", [qs[i], ks[i]]) for i in P]
        terms = [f"pp{i}" for i in P]
        lvl = 0
        while len(terms) > 1:
            nxt = []
            for j in range(0, len(terms), 2):
                nm = "dp" if len(terms) == 2 else f"ds{lvl}_{j // 2}"
                dot.append(Assign(nm, "add", [terms[j], terms[j + 1]]))
                nxt.append(nm)
            terms, lvl = nxt, lvl + 1
    sel = [(Bin(">", V("kv"), V("qi")), Lit(-math.inf))] if causal else []
    if mask:
        sel.append((Bin("==", V("mk"), 0), Lit(-math.inf)))
    safe = "mu" if mask else "mn"
    body_k = [
        Load(ks, "K", [V("b"), V("h"), V("kv"), V("d0")], "bf16"),
        *([Load(["mk"], "M", [V("qi"), V("kv")], "u8")] if mask else []),
        *dot,
        WarpShuffle(["dp"], ["dp_o"], _combine("dp", "dp_o", "add", "f32")),
        Assign("sc", "multiply", ["dp", Lit(scale)]),
        Select("sm", [*sel, (None, "sc")]),
        Assign("mn", "maximum", ["m", "sm"]),
        *([Assign("allm", "equal", ["mn", Lit(-math.inf)], "bool"),
           Select("mu", [(V("allm"), Lit(0.0)), (None, "mn")])] if mask else []),
        Assign("dm", "subtract", ["m", safe]),
        Assign("alpha", "exp", ["dm"]),
        Assign("ds", "subtract", ["sm", safe]),
        Assign("pe", "exp", ["ds"]),
        Assign("ls", "multiply", ["l", "alpha"]),
        Accum("l", "add", "pe", base="ls"),
        Load(vs, "V", [V("b"), V("h"), V("kv"), V("d0")], "bf16"),
        *[Assign(f"os{i}", "multiply", [os_[i], "alpha"]) for i in P],
        *[Assign(f"pv{i}", "multiply", ["pe", vs[i]]) for i in P],
        *[Accum(os_[i], "add", f"pv{i}", base=f"os{i}") for i in P],
        Accum("m", "maximum", "sm"),
    ]
    body = [Tile([Axis("b", batch), Axis("h", heads), Axis("qi", seq), Axis("ln", 32)], [
        Let("d0", Bin("*", V("ln"), per)),
        Load(qs, "Q", [V("b"), V("h"), V("qi"), V("d0")], "bf16"),
        Init("m", "f32", -math.inf),
        Init("l", "f32", 0.0),
        *[Init(o, "f32", 0.0) for o in os_],
        StridedLoop("kv", seq, 0, 1, body_k, end=seq),
        *[Assign(f"y{i}", "divide", [os_[i], "l"], "bf16") for i in P],
        Write("O", [f"y{i}" for i in P], [V("b"), V("h"), V("qi"), V("d0")], "bf16"),
    ])]
    shape = (batch, heads, seq, dim)
    args = [TensorSpec("Q", shape, "bf16", ("normal", 1.0)),
            TensorSpec("K", shape, "bf16", ("normal", 1.0)),
            TensorSpec("V", shape, "bf16", ("normal", 1.0))]
    if mask:
        args.append(TensorSpec("M", (seq, seq), "u8", ("randint", 0, 2)))
    args.append(TensorSpec("O", shape, "bf16", output=True))
    threads = 128
    grid = batch * heads * seq * 32 // threads
    return Problem(f"attn_{batch}x{heads}x{seq}x{dim}", "attention", "attention_causal" if causal else "attention",
                   _graph("attention_causal" if causal else "attention", args, body), args,
                   grid=grid, block=threads, rtol=1e-4, atol=1e-6,
                   params={"batch": batch, "heads": heads, "seq": seq, "dim": dim, "causal": causal,
                           "scale": scale, **({"mask": True} if mask else {})})


#: The five BASELINE configurations at full size.
FULL = {          # keyword arguments pass through to the builder (e.g. softmax_ir's recip)
    # one division per row (y = e * (1/s)): the lowering the softmax benchmark uses
    "c1": lambda **kw: softmax_ir(4096, 1024, **{"recip": True, **kw}),
    "c2": lambda **kw: sum_ir(1 << 28, "f32", **kw),
    "c2i": lambda **kw: sum_ir(1 << 28, "i32", **kw),
    "c3": lambda **kw: fused_ir(8192, 8192, **kw),
    "c4": lambda **kw: bmm_ir(16, 4096, 4096, 4096, **kw),
    "c5": lambda **kw: attention_ir(8, 32, 4096, 128, **kw),
}

#: Small instances of the same kernels, sized so the CPU oracle finishes in seconds.
SMALL = {
    "c1": lambda: softmax_ir(64, 1024),
    "c1b": lambda: softmax_ir(33, 256, schedule="block"),
    "c1w": lambda: softmax_ir(37, 384),
    "c2": lambda: sum_ir(1 << 16, "f32", blocks=8, threads=256),
    "c2odd": lambda: sum_ir(997, "f32", blocks=2, threads=128),
    "c2i": lambda: sum_ir(1 << 16, "i32", blocks=8, threads=256),
    "c3": lambda: fused_ir(64, 512),
    "c4": lambda: bmm_ir(2, 128, 128, 96),
    "c4tc": lambda: bmm_ir(2, 256, 512, 256),
    "c5": lambda: attention_ir(1, 2, 64, 128),
    "c5tc": lambda: attention_ir(1, 2, 512, 128),
    "c5tcnc": lambda: attention_ir(1, 1, 256, 128, causal=False),
    "c5nc": lambda: attention_ir(1, 2, 32, 64, causal=False),
}
