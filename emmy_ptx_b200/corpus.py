"""A coverage corpus of small Emmy-IR kernels in the categories of the reference's case files.

The reference grows its tests from torch expressions lowered by Emmy (cases.txt, cases_matmul.txt,
cases_fused.txt, cases_attention.txt: pointwise, reductions, normalisations, odd shapes, integer /
half / double dtypes, masks).  Emmy is not installed, so these kernels are authored directly in the
lowered IR vocabulary.  With the benchmark configurations (:mod:`.irgen`) they exercise every
statement the reference lowers:

* Tile, Let, Init, Accum, Assign (integer, float, predicate results and the math library);
* Load / Write in f32, f16, bf16, f64, i32 and u8 (a predicate stored as a byte), atomic adds;
* Select with several branches (first true branch wins), Cond with an else branch;
* Loop (rolled and unrolled), StridedLoop (block-strided and with a thread-dependent end);
* WarpShuffle as a reduction over one or two states and as an inclusive prefix scan, WarpBroadcast;
* Smem + Sync + TreeHalve block reductions;
* ZeroPrologue in a kernel that runs before the one accumulating into the zeroed buffer, and graphs
  of several kernels chained through an intermediate buffer.

Each builder returns a :class:`~.irgen.Problem` whose ``params["expr"]`` names the source expression
(the float64 torch form lives with the test oracle).
"""
from __future__ import annotations

import math

from .irgen import (Problem, TensorSpec, Tile, Axis, Load, Write, Assign, Let, Init, Accum, Select, Cond, Loop,
                    StridedLoop, WarpShuffle, TreeHalve, Smem, Sync, Lit, V, Bin, _graph)


def _problem(expr, name, entry, args, body, grid, block, rtol=1e-5, atol=1e-6, **params):
    return Problem(name, "corpus", entry, _graph(entry, args, body), args, grid=grid, block=block, rtol=rtol,
                   atol=atol, params={"expr": expr, **params})


def _block_reduce(states, bufs, ops, nwarps):
    """WarpShuffle over ``states``; lane 0 of each warp stores them to shared memory; Sync; a
    TreeHalve over the warps leaves the block's result in every thread."""
    others = [f"{s}_o" for s in states]
    second = [f"{s}_b" for s in states]
    return [
        WarpShuffle(states, others, [Assign(s, ops[s], [s, o]) for s, o in zip(states, others)]),
        Cond(Bin("==", V("lane"), 0), [Write(bf, [s], [V("warp")], "f32") for s, bf in zip(states, bufs)]),
        Sync(),
        TreeHalve(bufs, states, second, [Assign(s, ops[s], [s, b]) for s, b in zip(states, second)], nwarps, "t"),
    ]


# ---- normalisations: a block per row, block-strided loops over the columns ------------------------


def rmsnorm(rows=33, cols=512, eps=1e-6, threads=128):
    """y = x / sqrt(mean(x^2) + eps) * w."""
    nw = threads // 32
    body = [
        Smem("red", [nw], "f32", 16),
        Tile([Axis("row", rows), Axis("t", threads)], [
            StridedLoop("c", cols, V("t"), threads, [
                Load(["x"], "x", [V("row"), V("c")], "f32"),
                Assign("sq", "multiply", ["x", "x"]),
                Accum("ss", "add", "sq"),
            ], end=cols),
            *_block_reduce(["ss"], ["red"], {"ss": "add"}, nw),
            Assign("ms", "multiply", ["ss", Lit(1.0 / cols)]),
            Assign("d", "add", ["ms", Lit(eps)]),
            Assign("rs", "sqrt", ["d"]),
            StridedLoop("c2", cols, V("t"), threads, [
                Load(["x2"], "x", [V("row"), V("c2")], "f32"),
                Load(["w"], "w", [V("c2")], "f32"),
                Assign("xn", "divide", ["x2", "rs"]),
                Assign("y", "multiply", ["xn", "w"]),
                Write("y", ["y"], [V("row"), V("c2")], "f32"),
            ], end=cols),
        ]),
    ]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("w", (cols,), "f32", ("normal", 1.0)),
            TensorSpec("y", (rows, cols), "f32", output=True)]
    return _problem("rmsnorm", f"rmsnorm_{rows}x{cols}", "rms_norm", args, body, rows, threads, eps=eps)


def layernorm(rows=16, cols=256, eps=1e-5, threads=64):
    """y = (x - mean) / sqrt(var + eps) * g + b, mean and E[x^2] reduced together (two states)."""
    nw = threads // 32
    body = [
        Smem("red_s", [nw], "f32", 16),
        Smem("red_q", [nw], "f32", 16),
        Tile([Axis("row", rows), Axis("t", threads)], [
            StridedLoop("c", cols, V("t"), threads, [
                Load(["x"], "x", [V("row"), V("c")], "f32"),
                Accum("s", "add", "x"),
                Assign("xx", "multiply", ["x", "x"]),
                Accum("q", "add", "xx"),
            ], end=cols),
            *_block_reduce(["s", "q"], ["red_s", "red_q"], {"s": "add", "q": "add"}, nw),
            Assign("mean", "multiply", ["s", Lit(1.0 / cols)]),
            Assign("ex2_", "multiply", ["q", Lit(1.0 / cols)]),
            Assign("m2", "multiply", ["mean", "mean"]),
            Assign("var", "subtract", ["ex2_", "m2"]),
            Assign("ve", "add", ["var", Lit(eps)]),
            Assign("sd", "sqrt", ["ve"]),
            StridedLoop("c2", cols, V("t"), threads, [
                Load(["x2"], "x", [V("row"), V("c2")], "f32"),
                Load(["g"], "g", [V("c2")], "f32"),
                Load(["b"], "b", [V("c2")], "f32"),
                Assign("xc", "subtract", ["x2", "mean"]),
                Assign("xn", "divide", ["xc", "sd"]),
                Assign("xg", "multiply", ["xn", "g"]),
                Assign("y", "add", ["xg", "b"]),
                Write("y", ["y"], [V("row"), V("c2")], "f32"),
            ], end=cols),
        ]),
    ]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("g", (cols,), "f32", ("normal", 1.0)),
            TensorSpec("b", (cols,), "f32", ("normal", 1.0)), TensorSpec("y", (rows, cols), "f32", output=True)]
    return _problem("layernorm", f"layernorm_{rows}x{cols}", "layer_norm", args, body, rows, threads, eps=eps)


def log_softmax(rows=8, cols=512, threads=128):
    """y = x - max - log(sum(exp(x - max))), three passes over the row."""
    nw = threads // 32
    body = [
        Smem("red_m", [nw], "f32", 16),
        Smem("red_s", [nw], "f32", 16),
        Tile([Axis("row", rows), Axis("t", threads)], [
            StridedLoop("c", cols, V("t"), threads, [
                Load(["x"], "x", [V("row"), V("c")], "f32"),
                Accum("m", "maximum", "x"),
            ], end=cols),
            *_block_reduce(["m"], ["red_m"], {"m": "maximum"}, nw),
            StridedLoop("c1", cols, V("t"), threads, [
                Load(["x1"], "x", [V("row"), V("c1")], "f32"),
                Assign("z", "subtract", ["x1", "m"]),
                Assign("e", "exp", ["z"]),
                Accum("s", "add", "e"),
            ], end=cols),
            *_block_reduce(["s"], ["red_s"], {"s": "add"}, nw),
            Assign("ls", "log", ["s"]),
            StridedLoop("c2", cols, V("t"), threads, [
                Load(["x2"], "x", [V("row"), V("c2")], "f32"),
                Assign("z2", "subtract", ["x2", "m"]),
                Assign("y", "subtract", ["z2", "ls"]),
                Write("y", ["y"], [V("row"), V("c2")], "f32"),
            ], end=cols),
        ]),
    ]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("y", (rows, cols), "f32", output=True)]
    return _problem("logsoftmax", f"logsoftmax_{rows}x{cols}", "log_softmax", args, body, rows, threads)


# ---- reductions along other axes, scans, data-dependent loop bounds -------------------------------


def col_sum(rows=100, cols=96):
    """out[c] = sum over r of x[r, c]: a thread per column walks down the rows in a rolled Loop."""
    body = [Tile([Axis("c", cols)], [
        Loop("r", rows, [Load(["x"], "x", [V("r"), V("c")], "f32"), Accum("s", "add", "x")]),
        Write("out", ["s"], [V("c")], "f32"),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("out", (cols,), "f32", output=True)]
    return _problem("colsum", f"colsum_{rows}x{cols}", "col_sum", args, body, (cols + 63) // 64, 64)


def mid_sum(a=2, b=64, c=32):
    """out[i, k] = sum over j of x[i, j, k]: the middle axis, reduced in a fully unrolled Loop."""
    body = [Tile([Axis("i", a), Axis("k", c)], [
        Loop("j", b, [Load(["x"], "x", [V("i"), V("j"), V("k")], "f32"), Accum("s", "add", "x")], unroll=True),
        Write("out", ["s"], [V("i"), V("k")], "f32"),
    ])]
    args = [TensorSpec("x", (a, b, c), "f32", ("normal", 1.0)), TensorSpec("out", (a, c), "f32", output=True)]
    return _problem("midsum", f"midsum_{a}x{b}x{c}", "mid_sum", args, body, (a * c + 63) // 64, 64)


def prefix_sum_tri(n=96):
    """y[i] = sum over j <= i of x[j]: each thread's loop ends at its own index plus one."""
    body = [Tile([Axis("i", n)], [
        StridedLoop("j", n, 0, 1, [Load(["x"], "x", [V("j")], "f32"), Accum("s", "add", "x")],
                    end=Bin("+", V("i"), 1)),
        Write("y", ["s"], [V("i")], "f32"),
    ])]
    args = [TensorSpec("x", (n,), "f32", ("normal", 1.0)), TensorSpec("y", (n,), "f32", output=True)]
    return _problem("tri", f"tri_{n}", "tri_sum", args, body, (n + 31) // 32, 32)


def _scan(state):
    return {"kind": "WarpShuffle", "state": [state], "state_b": [f"{state}_o"],
            "combine_states": [Assign(state, "add", [state, f"{state}_o"])], "length": 32, "prefix": True}


def cumsum_rows(rows=4, cols=64):
    """y = cumsum(x, -1) for rows of 64: a warp per row, an inclusive prefix WarpShuffle over each
    32-column half, the first half's total (lane 31) carried into the second by a WarpBroadcast."""
    if cols != 64:
        raise ValueError("cumsum_rows is written for rows of 64")
    body = [Tile([Axis("row", rows), Axis("ln", 32)], [
        Load(["a"], "x", [V("row"), V("ln")], "f32"),
        Let("c1", Bin("+", V("ln"), 32)),
        Load(["b"], "x", [V("row"), V("c1")], "f32"),
        _scan("a"),
        _scan("b"),
        Assign("tot", "copy", ["a"]),
        {"kind": "WarpBroadcast", "state": ["tot"], "length": 32},
        Assign("b2", "add", ["b", "tot"]),
        Write("y", ["a"], [V("row"), V("ln")], "f32"),
        Write("y", ["b2"], [V("row"), V("c1")], "f32"),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("y", (rows, cols), "f32", output=True)]
    return _problem("cumsum", f"cumsum_{rows}x{cols}", "cumsum_rows", args, body, rows, 32)


def cumsum_1d(n=128):
    """y = cumsum(x) for one row of ``n`` (a multiple of 32): one warp walks the row in 32-element
    chunks in a rolled Loop; each chunk is an inclusive prefix WarpShuffle plus the carry of the
    chunks before it, and the chunk's total (lane 31, by WarpBroadcast) is added into the carry by an
    Accum.  This is the 1-D scan the reference lists as wrong past the first chunk."""
    if n % 32:
        raise ValueError("cumsum_1d needs n % 32 == 0")
    body = [Tile([Axis("row", 1), Axis("ln", 32)], [
        Loop("ch", n // 32, [
            Let("col", Bin("+", Bin("*", V("ch"), 32), V("ln"))),
            Load(["v"], "x", [V("row"), V("col")], "f32"),
            _scan("v"),
            Assign("y", "add", ["v", "carry"]),
            Write("y", ["y"], [V("row"), V("col")], "f32"),
            Assign("tot", "copy", ["v"]),
            {"kind": "WarpBroadcast", "state": ["tot"], "length": 32},
            Accum("carry", "add", "tot"),
        ]),
    ])]
    args = [TensorSpec("x", (1, n), "f32", ("normal", 1.0)), TensorSpec("y", (1, n), "f32", output=True)]
    return _problem("cumsum", f"cumsum1d_{n}", "cumsum_1d", args, body, 1, 32)


# ---- dtypes, predicates, branches -------------------------------------------------------------------


def int_ops(n=1000):
    """Integer elementwise work with a two-way and two three-way Selects, one of them with overlapping
    predicates (x > 10 and x > 0 are both true above 10: the first true branch wins); division and
    remainder truncate toward zero as in C."""
    body = [Tile([Axis("i", n)], [
        Load(["x"], "x", [V("i")], "i32"),
        Load(["y"], "y", [V("i")], "i32"),
        Assign("a", "bitwise_and", ["x", "y"], "i32"),
        Assign("o", "bitwise_or", ["x", "y"], "i32"),
        Assign("o3", "subtract", ["o", 3], "i32"),
        Assign("gt", "greater", ["x", 4], "bool"),
        Select("z", [(V("gt"), "a"), (None, "o3")]),
        Select("sg", [(Bin("<", V("x"), 0), -1), (Bin("==", V("x"), 0), 0), (None, 1)]),
        Select("bd", [(Bin(">", V("x"), 10), 2), (Bin(">", V("x"), 0), 1), (None, 0)]),
        Assign("q", "divide", ["x", 3], "i32"),
        Assign("r", "modulo", ["x", 3], "i32"),
        Assign("sh", "left_shift", ["y", 2], "i32"),
        Assign("mx", "maximum", ["q", "r"], "i32"),
        Assign("w", "add", ["mx", "sh"], "i32"),
        Write("z", ["z"], [V("i")], "i32"),
        Write("s", ["sg"], [V("i")], "i32"),
        Write("w", ["w"], [V("i")], "i32"),
        Write("bd", ["bd"], [V("i")], "i32"),
    ])]
    args = [TensorSpec("x", (n,), "i32", ("randint", -20, 21)), TensorSpec("y", (n,), "i32", ("randint", 0, 9)),
            TensorSpec("z", (n,), "i32", output=True), TensorSpec("s", (n,), "i32", output=True),
            TensorSpec("w", (n,), "i32", output=True), TensorSpec("bd", (n,), "i32", output=True)]
    return _problem("intops", f"intops_{n}", "int_ops", args, body, (n + 127) // 128, 128, rtol=0.0, atol=0.0)


def half_gelu(rows=16, cols=256):
    """f16 in and out: exact (erf) and tanh GELU over 8-wide (16-byte) vectors."""
    ks = range(8)
    body = [Tile([Axis("i", rows), Axis("j8", cols // 8)], [
        Let("j", Bin("*", V("j8"), 8)),
        Load([f"x{k}" for k in ks], "x", [V("i"), V("j")], "f16"),
        *[Assign(f"g{k}", "gelu", [f"x{k}"], "f16") for k in ks],
        *[Assign(f"h{k}", "gelu_tanh", [f"x{k}"], "f16") for k in ks],
        Write("y", [f"g{k}" for k in ks], [V("i"), V("j")], "f16"),
        Write("yt", [f"h{k}" for k in ks], [V("i"), V("j")], "f16"),
    ])]
    args = [TensorSpec("x", (rows, cols), "f16", ("normal", 1.0)), TensorSpec("y", (rows, cols), "f16", output=True),
            TensorSpec("yt", (rows, cols), "f16", output=True)]
    return _problem("gelu_f16", f"gelu_f16_{rows}x{cols}", "gelu_f16", args, body, rows * cols // 8 // 64, 64)


def mask_where(n=777):
    """A predicate stored as a u8 mask, and where(mask, x, 0)."""
    body = [Tile([Axis("i", n)], [
        Load(["x"], "x", [V("i")], "f32"),
        Assign("m", "greater", ["x", Lit(0.0)], "bool"),
        Assign("y", "where", ["m", "x", Lit(0.0)], "f32"),
        Write("mask", ["m"], [V("i")], "u8"),
        Write("y", ["y"], [V("i")], "f32"),
    ])]
    args = [TensorSpec("x", (n,), "f32", ("normal", 1.0)), TensorSpec("mask", (n,), "u8", output=True),
            TensorSpec("y", (n,), "f32", output=True)]
    return _problem("mask", f"mask_{n}", "mask_where", args, body, (n + 127) // 128, 128)


def f64_affine(rows=2, cols=32):
    """f64 buffers: narrowed to f32 in registers, widened at the store."""
    body = [Tile([Axis("i", rows), Axis("j", cols)], [
        Load(["x"], "x", [V("i"), V("j")], "f64"),
        Assign("a", "multiply", ["x", Lit(2.5)]),
        Assign("y", "add", ["a", Lit(1.0)], "f64"),
        Write("y", ["y"], [V("i"), V("j")], "f64"),
    ])]
    args = [TensorSpec("x", (rows, cols), "f64", ("normal", 1.0)), TensorSpec("y", (rows, cols), "f64", output=True)]
    return _problem("f64", f"f64_{rows}x{cols}", "f64_affine", args, body, 1, rows * cols)


def cond_else(n=300):
    """y = sqrt(x) where x >= 0, else -x/2: a Cond whose two sides each write."""
    body = [Tile([Axis("i", n)], [
        Load(["x"], "x", [V("i")], "f32"),
        Cond(Bin(">=", V("x"), Lit(0.0)),
             [Assign("r", "sqrt", ["x"]), Write("y", ["r"], [V("i")], "f32")],
             [Assign("h", "multiply", ["x", Lit(-0.5)]), Write("y", ["h"], [V("i")], "f32")]),
    ])]
    args = [TensorSpec("x", (n,), "f32", ("normal", 1.0)), TensorSpec("y", (n,), "f32", output=True)]
    return _problem("cond", f"cond_{n}", "cond_else", args, body, (n + 127) // 128, 128)


MATH_UNARY = ("tanh", "sigmoid", "silu", "softplus", "erf", "absolute", "reciprocal", "sign", "square", "floor")
MATH_BINARY = (("log", ("p1",)), ("log2", ("p1",)), ("rsqrt", ("p1",)), ("power", ("p1", "z")),
               ("floor_divide", ("x", "p1")), ("fmod", ("x", "p1")),
               ("maximum", ("x", "z")), ("minimum", ("x", "z")))


def math_zoo(n=256):
    """The rest of the math library on one vector; output [n, ops] flattened (p1 = |x| + 0.5)."""
    stmts = [Load(["x"], "x", [V("i")], "f32"), Load(["z"], "z", [V("i")], "f32"),
             Assign("ax", "absolute", ["x"]), Assign("p1", "add", ["ax", Lit(0.5)])]
    outs = []
    for k, op in enumerate(MATH_UNARY):
        stmts.append(Assign(f"u{k}", op, ["x"]))
        outs.append(f"u{k}")
    for k, (op, a) in enumerate(MATH_BINARY):
        stmts.append(Assign(f"v{k}", op, list(a)))
        outs.append(f"v{k}")
    nops = len(outs)
    stmts += [Write("y", [o], [Bin("+", Bin("*", V("i"), nops), k)], "f32") for k, o in enumerate(outs)]
    args = [TensorSpec("x", (n,), "f32", ("normal", 1.0)), TensorSpec("z", (n,), "f32", ("normal", 1.0)),
            TensorSpec("y", (n * nops,), "f32", output=True)]
    return _problem("mathzoo", f"mathzoo_{n}", "math_zoo", args, [Tile([Axis("i", n)], stmts)],
                    (n + 127) // 128, 128, ops=nops)


def hypot(n=256):
    """y = hypot(x, z) = sqrt(x*x + z*z).  The reference emitter has this op in its table but raises a
    TypeError building it (compile.py:973 passes one operand to a two-operand helper), so this case has
    no reference PTX; the source expression pins it."""
    body = [Tile([Axis("i", n)], [Load(["x"], "x", [V("i")], "f32"), Load(["z"], "z", [V("i")], "f32"),
                                  Assign("h", "hypot", ["x", "z"]), Write("y", ["h"], [V("i")], "f32")])]
    args = [TensorSpec("x", (n,), "f32", ("normal", 1.0)), TensorSpec("z", (n,), "f32", ("normal", 1.0)),
            TensorSpec("y", (n,), "f32", output=True)]
    return _problem("hypot", f"hypot_{n}", "hypot", args, body, (n + 127) // 128, 128)


def exprs(rows=8, cols=64):
    """The expression forms inside statements: FlatIndex, CastExpr (int to float), TernaryExpr, Dim,
    FuncCallExpr, and logical_and / logical_not predicates feeding a where.

    lin = r*cols + c;  t = (c < 32 ? x : 0) + 0.01*lin;  e = 0.5*exp(x);
    y = where(not (x > 0 and c < 48), e, t)
    """
    body = [Tile([Axis("r", rows), Axis("c", cols)], [
        Load(["x"], "x", [V("r"), V("c")], "f32"),
        Let("lin", {"kind": "FlatIndex", "buffer": "x", "index": [V("r"), V("c")]}),
        Assign("w", "multiply", [{"kind": "CastExpr", "expr": V("lin"), "dtype": "f32"}, Lit(0.01)]),
        Assign("t", "add", [{"kind": "TernaryExpr", "cond": Bin("<", V("c"), {"kind": "Dim", "value": 32}),
                             "if_true": V("x"), "if_false": Lit(0.0)}, "w"]),
        Assign("e", "multiply", [{"kind": "FuncCallExpr", "name": "exp", "args": [V("x")]}, Lit(0.5)]),
        Assign("pa", "logical_and", [Bin(">", V("x"), Lit(0.0)), Bin("<", V("c"), 48)], "bool"),
        Assign("pn", "logical_not", ["pa"], "bool"),
        Assign("y", "where", ["pn", "e", "t"]),
        Write("y", ["y"], [V("r"), V("c")], "f32"),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("y", (rows, cols), "f32", output=True)]
    return _problem("exprs", f"exprs_{rows}x{cols}", "expr_forms", args, body, rows * cols // 128, 128)


# ---- graphs of several kernels ----------------------------------------------------------------------


class MultiProblem(Problem):
    """A problem whose graph holds several kernels, launched in ``launches`` order; each launch is
    ``(entry, grid, block, zero_outputs, arg_order)``."""

    def __init__(self, *a, launches=(), **kw):
        super().__init__(*a, **kw)
        self.launches = [tuple(x) for x in launches]

    def meta(self) -> dict:
        ks = []
        for entry, grid, block, zero, order in self.launches:
            recs = []
            for name in order:
                s = self.spec(name)
                rec = {"name": s.name, "dtype": s.dtype, "shape": list(s.shape)}
                if s.output:
                    rec["output"] = True
                recs.append(rec)
            ks.append({"entry": entry, "arg_order": list(order), "args": recs, "grid": [grid, 1, 1],
                       "block": [block, 1, 1], "smem_bytes": 0, "zero_outputs": list(zero)})
        return {"kernels": ks, "rtol": self.rtol, "atol": self.atol}


def bcast3d(a=3, b=5, c=37):
    """y[i, j, k] = relu(x[i, j, k] * w[i] + bias[k]) in bf16: broadcasts along the leading and the
    trailing axis of an odd 3-D shape (555 cells over 64-thread blocks, so the last block is partial)."""
    body = [Tile([Axis("i", a), Axis("j", b), Axis("k", c)], [
        Load(["x"], "x", [V("i"), V("j"), V("k")], "f32"),
        Load(["w"], "w", [V("i")], "f32"),
        Load(["bias"], "bias", [V("k")], "f32"),
        Assign("m", "multiply", ["x", "w"]),
        Assign("s", "add", ["m", "bias"]),
        Assign("y", "maximum", ["s", Lit(0.0)], "bf16"),
        Write("y", ["y"], [V("i"), V("j"), V("k")], "bf16"),
    ])]
    args = [TensorSpec("x", (a, b, c), "f32", ("normal", 1.0)), TensorSpec("w", (a,), "f32", ("normal", 1.0)),
            TensorSpec("bias", (c,), "f32", ("normal", 0.5)), TensorSpec("y", (a, b, c), "bf16", output=True)]
    return _problem("bcast3d", f"bcast3d_{a}x{b}x{c}", "bcast3d", args, body, (a * b * c + 63) // 64, 64)


def row_minmax(rows=19, cols=777):
    """mx[r] = max and mn[r] = min of an odd-length row: a warp per row, lanes striding the columns,
    one warp shuffle over both states."""
    body = [Tile([Axis("row", rows), Axis("t", 32)], [
        StridedLoop("c", cols, V("t"), 32, [
            Load(["x"], "x", [V("row"), V("c")], "f32"),
            Accum("mx", "maximum", "x"),
            Accum("mn", "minimum", "x"),
        ], end=cols),
        WarpShuffle(["mx", "mn"], ["mx_o", "mn_o"], [Assign("mx", "maximum", ["mx", "mx_o"]),
                                                     Assign("mn", "minimum", ["mn", "mn_o"])]),
        Cond(Bin("==", V("t"), 0), [Write("mx", ["mx"], [V("row")], "f32"), Write("mn", ["mn"], [V("row")], "f32")]),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("mx", (rows,), "f32", output=True),
            TensorSpec("mn", (rows,), "f32", output=True)]
    return _problem("minmax", f"minmax_{rows}x{cols}", "row_minmax", args, body, rows, 32)


def small_softmax(a=2, b=3, c=45):
    """softmax over the last axis of a [2, 3, 45] tensor, a thread per row: three rolled loops (max,
    sum of exps, normalised write) over a length that is not a power of two."""
    body = [Tile([Axis("i", a), Axis("j", b)], [
        Loop("k", c, [Load(["x"], "x", [V("i"), V("j"), V("k")], "f32"), Accum("m", "maximum", "x")]),
        Loop("k1", c, [
            Load(["x1"], "x", [V("i"), V("j"), V("k1")], "f32"),
            Assign("z", "subtract", ["x1", "m"]),
            Assign("e", "exp", ["z"]),
            Accum("s", "add", "e"),
        ]),
        Loop("k2", c, [
            Load(["x2"], "x", [V("i"), V("j"), V("k2")], "f32"),
            Assign("z2", "subtract", ["x2", "m"]),
            Assign("e2", "exp", ["z2"]),
            Assign("y", "divide", ["e2", "s"]),
            Write("y", ["y"], [V("i"), V("j"), V("k2")], "f32"),
        ]),
    ])]
    args = [TensorSpec("x", (a, b, c), "f32", ("normal", 2.0)), TensorSpec("y", (a, b, c), "f32", output=True)]
    return _problem("softmax3d", f"softmax3d_{a}x{b}x{c}", "small_softmax", args, body, 1, a * b)


def _int_op(name, identity):
    """A reduce op over i32 with an explicit identity (the float table's infinities do not fit)."""
    return {"kind": "ReduceOp", "name": name, "identity": identity, "has_identity": True}


def row_argmax(rows=37, cols=333, thresh=2.0):
    """idx[r] = argmax of row r (the first index holding the maximum) and cnt[r] = the number of
    entries above ``thresh``, a warp per row of an odd length.  Pass 1 reduces the max (f32) and the
    count (i32) in one two-state shuffle; pass 2 takes the smallest column whose value equals the max
    (a Select feeding an i32 min accumulator), so ties resolve as torch.argmax does."""
    body = [Tile([Axis("row", rows), Axis("t", 32)], [
        StridedLoop("c", cols, V("t"), 32, [
            Load(["x"], "x", [V("row"), V("c")], "f32"),
            Accum("m", "maximum", "x"),
            Assign("hi", "greater", ["x", Lit(thresh)], "bool"),
            Select("one", [(V("hi"), 1), (None, 0)]),
            {**Accum("n", "add", "one", "i32"), "op": _int_op("add", 0)},
        ], end=cols),
        WarpShuffle(["m", "n"], ["m_o", "n_o"], [Assign("m", "maximum", ["m", "m_o"]),
                                                 Assign("n", "add", ["n", "n_o"], "i32")]),
        StridedLoop("c2", cols, V("t"), 32, [
            Load(["x2"], "x", [V("row"), V("c2")], "f32"),
            Assign("hit", "equal", ["x2", "m"], "bool"),
            Select("cand", [(V("hit"), "c2"), (None, cols)]),
            {**Accum("idx", "minimum", "cand", "i32"), "op": _int_op("minimum", 2 ** 31 - 1)},
        ], end=cols),
        WarpShuffle(["idx"], ["idx_o"], [Assign("idx", "minimum", ["idx", "idx_o"], "i32")]),
        Cond(Bin("==", V("t"), 0), [Write("idx", ["idx"], [V("row")], "i32"),
                                    Write("cnt", ["n"], [V("row")], "i32")]),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("idx", (rows,), "i32", output=True),
            TensorSpec("cnt", (rows,), "i32", output=True)]
    return _problem("argmax", f"argmax_{rows}x{cols}", "row_argmax", args, body, rows, 32, rtol=0.0, atol=0.0,
                    thresh=thresh)


def row_var_std(rows=4, cols=128):
    """var[r] (unbiased, n - 1) and std[r] of each row, two passes: the mean, then the sum of squared
    deviations; a warp per row, lanes striding the columns."""
    body = [Tile([Axis("row", rows), Axis("t", 32)], [
        StridedLoop("c", cols, V("t"), 32, [Load(["x"], "x", [V("row"), V("c")], "f32"), Accum("s", "add", "x")],
                    end=cols),
        WarpShuffle(["s"], ["s_o"], [Assign("s", "add", ["s", "s_o"])]),
        Assign("mean", "divide", ["s", Lit(float(cols))]),
        StridedLoop("c2", cols, V("t"), 32, [
            Load(["x2"], "x", [V("row"), V("c2")], "f32"),
            Assign("d", "subtract", ["x2", "mean"]),
            Assign("d2", "multiply", ["d", "d"]),
            Accum("q", "add", "d2"),
        ], end=cols),
        WarpShuffle(["q"], ["q_o"], [Assign("q", "add", ["q", "q_o"])]),
        Assign("var", "divide", ["q", Lit(float(cols - 1))]),
        Assign("sd", "sqrt", ["var"]),
        Cond(Bin("==", V("t"), 0), [Write("var", ["var"], [V("row")], "f32"), Write("std", ["sd"], [V("row")], "f32")]),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("var", (rows,), "f32", output=True),
            TensorSpec("std", (rows,), "f32", output=True)]
    return _problem("varstd", f"varstd_{rows}x{cols}", "row_var_std", args, body, rows, 32)


def group_norm(n=1, c=4, h=8, w=16, groups=2, eps=1e-5, threads=64):
    """group_norm(x, groups) without affine parameters: a block per (sample, group) reduces the
    group's sum and sum of squares (two states), then normalises.  The group's flat element e maps
    to x[s, g*cpg + e // (h*w), (e % (h*w)) // w, e % w]: integer division and remainder by
    constants in the index."""
    cpg = c // groups
    hw = h * w
    ne = cpg * hw
    nw = threads // 32

    def index(e):
        return [V("s"), Bin("+", Bin("*", V("g"), cpg), Bin("/", V(e), hw)), Bin("/", Bin("%", V(e), hw), w),
                Bin("%", V(e), w)]
    body = [
        Smem("red_s", [nw], "f32", 16),
        Smem("red_q", [nw], "f32", 16),
        Tile([Axis("s", n), Axis("g", groups), Axis("t", threads)], [
            StridedLoop("e", ne, V("t"), threads, [
                Load(["x"], "x", index("e"), "f32"),
                Accum("sm", "add", "x"),
                Assign("x2", "multiply", ["x", "x"]),
                Accum("sq", "add", "x2"),
            ], end=ne),
            *_block_reduce(["sm", "sq"], ["red_s", "red_q"], {"sm": "add", "sq": "add"}, nw),
            Assign("mean", "multiply", ["sm", Lit(1.0 / ne)]),
            Assign("ex2", "multiply", ["sq", Lit(1.0 / ne)]),
            Assign("mm", "multiply", ["mean", "mean"]),
            Assign("var", "subtract", ["ex2", "mm"]),
            Assign("ve", "add", ["var", Lit(eps)]),
            Assign("rs", "rsqrt", ["ve"]),
            StridedLoop("e2", ne, V("t"), threads, [
                Load(["x3"], "x", index("e2"), "f32"),
                Assign("dx", "subtract", ["x3", "mean"]),
                Assign("y", "multiply", ["dx", "rs"]),
                Write("y", ["y"], index("e2"), "f32"),
            ], end=ne),
        ]),
    ]
    args = [TensorSpec("x", (n, c, h, w), "f32", ("normal", 1.0)), TensorSpec("y", (n, c, h, w), "f32", output=True)]
    return _problem("groupnorm", f"groupnorm_{n}x{c}x{h}x{w}_g{groups}", "group_norm", args, body, n * groups,
                    threads, groups=groups, eps=eps)


def pad_rows(rows=3, cols=64, left=2, right=3):
    """y = pad(x, (left, right)) along the last axis: a cell inside the source range loads and copies
    x[r, j - left], the others write zero (a Cond with an else branch around a guarded load)."""
    out = cols + left + right
    inside = Bin("&&", Bin(">=", V("j"), left), Bin("<", V("j"), left + cols))
    body = [Tile([Axis("r", rows), Axis("j", out)], [
        Cond(inside,
             [Let("src", Bin("-", V("j"), left)), Load(["x"], "x", [V("r"), V("src")], "f32"),
              Write("y", ["x"], [V("r"), V("j")], "f32")],
             [Let("zero", Lit(0.0), "f32"), Write("y", ["zero"], [V("r"), V("j")], "f32")]),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("y", (rows, out), "f32", output=True)]
    return _problem("pad", f"pad_{rows}x{cols}_{left}_{right}", "pad_rows", args, body, (rows * out + 63) // 64, 64,
                    left=left, right=right)


def log_sum_exp(a=2, b=32, c=64):
    """logsumexp over the last axis, a warp per row of 64 (two columns a lane): the max, the sum of
    exp(x - max), then max + log(sum)."""
    body = [Tile([Axis("i", a), Axis("j", b), Axis("t", 32)], [
        StridedLoop("k", c, V("t"), 32, [Load(["x"], "x", [V("i"), V("j"), V("k")], "f32"),
                                         Accum("m", "maximum", "x")], end=c),
        WarpShuffle(["m"], ["m_o"], [Assign("m", "maximum", ["m", "m_o"])]),
        StridedLoop("k2", c, V("t"), 32, [
            Load(["x2"], "x", [V("i"), V("j"), V("k2")], "f32"),
            Assign("z", "subtract", ["x2", "m"]),
            Assign("e", "exp", ["z"]),
            Accum("s", "add", "e"),
        ], end=c),
        WarpShuffle(["s"], ["s_o"], [Assign("s", "add", ["s", "s_o"])]),
        Assign("ls", "log", ["s"]),
        Assign("y", "add", ["m", "ls"]),
        Cond(Bin("==", V("t"), 0), [Write("y", ["y"], [V("i"), V("j")], "f32")]),
    ])]
    args = [TensorSpec("x", (a, b, c), "f32", ("normal", 1.0)), TensorSpec("y", (a, b), "f32", output=True)]
    return _problem("logsumexp", f"logsumexp_{a}x{b}x{c}", "log_sum_exp", args, body, a * b * 32 // 128, 128)


def matmul_odd(m=33, k=65, n=17):
    """C = A @ B for odd sizes, a thread per output cell with a rolled Loop over k: f32 operands and
    a K of 65 (not a multiple of 8, so A's rows are no whole number of 16-byte TMA units), which the
    tensor-core lowering declines, so it stays on the CUDA cores.  Held to the matmul tolerance."""
    body = [Tile([Axis("i", m), Axis("j", n)], [
        Loop("kk", k, [
            Load(["a"], "A", [V("i"), V("kk")], "f32"),
            Load(["b"], "B", [V("kk"), V("j")], "f32"),
            Assign("p", "multiply", ["a", "b"]),
            Accum("acc", "add", "p"),
        ]),
        Write("C", ["acc"], [V("i"), V("j")], "f32"),
    ])]
    args = [TensorSpec("A", (m, k), "f32", ("normal", 1.0)), TensorSpec("B", (k, n), "f32", ("normal", 1.0)),
            TensorSpec("C", (m, n), "f32", output=True)]
    return _problem("matmul", f"matmul_{m}x{k}x{n}", "matmul_odd", args, body, (m * n + 127) // 128, 128,
                    rtol=1e-4, contraction=True)


def bmm_small(batch=2, m=32, n=32, k=64):
    """C = A @ B for [2, 32, 64] x [2, 64, 32] bf16 (the small batched matmul of the reference's
    cases): the unscheduled nest, a thread per output element.  Far below one 128 x 256 tile, it
    runs on the tensor cores as a single edge tile (TMA zero-fills the box past M, N and the store
    keeps rows below M and columns below N)."""
    from .irgen import bmm_naive_ir
    base = bmm_naive_ir(batch, m, n, k)
    args = [TensorSpec("A", (batch, m, k), "bf16", ("normal", 1.0)),
            TensorSpec("B", (batch, k, n), "bf16", ("normal", 1.0)),
            TensorSpec("C", (batch, m, n), "f32", output=True)]
    return Problem(f"bmm_small_{batch}x{m}x{n}x{k}", "corpus", base.entry, base.graph, args, grid=base.grid,
                   block=base.block, rtol=1e-4, atol=1e-6, params={"expr": "matmul", "contraction": True})


def sdpa(batch, heads, seq, dim, causal, scale=None, mask=False):
    """scaled_dot_product_attention of bf16 Q, K, V [batch, heads, seq, dim] (optionally causal, with
    an explicit scale): the online-softmax nest of the attention IR at the small shapes of the
    reference's attention cases.  Head dim 32, 64 or 128 runs on the tensor cores at any S (the mask
    also needs S % 16 == 0); other head dims run on the CUDA cores."""
    from .irgen import attention_ir
    base = attention_ir(batch, heads, seq, dim, causal, scale=scale, mask=mask)
    return Problem(f"sdpa_{batch}x{heads}x{seq}x{dim}{'_causal' if causal else ''}{'_mask' if mask else ''}",
                   "corpus", base.entry, base.graph, base.args, grid=base.grid, block=base.block, rtol=1e-4,
                   atol=1e-6, params={"expr": "sdpa", "contraction": True, "attention": True, "causal": causal,
                                      "scale": base.params["scale"], "mask": mask})


def sdpa_rows(batch, heads, seq, dim, dv, causal, scale=None, threads=64):
    """scaled_dot_product_attention with a value head dim ``dv`` that may differ from the query/key
    head dim ``dim``, and head dims that are no multiple of 32 (40, 16): one thread per query row.
    The thread loads its query row once (``dim`` lanes of one Load), and for each key row loads it,
    forms the dot product as a pairwise sum, masks it (causal: a Select to -inf), and runs the online
    softmax with ``dv`` output accumulators whose ``base`` is the rescaled previous value."""
    scale = 1.0 / math.sqrt(dim) if scale is None else float(scale)
    qs = [f"q{i}" for i in range(dim)]
    ks = [f"k{i}" for i in range(dim)]
    vs = [f"v{i}" for i in range(dv)]
    os_ = [f"o{i}" for i in range(dv)]
    dot = [Assign(f"pp{i}", "multiply", [qs[i], ks[i]]) for i in range(dim)]
    terms, lvl = [f"pp{i}" for i in range(dim)], 0
    while len(terms) > 1:
        nxt = []
        for j in range(0, len(terms) - 1, 2):
            nm = "dp" if len(terms) == 2 else f"ds{lvl}_{j // 2}"
            dot.append(Assign(nm, "add", [terms[j], terms[j + 1]]))
            nxt.append(nm)
        if len(terms) % 2:
            nxt.append(terms[-1])                  # an odd term carries to the next level
        terms, lvl = nxt, lvl + 1
    sel = [(Bin(">", V("kv"), V("qi")), Lit(-math.inf))] if causal else []
    body_k = [
        Load(ks, "K", [V("b"), V("h"), V("kv"), 0], "bf16"),
        *dot,
        Assign("sc", "multiply", ["dp", Lit(scale)]),
        Select("sm", [*sel, (None, "sc")]),
        Assign("mn", "maximum", ["m", "sm"]),
        Assign("dm", "subtract", ["m", "mn"]),
        Assign("alpha", "exp", ["dm"]),
        Assign("ds", "subtract", ["sm", "mn"]),
        Assign("pe", "exp", ["ds"]),
        Assign("ls", "multiply", ["l", "alpha"]),
        Accum("l", "add", "pe", base="ls"),
        Load(vs, "V", [V("b"), V("h"), V("kv"), 0], "bf16"),
        *[Assign(f"os{i}", "multiply", [os_[i], "alpha"]) for i in range(dv)],
        *[Assign(f"pv{i}", "multiply", ["pe", vs[i]]) for i in range(dv)],
        *[Accum(os_[i], "add", f"pv{i}", base=f"os{i}") for i in range(dv)],
        Accum("m", "maximum", "sm"),
    ]
    body = [Tile([Axis("b", batch), Axis("h", heads), Axis("qi", seq)], [
        Load(qs, "Q", [V("b"), V("h"), V("qi"), 0], "bf16"),
        Init("m", "f32", -math.inf),
        Init("l", "f32", 0.0),
        *[Init(o, "f32", 0.0) for o in os_],
        Loop("kv", seq, body_k),
        *[Assign(f"y{i}", "divide", [os_[i], "l"], "bf16") for i in range(dv)],
        Write("O", [f"y{i}" for i in range(dv)], [V("b"), V("h"), V("qi"), 0], "bf16"),
    ])]
    args = [TensorSpec("Q", (batch, heads, seq, dim), "bf16", ("normal", 1.0)),
            TensorSpec("K", (batch, heads, seq, dim), "bf16", ("normal", 1.0)),
            TensorSpec("V", (batch, heads, seq, dv), "bf16", ("normal", 1.0)),
            TensorSpec("O", (batch, heads, seq, dv), "bf16", output=True)]
    rows = batch * heads * seq
    return _problem("sdpa", f"sdpa_rows_{batch}x{heads}x{seq}x{dim}x{dv}{'_causal' if causal else ''}",
                    "attention_rows", args, body, (rows + threads - 1) // threads, threads, rtol=1e-4,
                    contraction=True, attention=True, causal=causal, scale=scale, mask=False)


def scan_max_and_prod(rows=4, cols=64):
    """cm[r, c] = max of x[r, :c+1] (a running max: a thread per row, the Accum read after each step
    of a rolled Loop) and pr[r] = prod of x[r, :] (a warp per row: Accum multiply, then a shuffle
    whose combine is a product, which has no redux form)."""
    body = [Tile([Axis("row", rows), Axis("t", 32)], [
        Cond(Bin("==", V("t"), 0), [
            Loop("c", cols, [
                Load(["x"], "x", [V("row"), V("c")], "f32"),
                Accum("cm", "maximum", "x"),
                Write("cm", ["cm"], [V("row"), V("c")], "f32"),
            ]),
        ]),
        StridedLoop("c2", cols, V("t"), 32, [Load(["x2"], "x", [V("row"), V("c2")], "f32"),
                                             Accum("pr", "multiply", "x2")], end=cols),
        WarpShuffle(["pr"], ["pr_o"], [Assign("pr", "multiply", ["pr", "pr_o"])]),
        Cond(Bin("==", V("t"), 0), [Write("pr", ["pr"], [V("row")], "f32")]),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("uniform", 0.5, 1.5)),
            TensorSpec("cm", (rows, cols), "f32", output=True), TensorSpec("pr", (rows,), "f32", output=True)]
    return _problem("scanprod", f"scanprod_{rows}x{cols}", "scan_max_prod", args, body, rows, 32)


def special_values(n=777):
    """IEEE special values through the elementwise forms (the input holds NaN, +-inf, +0, 1e30 and a
    small negative number at fixed positions, normal values elsewhere).  The results follow the PTX
    instructions the reference emits: ``max.f32`` / ``min.f32`` return the non-NaN operand (relu of
    NaN is 0), ``setp`` comparisons are ordered (NaN > 0 is false, and so is NaN != NaN), ``testp``
    detects NaN; exp, log, sqrt and 1/x give IEEE's infinities and NaNs."""
    outs = ["relu", "mn", "ex", "lg", "sq", "rc", "wh"]
    body = [Tile([Axis("i", n)], [
        Load(["x"], "x", [V("i")], "f32"),
        Assign("relu", "maximum", ["x", Lit(0.0)]),
        Assign("mn", "minimum", ["x", Lit(1.0)]),
        Assign("ex", "exp", ["x"]),
        Assign("lg", "log", ["x"]),
        Assign("sq", "sqrt", ["x"]),
        Assign("rc", "divide", [Lit(1.0), "x"]),
        Assign("pos", "greater", ["x", Lit(0.0)], "bool"),
        Assign("wh", "where", ["pos", "x", Lit(-1.0)]),
        Assign("isn", "isnan", ["x"], "bool"),
        Assign("ne", "not_equal", ["x", "x"], "bool"),
        Assign("xb", "multiply", ["x", Lit(2.0)], "bf16"),
        *[Write(o, [o], [V("i")], "f32") for o in outs],
        Write("nanm", ["isn"], [V("i")], "u8"),
        Write("nem", ["ne"], [V("i")], "u8"),
        Write("xb", ["xb"], [V("i")], "bf16"),
    ])]
    args = [TensorSpec("x", (n,), "f32", ("special", 1.0)),
            *[TensorSpec(o, (n,), "f32", output=True) for o in outs],
            TensorSpec("nanm", (n,), "u8", output=True), TensorSpec("nem", (n,), "u8", output=True),
            TensorSpec("xb", (n,), "bf16", output=True)]
    return _problem("special", f"special_{n}", "special_values", args, body, (n + 127) // 128, 128)


def special_values_16bit(n=640):
    """The special values through 16-bit loads and stores: bf16 and f16 inputs holding NaN, +-inf
    and +0 (the 1e30 of the f32 pattern is already inf in f16) are widened to f32 (bf16 by a shift of
    the packed word, f16 by ``cvt``), go through max / multiply / isnan, and are narrowed back."""
    body = [Tile([Axis("i8", n // 8)], [
        Let("i", Bin("*", V("i8"), 8)),
        Load([f"b{k}" for k in range(8)], "xb", [V("i")], "bf16"),
        Load([f"h{k}" for k in range(8)], "xh", [V("i")], "f16"),
        *[Assign(f"rb{k}", "maximum", [f"b{k}", Lit(0.0)], "bf16") for k in range(8)],
        *[Assign(f"dh{k}", "multiply", [f"h{k}", Lit(2.0)], "f16") for k in range(8)],
        *[Assign(f"nb{k}", "isnan", [f"b{k}"], "bool") for k in range(8)],
        Write("yb", [f"rb{k}" for k in range(8)], [V("i")], "bf16"),
        Write("yh", [f"dh{k}" for k in range(8)], [V("i")], "f16"),
        *[Write("nanb", [f"nb{k}"], [Bin("+", V("i"), k)], "u8") for k in range(8)],
    ])]
    args = [TensorSpec("xb", (n,), "bf16", ("special", 1.0)), TensorSpec("xh", (n,), "f16", ("special", 1.0)),
            TensorSpec("yb", (n,), "bf16", output=True), TensorSpec("yh", (n,), "f16", output=True),
            TensorSpec("nanb", (n,), "u8", output=True)]
    return _problem("special16", f"special16_{n}", "special_values_16bit", args, body, (n // 8 + 63) // 64, 64)


def softmax_mid(a=4, b=32, c=16):
    """softmax over the middle axis of [4, 32, 16] (torch dim=1): a thread per (i, k) column walks j
    in three rolled loops, every load 16 elements (64 bytes) from the previous one."""
    body = [Tile([Axis("i", a), Axis("k", c)], [
        Loop("j", b, [Load(["x"], "x", [V("i"), V("j"), V("k")], "f32"), Accum("m", "maximum", "x")]),
        Loop("j1", b, [
            Load(["x1"], "x", [V("i"), V("j1"), V("k")], "f32"),
            Assign("z", "subtract", ["x1", "m"]),
            Assign("e", "exp", ["z"]),
            Accum("s", "add", "e"),
        ]),
        Loop("j2", b, [
            Load(["x2"], "x", [V("i"), V("j2"), V("k")], "f32"),
            Assign("z2", "subtract", ["x2", "m"]),
            Assign("e2", "exp", ["z2"]),
            Assign("y", "divide", ["e2", "s"]),
            Write("y", ["y"], [V("i"), V("j2"), V("k")], "f32"),
        ]),
    ])]
    args = [TensorSpec("x", (a, b, c), "f32", ("normal", 1.0)), TensorSpec("y", (a, b, c), "f32", output=True)]
    return _problem("softmax_mid", f"softmax_mid_{a}x{b}x{c}", "softmax_mid", args, body, 1, a * c)


FLT_MAX = 3.4028234663852886e38


def nan_to_num(n=777):
    """y = nan_to_num(x): NaN -> 0, +inf -> the largest f32, -inf -> its negative, other values
    unchanged (torch's defaults).  NaN is found with ``isnan`` (``testp.notanumber``): an ordered
    comparison such as x != x is false on NaN in the instructions the IR lowers to."""
    body = [Tile([Axis("i", n)], [
        Load(["x"], "x", [V("i")], "f32"),
        Assign("isn", "isnan", ["x"], "bool"),
        Assign("isi", "isinf", ["x"], "bool"),
        Assign("pos", "greater", ["x", Lit(0.0)], "bool"),
        Select("y", [(V("isn"), Lit(0.0)),
                     (Bin("&&", V("isi"), V("pos")), Lit(FLT_MAX)),
                     (V("isi"), Lit(-FLT_MAX)),
                     (None, "x")]),
        Write("y", ["y"], [V("i")], "f32"),
    ])]
    args = [TensorSpec("x", (n,), "f32", ("special", 1.0)), TensorSpec("y", (n,), "f32", output=True)]
    return _problem("nan_to_num", f"nan_to_num_{n}", "nan_to_num", args, body, (n + 127) // 128, 128)


def log_add_exp(n=1000):
    """y = logaddexp(a, b) = max(a, b) + log1p(exp(-|a - b|)), the overflow-free form."""
    body = [Tile([Axis("i", n)], [
        Load(["a"], "a", [V("i")], "f32"), Load(["b"], "b", [V("i")], "f32"),
        Assign("m", "maximum", ["a", "b"]),
        Assign("d", "subtract", ["a", "b"]),
        Assign("ad", "absolute", ["d"]),
        Assign("nd", "negative", ["ad"]),
        Assign("e", "exp", ["nd"]),
        Assign("l", "log1p", ["e"]),
        Assign("y", "add", ["m", "l"]),
        Write("y", ["y"], [V("i")], "f32"),
    ])]
    args = [TensorSpec("a", (n,), "f32", ("normal", 3.0)), TensorSpec("b", (n,), "f32", ("normal", 3.0)),
            TensorSpec("y", (n,), "f32", output=True)]
    return _problem("logaddexp", f"logaddexp_{n}", "log_add_exp", args, body, (n + 127) // 128, 128)


SELU_ALPHA = 1.6732632423543772
SELU_SCALE = 1.0507009873554805


def elu_selu(rows=2, cols=320):
    """elu(x) = x if x > 0 else expm1(x) (alpha 1) and selu(x) = scale * (x if x > 0 else
    alpha * expm1(x)), four elements a thread through 16-byte vector loads and stores."""
    n = rows * cols
    body = [Tile([Axis("i4", n // 4)], [
        Let("i", Bin("*", V("i4"), 4)),
        Load([f"x{k}" for k in range(4)], "x", [V("i")], "f32"),
        *[st for k in range(4) for st in (
            Assign(f"p{k}", "greater", [f"x{k}", Lit(0.0)], "bool"),
            Assign(f"m{k}", "expm1", [f"x{k}"]),
            Assign(f"e{k}", "where", [f"p{k}", f"x{k}", f"m{k}"]),
            Assign(f"am{k}", "multiply", [f"m{k}", Lit(SELU_ALPHA)]),
            Assign(f"sv{k}", "where", [f"p{k}", f"x{k}", f"am{k}"]),
            Assign(f"s{k}", "multiply", [f"sv{k}", Lit(SELU_SCALE)]))],
        Write("elu", [f"e{k}" for k in range(4)], [V("i")], "f32"),
        Write("selu", [f"s{k}" for k in range(4)], [V("i")], "f32"),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("elu", (rows, cols), "f32", output=True),
            TensorSpec("selu", (rows, cols), "f32", output=True)]
    return _problem("elu_selu", f"elu_selu_{rows}x{cols}", "elu_selu", args, body, (n // 4 + 63) // 64, 64)


def row_any(rows=64, cols=96, thresh=2.5):
    """out[r] = any(x[r, :] > thresh) as a byte, a warp per row: each lane folds its columns' tests
    into an i32 flag with a maximum Accum, one shuffle takes the warp's maximum."""
    body = [Tile([Axis("row", rows), Axis("t", 32)], [
        StridedLoop("c", cols, V("t"), 32, [
            Load(["x"], "x", [V("row"), V("c")], "f32"),
            Assign("hi", "greater", ["x", Lit(thresh)], "bool"),
            Select("one", [(V("hi"), 1), (None, 0)]),
            {**Accum("f", "maximum", "one", "i32"), "op": _int_op("maximum", 0)},
        ], end=cols),
        WarpShuffle(["f"], ["f_o"], [Assign("f", "maximum", ["f", "f_o"], "i32")]),
        Assign("any", "greater", ["f", 0], "bool"),
        Cond(Bin("==", V("t"), 0), [Write("out", ["any"], [V("row")], "u8")]),
    ])]
    args = [TensorSpec("x", (rows, cols), "f32", ("normal", 1.0)), TensorSpec("out", (rows,), "u8", output=True)]
    return _problem("any", f"any_{rows}x{cols}", "row_any", args, body, rows, 32, rtol=0.0, atol=0.0,
                    thresh=thresh)


def l2_normalize(rows=64, cols=256, eps=1e-12, threads=64):
    """y = x / max(||x||_2, eps) along the last axis of [2, 32, 256] (torch.nn.functional.normalize),
    a block per row: block-strided sum of squares, block reduction, one division per element."""
    nw = threads // 32
    body = [
        Smem("red", [nw], "f32", 16),
        Tile([Axis("row", rows), Axis("t", threads)], [
            StridedLoop("c", cols, V("t"), threads, [
                Load(["x"], "x", [V("row"), V("c")], "f32"),
                Assign("sq", "multiply", ["x", "x"]),
                Accum("ss", "add", "sq"),
            ], end=cols),
            *_block_reduce(["ss"], ["red"], {"ss": "add"}, nw),
            Assign("nrm", "sqrt", ["ss"]),
            Assign("den", "maximum", ["nrm", Lit(eps)]),
            StridedLoop("c2", cols, V("t"), threads, [
                Load(["x2"], "x", [V("row"), V("c2")], "f32"),
                Assign("y", "divide", ["x2", "den"]),
                Write("y", ["y"], [V("row"), V("c2")], "f32"),
            ], end=cols),
        ]),
    ]
    args = [TensorSpec("x", (2, 32, cols), "f32", ("normal", 1.0)), TensorSpec("y", (2, 32, cols), "f32", output=True)]
    return _problem("l2norm", f"l2norm_{rows}x{cols}", "l2_normalize", args, body, rows, threads, eps=eps)


def _kernel_node(entry, inputs, outputs, body):
    return {"op": "KernelOp", "op_fields": {"name": entry, "body": body}, "inputs": list(inputs),
            "outputs": [{"name": o.name, "shape": list(o.shape), "dtype": o.dtype} for o in outputs]}


def _multi_graph(inputs, kernels, outputs):
    nodes = {a.name: {"op": "InputOp", "op_fields": {}, "inputs": [],
                      "outputs": [{"name": a.name, "shape": list(a.shape), "dtype": a.dtype}]} for a in inputs}
    for entry, ins, outs, body in kernels:
        nodes[entry] = _kernel_node(entry, ins, outs, body)
    return {"nodes": nodes, "inputs": [a.name for a in inputs], "outputs": [a.name for a in outputs]}


def chain_mul_relu(n=1024):
    """Kernel 1: t = a * b into an intermediate buffer; kernel 2: y = relu(t + c)."""
    a, b, c = (TensorSpec(nm, (n,), "f32", ("normal", 1.0)) for nm in "abc")
    t = TensorSpec("t", (n,), "f32", output=True)
    y = TensorSpec("y", (n,), "f32", output=True)
    k1 = [Tile([Axis("i", n)], [Load(["a"], "a", [V("i")], "f32"), Load(["b"], "b", [V("i")], "f32"),
                                Assign("p", "multiply", ["a", "b"]), Write("t", ["p"], [V("i")], "f32")])]
    k2 = [Tile([Axis("i", n)], [Load(["t"], "t", [V("i")], "f32"), Load(["c"], "c", [V("i")], "f32"),
                                Assign("q", "add", ["t", "c"]), Assign("r", "relu", ["q"]),
                                Write("y", ["r"], [V("i")], "f32")])]
    g = _multi_graph([a, b, c], [("mul_kernel", ["a", "b"], [t], k1), ("relu_kernel", ["t", "c"], [y], k2)], [y])
    return MultiProblem(f"chain_{n}", "corpus", "mul_kernel", g, [a, b, c, t, y], grid=n // 128, block=128,
                        params={"expr": "chain"},
                        launches=[("mul_kernel", n // 128, 128, [], ["a", "b", "t"]),
                                  ("relu_kernel", n // 128, 128, [], ["t", "c", "y"])])


def zero_then_histogram(n=4096, bins=16):
    """Kernel 1 zeroes the histogram with a ZeroPrologue (no host memset); kernel 2 adds one per
    element atomically into bin x % bins."""
    x = TensorSpec("x", (n,), "i32", ("randint", 0, 1000))
    h = TensorSpec("hist", (bins,), "i32", output=True)
    k1 = [{"kind": "ZeroPrologue", "dst": "hist", "words": bins}]
    k2 = [Tile([Axis("i", n)], [Load(["x"], "x", [V("i")], "i32"),
                                Assign("bn", "modulo", ["x", bins], "i32"),
                                Let("one", 1),
                                Write("hist", ["one"], [V("bn")], "i32", atomic=True)])]
    g = _multi_graph([x], [("zero_kernel", ["x"], [h], k1), ("hist_kernel", ["x", "hist"], [], k2)], [h])
    return MultiProblem(f"hist_{n}", "corpus", "zero_kernel", g, [x, h], grid=2, block=64, rtol=0.0, atol=0.0,
                        params={"expr": "hist", "bins": bins},
                        launches=[("zero_kernel", 2, 64, [], ["x", "hist"]),
                                  ("hist_kernel", n // 128, 128, [], ["x", "hist"])])


CORPUS = {
    "k_rmsnorm": rmsnorm,
    "k_layernorm": layernorm,
    "k_logsoftmax": log_softmax,
    "k_colsum": col_sum,
    "k_midsum": mid_sum,
    "k_tri": prefix_sum_tri,
    "k_cumsum": cumsum_rows,
    "k_cumsum1d": cumsum_1d,
    "k_intops": int_ops,
    "k_gelu_f16": half_gelu,
    "k_mask": mask_where,
    "k_f64": f64_affine,
    "k_cond": cond_else,
    "k_mathzoo": math_zoo,
    "k_hypot": hypot,
    "k_exprs": exprs,
    "k_chain": chain_mul_relu,
    "k_hist": zero_then_histogram,
    "k_bcast3d": bcast3d,
    "k_minmax": row_minmax,
    "k_softmax3d": small_softmax,
    "k_argmax": row_argmax,
    "k_varstd": row_var_std,
    "k_groupnorm": group_norm,
    "k_pad": pad_rows,
    "k_logsumexp": log_sum_exp,
    "k_matmul_odd": matmul_odd,
    "k_special": special_values,
    "k_scanprod": scan_max_and_prod,
    "k_special16": special_values_16bit,
    "k_softmax_mid": softmax_mid,
    "k_nan_to_num": nan_to_num,
    "k_logaddexp": log_add_exp,
    "k_elu_selu": elu_selu,
    "k_any": row_any,
    "k_l2norm": l2_normalize,
    "k_bmm_small": bmm_small,
    # m_vec / m_col of the reference's cases: a row vector times a matrix, a matrix times a column
    "k_matvec": lambda: matmul_odd(1, 256, 256),
    "k_matcol": lambda: matmul_odd(256, 256, 1),
    # a_sdpa_causal and a_sdpa_scale: causal at head dim 64, and an explicit scale at 48 rows, dim 32
    "k_sdpa_causal": lambda: sdpa(1, 2, 64, 64, True),
    "k_sdpa_scale": lambda: sdpa(1, 4, 48, 32, False, scale=0.2),
    # a_mask: an explicit boolean attention mask (random here, so some rows start with masked keys)
    "k_sdpa_mask": lambda: sdpa(1, 2, 16, 32, False, mask=True),
    # a_sdpa_odd and a_sdpa_causal2: a query/key head dim of 40 with 32-wide values, and a causal
    # case with 32-wide queries and keys but 16-wide values
    "k_sdpa_odd": lambda: sdpa_rows(1, 3, 48, 40, 32, False),
    # a_sdpa_big: 128 rows at head dim 64, on the tensor cores (one CTA per head, its second query
    # tile entirely past S)
    "k_sdpa_big": lambda: sdpa(1, 4, 128, 64, False),
    "k_sdpa_causal2": lambda: sdpa_rows(2, 4, 64, 32, 16, True),
}
