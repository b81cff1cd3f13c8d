"""CPU oracle: a numpy SIMT interpreter of Emmy kernel IR, restating the reference's semantics.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline / reference arm may import this module, and only as the checker or the timed CPU
baseline.  The product path (``emmy_ptx_b200``) never calls it.

What it restates: the meaning of each IR statement as the reference PTX emitter lowers it
(``compile.py`` in fanjialin8-create/emmy-ptx; line numbers cite that file).  Every thread of
a block chunk runs in lockstep, one statement at a time, over numpy arrays of shape
``(blocks * threads,)``.  Lockstep execution is one legal interleaving of a race-free kernel,
so ``Sync``/``CpAsyncWait`` are no-ops here; branches and data-dependent loops run under a
lane mask, exactly like divergent SIMT code.

Numerics follow the emitted instructions: f16/bf16 are widened to f32 on load and narrowed
once, round-to-nearest-even, at the store (compile.py:1178-1182, 1257-1260); arithmetic is
IEEE f32 (``add/sub/mul/div.rn/sqrt.rn/rcp.rn``); ``exp(x)`` is ``2^(x*log2 e)`` evaluated in f32
(compile.py:1017-1018); integer ``/`` and ``%`` truncate toward zero (compile.py:274-275);
``max``/``min`` return the non-NaN operand like ``max.f32`` (compile.py:73-74).  The hardware
``ex2.approx``/``lg2.approx`` are evaluated exactly here, so GPU results differ from the oracle
by a few f32 ulp in transcendental-heavy kernels; the tests' tolerances cover that.

Pinning: the oracle is checked against (1) torch-CPU evaluations of each source expression
(``oracle/torch_ref.py``) and (2) the reference emitter's own PTX, committed under
``tests/golden/ref_ptx`` and run on the GPU on the same seeded inputs.
"""
from __future__ import annotations

import math
import numpy as np

LW = np.float32(1.4426950408889634)   # log2(e), compile.py:163
LN2 = np.float32(0.6931471805599453)  # compile.py:164
_F = np.float32


# ---- storage formats --------------------------------------------------------------------

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen raw bf16 bits to f32 (``cvt.f32.bf16``, exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Narrow f32 to bf16 bits, round to nearest even, NaN kept quiet (``cvt.rn.bf16.f32``)."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(x)
    out = rounded.astype(np.uint32)
    out = np.where(nan, (u >> 16).astype(np.uint32) | 0x40, out)
    return out.astype(np.uint16)


def _dt(dt) -> str:
    n = getattr(dt, "name", None)
    if n is None:
        n = str(dt)
    return {"float32": "f32", "float16": "f16", "float64": "f64", "int32": "i32", "int64": "i64",
            "float": "f32", "double": "f64", "half": "f16", "int": "i32", "bfloat16": "bf16"}.get(n, n)


_BYTES = {"f16": 2, "bf16": 2, "f32": 4, "f64": 8, "i32": 4, "i64": 8, "u32": 4, "u64": 8,
          "bool": 1, "bool8": 1, "i1": 1, "u8": 1, "i8": 1}
_STORE = {"f16": np.uint16, "bf16": np.uint16, "f32": np.float32, "f64": np.float64, "i32": np.int32,
          "i64": np.int64, "u32": np.uint32, "u64": np.uint64, "bool": np.uint8, "bool8": np.uint8,
          "i1": np.uint8, "u8": np.uint8, "i8": np.int8}
FLOATS = ("f16", "bf16", "f32", "f64")


def storage_dtype(dt: str):
    """The numpy dtype that holds a buffer of this IR dtype (16-bit floats as raw bits)."""
    return _STORE[_dt(dt)]


def widen(raw: np.ndarray, dt: str) -> np.ndarray:
    """A buffer's elements as the register values a Load produces (compile.py:1159-1204)."""
    dt = _dt(dt)
    if dt == "bf16":
        return bf16_bits_to_f32(raw)
    if dt == "f16":
        return raw.view(np.float16).astype(np.float32)
    if dt == "f64":
        return raw.astype(np.float32)           # narrowed in the register (compile.py:1183-1193)
    if dt in ("f32",):
        return raw.astype(np.float32)
    return raw.astype(np.int32)


def narrow(vals: np.ndarray, dt: str) -> np.ndarray:
    """Register values as stored bits of a buffer of this dtype (compile.py:1346-1382)."""
    dt = _dt(dt)
    if dt == "bf16":
        return f32_to_bf16_bits(vals)
    if dt == "f16":
        return np.asarray(vals, dtype=np.float32).astype(np.float16).view(np.uint16)
    if dt == "f64":
        return np.asarray(vals, dtype=np.float32).astype(np.float64)
    return np.asarray(vals).astype(_STORE[dt])


def _trunc_div(a, b):
    a = np.asarray(a, dtype=np.int64)
    b = np.asarray(b, dtype=np.int64)
    safe = np.where(b == 0, 1, b)
    q = np.abs(a) // np.abs(safe)
    return np.where((a < 0) ^ (safe < 0), -q, q)


def _wrap(x):
    return np.asarray(x, dtype=np.int64).astype(np.int32)


# ---- the math library (compile.py:1006-1111) ----------------------------------------------

def _exp(x):
    return np.exp2(_F(x) * LW, dtype=np.float32)


def _lg2(x):
    with np.errstate(divide="ignore", invalid="ignore"):
        return np.log2(np.asarray(x, dtype=np.float32))


def _rcp(x):
    with np.errstate(divide="ignore"):
        return _F(1.0) / np.asarray(x, dtype=np.float32)


def _sigmoid(x):
    return _rcp(np.exp2(np.asarray(x, dtype=np.float32) * _F(-LW)) + _F(1.0))


def _tanh(x):
    e2 = np.exp2(np.asarray(x, dtype=np.float32) * _F(2.0 * 1.4426950408889634))
    return _F(1.0) - _F(2.0) / (e2 + _F(1.0))


def _erf(x):
    """Abramowitz & Stegun 7.1.26 with the sign restored (compile.py:1038-1056)."""
    x = np.asarray(x, dtype=np.float32)
    ax = np.abs(x)
    t = _rcp(_F(0.3275911) * ax + _F(1.0))
    poly = np.full_like(t, _F(1.061405429))
    for c in (-1.453152027, 1.421413741, -0.284496736, 0.254829592):
        poly = poly * t + _F(c)
    series = poly * t
    tail = series * _exp(-(ax * ax))
    y = _F(1.0) - tail
    return np.where(np.signbit(x), -y, y).astype(np.float32)


def _gelu(x):
    x = np.asarray(x, dtype=np.float32)
    return (x * _F(0.5)) * (_erf(x * _F(0.7071067811865476)) + _F(1.0))


def _gelu_tanh(x):
    x = np.asarray(x, dtype=np.float32)
    x3 = (x * x) * x
    inner = _F(0.7978845608028654) * (x + _F(0.044715) * x3)
    return (x * _F(0.5)) * (_tanh(inner) + _F(1.0))


def _softplus(x):
    x = np.asarray(x, dtype=np.float32)
    e = _exp(np.abs(x) * _F(-1.0))
    return np.fmax(x, _F(0.0)) + _lg2(e + _F(1.0)) * LN2


def _sign(x):
    x = np.asarray(x, dtype=np.float32)
    return np.where(x != 0, np.where(x > 0, _F(1.0), _F(-1.0)), _F(0.0)).astype(np.float32)


def _fmod(x, y):
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.trunc(np.asarray(x, dtype=np.float32) / np.asarray(y, dtype=np.float32))
        return np.asarray(x, dtype=np.float32) - q * np.asarray(y, dtype=np.float32)


def _floor_div(x, y):
    with np.errstate(divide="ignore", invalid="ignore"):
        return np.floor(np.asarray(x, dtype=np.float32) / np.asarray(y, dtype=np.float32))


UNARY_F = {
    "neg": np.negative, "negative": np.negative, "absolute": np.abs, "abs": np.abs, "fabs": np.abs,
    "sqrt": np.sqrt, "rsqrt": lambda x: _rcp(np.sqrt(x)), "reciprocal": _rcp,
    "sin": np.sin, "cos": np.cos, "floor": np.floor, "ceil": np.ceil, "round": np.rint,
    "rint": np.rint, "trunc": np.trunc,
    "relu": lambda x: np.fmax(x, _F(0.0)),
    "exp": _exp, "exp_fast": _exp, "exp2": lambda x: np.exp2(np.asarray(x, dtype=np.float32)),
    "log": lambda x: _lg2(x) * LN2, "ln": lambda x: _lg2(x) * LN2, "log2": _lg2,
    "log10": lambda x: _lg2(x) * _F(0.30102999566398120),
    "tanh": _tanh, "sigmoid": _sigmoid, "silu": lambda x: np.asarray(x, dtype=np.float32) * _sigmoid(x),
    "softplus": _softplus, "gelu": _gelu, "gelu_tanh": _gelu_tanh, "erf": _erf, "sign": _sign,
    "square": lambda x: np.asarray(x, dtype=np.float32) * np.asarray(x, dtype=np.float32),
    "positive": lambda x: x,
    "log1p": lambda x: _lg2(np.asarray(x, dtype=np.float32) + _F(1.0)) * LN2,
    "expm1": lambda x: _exp(x) - _F(1.0),
    "sinh": lambda x: _F(0.5) * (_exp(x) - _exp(np.asarray(x, dtype=np.float32) * _F(-1.0))),
    "cosh": lambda x: _F(0.5) * (_exp(x) + _exp(np.asarray(x, dtype=np.float32) * _F(-1.0))),
}
BINARY_F = {
    "add": np.add, "subtract": np.subtract, "multiply": np.multiply,
    "divide": np.divide, "maximum": np.fmax, "minimum": np.fmin,
    "power": lambda x, y: np.exp2(np.asarray(y, dtype=np.float32) * _lg2(x)),
    "pow": lambda x, y: np.exp2(np.asarray(y, dtype=np.float32) * _lg2(x)),
    "mod": _fmod, "remainder": _fmod, "fmod": _fmod, "floor_divide": _floor_div,
    "hypot": lambda x, y: np.sqrt(np.asarray(x, np.float32) * x + np.asarray(y, np.float32) * y),
}
BINARY_I = {
    "add": lambda a, b: _wrap(np.int64(0) + a + b), "subtract": lambda a, b: _wrap(np.int64(0) + a - b),
    "multiply": lambda a, b: _wrap(np.asarray(a, np.int64) * b),
    "divide": lambda a, b: _wrap(_trunc_div(a, b)),
    "modulo": lambda a, b: _wrap(np.asarray(a, np.int64) - _trunc_div(a, b) * b),
    "remainder": lambda a, b: _wrap(np.asarray(a, np.int64) - _trunc_div(a, b) * b),
    "fmod": lambda a, b: _wrap(np.asarray(a, np.int64) - _trunc_div(a, b) * b),
    "maximum": np.maximum, "minimum": np.minimum,
    "bitwise_and": np.bitwise_and, "bitwise_or": np.bitwise_or, "bitwise_xor": np.bitwise_xor,
    "and": np.bitwise_and, "or": np.bitwise_or, "xor": np.bitwise_xor,
    "left_shift": lambda a, b: _wrap(np.left_shift(np.asarray(a, np.int64), b)),
    "right_shift": lambda a, b: np.right_shift(np.asarray(a, np.int32), b),
}
def _not_equal(a, b):
    """``setp.ne``: an ordered comparison, false when either float operand is NaN (the reference maps
    not_equal and ``!=`` to ``ne``, compile.py:84 and 760), where numpy's ``!=`` is true."""
    r = np.not_equal(a, b)
    for x in (a, b):
        x = np.asarray(x)
        if x.dtype.kind == "f":
            r = r & ~np.isnan(x)
    return r


COMPARE = {"greater": np.greater, "less": np.less, "greater_equal": np.greater_equal,
           "less_equal": np.less_equal, "equal": np.equal, "not_equal": _not_equal}
EXPR_CMP = {"==": np.equal, "!=": _not_equal, "<": np.less, "<=": np.less_equal,
            ">": np.greater, ">=": np.greater_equal}
EXPR_I = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide", "%": "modulo",
          "&": "bitwise_and", "|": "bitwise_or", "^": "bitwise_xor", "<<": "left_shift",
          ">>": "right_shift"}
EXPR_F = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide"}


class Val:
    """A register file slice: one value per lane, of kind f (f32), i (s32) or p (predicate)."""

    __slots__ = ("v", "k")

    def __init__(self, v, k: str) -> None:
        self.v = v
        self.k = k


def _cast(val: Val, want: str) -> Val:
    """compile.py:806-845: register casts between the three kinds."""
    if want in FLOATS:
        if val.k == "f":
            return val
        if val.k == "i":
            return Val(np.asarray(val.v, dtype=np.int64).astype(np.float32), "f")   # cvt.rn
        return Val(np.asarray(val.v).astype(np.float32), "f")
    if want in ("bool", "bool8", "i1", "pred"):
        if val.k == "p":
            return val
        return Val(np.asarray(val.v) != 0, "p")
    # integer target
    if val.k == "i":
        return val
    if val.k == "p":
        return val                                               # a pred stays a pred (compile.py:816)
    with np.errstate(invalid="ignore"):
        return Val(_wrap(np.nan_to_num(np.trunc(np.asarray(val.v, np.float64)), nan=0.0,
                                       posinf=2**31 - 1, neginf=-2**31)), "i")    # cvt.rzi


class Interpreter:
    """Run one KernelOp of a graph over host numpy buffers.

    ``buffers`` maps every kernel argument name to a flat numpy array in storage format
    (``storage_dtype``); 16-bit floats are raw ``uint16`` bits.  Outputs are updated in place.
    """

    def __init__(self, graph, kernel_node=None) -> None:
        self.g = graph
        self.node = kernel_node if kernel_node is not None else graph.kernels()[0]
        self.op = self.node.op
        self.shapes: dict[str, tuple] = {}
        self.dtypes: dict[str, str] = {}
        for nd in graph.nodes.values():
            for v in nd.outputs:
                self.shapes[v.name] = tuple(int(x) for x in v.shape)
                self.dtypes[v.name] = _dt(v.dtype)
        self.smem_decl: dict[str, tuple] = {}
        self._collect_smem(self.op.body)
        self.seed_sets: dict[int, list] = {}
        self._plan_seeds()

    # -- static analyses ------------------------------------------------------------------

    def _collect_smem(self, body) -> None:
        """compile.py:492-504: every Smem is known before the first statement runs."""
        for st in body or ():
            if type(st).__name__ == "Smem":
                ext = tuple(int(getattr(x, "value", x)) for x in st.extents)
                self.smem_decl[st.name] = (ext, _dt(st.dtype))
            self._collect_smem(getattr(st, "body", None))
            self._collect_smem(getattr(st, "else_body", None))

    def _plan_seeds(self) -> None:
        """Which Accum names each loop seeds with their identity when control reaches it.

        compile.py:1296-1310 seeds, in front of a loop, every Accum directly in its body (not in a
        nested loop, compile.py:1319-1320) whose name was not yet bound in emission order.  That is
        a static property of statement order, so it is computed once here.
        """
        bound = {"lane", "warp"}

        def accums(body, out):
            for st in body:
                cls = type(st).__name__
                if cls == "Accum":
                    out.append(st)
                elif cls in ("StridedLoop", "Loop"):
                    continue
                else:
                    accums(getattr(st, "body", None) or (), out)
                    accums(getattr(st, "else_body", None) or (), out)
            return out

        def visit(body):
            for st in body or ():
                cls = type(st).__name__
                if cls in ("Loop", "StridedLoop"):
                    seeds = []
                    for a in accums(st.body, []):
                        if a.name not in bound and a.name not in [s.name for s in seeds]:
                            seeds.append(a)
                    for a in seeds:
                        bound.add(a.name)
                    self.seed_sets[id(st)] = seeds
                    bound.add(st.axis.name)
                    visit(st.body)
                    continue
                if cls == "Tile":
                    for ax in st.axes:
                        bound.add(ax.name)
                elif cls in ("Assign", "Let", "Init", "Select"):
                    bound.add(st.name)
                elif cls == "Load":
                    bound.update(st.names)
                elif cls in ("WarpShuffle", "TreeHalve"):
                    states = list(st.state)
                    others = list(getattr(st, "state_b", None) or ())
                    for i, nm in enumerate(states):
                        bound.add(others[i] if i < len(others) else f"{nm}__o")
                    for a in getattr(st, "combine_states", None) or ():
                        bound.add(a.name)
                visit(getattr(st, "body", None))
                visit(getattr(st, "else_body", None))

        visit(self.op.body)

    # -- running --------------------------------------------------------------------------

    def run(self, buffers: dict, grid: int, block: int, blocks=None, max_lanes: int = 1 << 20) -> None:
        """Execute blocks ``blocks`` (default: all of ``grid``) of ``block`` threads each."""
        self.buf = buffers
        for name, arr in buffers.items():
            if arr.ndim != 1:
                raise ValueError(f"buffer {name!r} must be flat")
        ids = np.arange(grid) if blocks is None else np.asarray(list(blocks))
        chunk = max(1, max_lanes // max(block, 1))
        self.T = block
        self.zeroed = set()
        for s in range(0, len(ids), chunk):
            self._run_chunk(ids[s:s + chunk], block)

    def _run_chunk(self, blk_ids: np.ndarray, T: int) -> None:
        nb = len(blk_ids)
        L = nb * T
        self.nb = nb
        self.blk = np.repeat(blk_ids.astype(np.int64), T)           # block id per lane
        self.bslot = np.repeat(np.arange(nb), T)                     # block slot within the chunk
        self.tid = np.tile(np.arange(T, dtype=np.int32), nb)
        self.gid = _wrap(self.blk * T + self.tid)
        self.lane_in_warp = self.tid & 31
        self.env: dict[str, Val] = {
            "lane": Val(self.tid & 31, "i"),                         # compile.py:558-563
            "warp": Val(self.tid >> 5, "i"),
        }
        self.smem = {}
        for name, (ext, dt) in self.smem_decl.items():
            n = int(np.prod(ext)) if ext else 1
            sd = _STORE[dt]
            fill = {np.float32: np.nan, np.float64: np.nan, np.uint16: 0x7FC1}.get(sd, -0x5A5A5A5B)
            self.smem[name] = np.full((nb, n), fill, dtype=sd)
        self.block(self.op.body, np.ones(L, dtype=bool))

    # -- statements -----------------------------------------------------------------------

    def block(self, body, mask) -> None:
        for st in body or ():
            getattr(self, "st_" + type(st).__name__)(st, mask)

    def st_Smem(self, st, mask) -> None:
        pass

    def st_Sync(self, st, mask) -> None:
        pass                                                         # lockstep: every write is visible

    def st_CpAsyncCommit(self, st, mask) -> None:
        pass

    def st_CpAsyncWait(self, st, mask) -> None:
        pass

    def st_Tile(self, st, mask) -> None:
        """compile.py:1135-1157: guard ``gid < ncells``, decode coordinates row major."""
        ext = [int(getattr(a.extent, "value", a.extent)) for a in st.axes]
        total = int(np.prod(ext))
        m = mask & (self.gid < total)
        rest = self.gid.astype(np.int64)
        for i, ax in enumerate(st.axes):
            inner = int(np.prod(ext[i + 1:])) if i + 1 < len(ext) else 1
            if i == len(ext) - 1:
                self.env[ax.name] = Val(_wrap(rest), "i")
            else:
                q = rest // inner
                self.env[ax.name] = Val(_wrap(q), "i")
                rest = rest - q * inner
        self.block(st.body, m)

    def st_Let(self, st, mask) -> None:
        """compile.py:1262-1274."""
        if type(st.value).__name__ == "FlatIndex":
            self.env[st.name] = Val(self.linear(st.value.buffer, st.value.index), "i")
            return
        self.env[st.name] = _cast(self.expr(st.value), _dt(st.dtype))

    def st_Init(self, st, mask) -> None:
        """compile.py:1276-1286: a register holding the identity."""
        dt = _dt(st.dtype)
        L = len(mask)
        if dt in FLOATS:
            self.env[st.name] = Val(np.full(L, float(st.identity), dtype=np.float32), "f")
        else:
            self.env[st.name] = Val(np.full(L, int(st.identity), dtype=np.int32), "i")

    def st_Assign(self, st, mask) -> None:
        """compile.py:1206-1227: elementwise op; bool results are predicates; 16-bit stays f32."""
        name = getattr(st.op, "name", None) or str(st.op)
        args = [self.value(a) for a in st.args]
        res = self.elementwise(name, args)
        want = _dt(st.dtype) if st.dtype is not None else None
        if want in ("bool", "bool8", "i1"):
            res = _cast(res, "pred")
        elif want is not None and want not in ("f16", "bf16"):
            if (res.k == "f") != (want in FLOATS):
                res = _cast(res, want)
        self.env[st.name] = res

    def st_Accum(self, st, mask) -> None:
        """compile.py:1328-1344: ``acc = op(base if base != name else acc, value)``."""
        name = getattr(st.op, "name", "") or str(st.op)
        acc = self.env[st.name]
        val = self.value(st.value)
        left = acc
        base = getattr(st, "base", None)
        if base is not None and base != st.name:
            left = self.value(base)
        if acc.k == "f":
            with np.errstate(all="ignore"):
                new = BINARY_F[name](np.asarray(left.v, np.float32), np.asarray(val.v, np.float32))
            new = np.asarray(new, dtype=np.float32)
        else:
            new = np.asarray(BINARY_I[name](left.v, val.v)).astype(np.int32)
        self.env[st.name] = Val(np.where(mask, new, acc.v), acc.k)

    def _seed(self, st) -> None:
        for a in self.seed_sets.get(id(st), ()):
            dt = _dt(a.dtype)
            op = a.op
            if getattr(op, "has_identity", False) and getattr(op, "identity", None) is not None:
                ident = op.identity
            else:
                ident = {"add": 0.0, "multiply": 1.0, "maximum": -math.inf,
                         "minimum": math.inf}.get(getattr(op, "name", ""), 0.0)   # compile.py:1288-1294
            L = len(self.gid)
            if dt in FLOATS:
                self.env[a.name] = Val(np.full(L, float(ident), dtype=np.float32), "f")
            else:
                self.env[a.name] = Val(np.full(L, int(ident), dtype=np.int32), "i")

    def _loop(self, st, mask, start, step, end) -> None:
        self._seed(st)
        L = len(mask)
        cur = np.broadcast_to(np.asarray(start, dtype=np.int64), (L,)).copy()
        end = np.broadcast_to(np.asarray(end, dtype=np.int64), (L,))
        step = np.broadcast_to(np.asarray(step, dtype=np.int64), (L,))
        name = st.axis.name
        while True:
            live = mask & (cur < end)
            if not live.any():
                break
            self.env[name] = Val(_wrap(cur), "i")
            self.block(st.body, live)
            cur = np.where(live, cur + step, cur)
        self.env[name] = Val(_wrap(cur), "i")

    def st_Loop(self, st, mask) -> None:
        """compile.py:1588-1618: counter 0..end (unrolling does not change the meaning)."""
        lim = st.end if st.end is not None else st.axis.extent
        self._loop(st, mask, 0, 1, self.ival(lim))

    def st_StridedLoop(self, st, mask) -> None:
        """compile.py:1552-1586: ``for v = start; v < end; v += step``."""
        lim = st.end if st.end is not None else st.axis.extent
        self._loop(st, mask, self.ival(st.start), self.ival(st.step), self.ival(lim))

    def st_Cond(self, st, mask) -> None:
        """compile.py:1480-1496."""
        p = _cast(self.expr(st.cond), "pred").v
        p = np.broadcast_to(p, mask.shape)
        self.block(st.body, mask & p)
        if st.else_body:
            self.block(st.else_body, mask & ~p)

    def st_Select(self, st, mask) -> None:
        """compile.py:1498-1520: first true branch wins; the last branch is the catch-all."""
        brs = list(st.branches)
        vals = [self.value(b.value) for b in brs]
        kind = vals[0].k
        L = len(mask)
        out = np.broadcast_to(np.asarray(_cast(vals[-1], "f32" if kind == "f" else "i32").v), (L,)).copy()
        for b, v in zip(reversed(brs[:-1]), reversed(vals[:-1])):
            p = np.broadcast_to(_cast(self.expr(b.select), "pred").v, (L,))
            vv = np.broadcast_to(np.asarray(v.v), (L,))
            out = np.where(p, vv, out)
        self.env[st.name] = Val(out.astype(np.float32 if kind == "f" else np.int32), kind)

    def st_Load(self, st, mask) -> None:
        """compile.py:1159-1204: n consecutive elements from the index onward."""
        buf = st.input
        if st.dtype is not None:
            dt = _dt(st.dtype)
        elif buf in self.smem_decl:
            dt = self.smem_decl[buf][1]
        else:
            dt = self.dtypes.get(buf, "f32")
        lin = np.broadcast_to(np.asarray(self.linear(buf, st.index), dtype=np.int64), mask.shape)
        for i, nm in enumerate(st.names):
            idx = lin + i
            if buf in self.smem:
                arr = self.smem[buf]
                safe = np.where(mask, idx, 0)
                raw = arr[self.bslot, np.clip(safe, 0, arr.shape[1] - 1)]
                bad = mask & ((safe < 0) | (safe >= arr.shape[1]))
            else:
                arr = self.buf[buf]
                safe = np.where(mask, idx, 0)
                raw = arr[np.clip(safe, 0, arr.size - 1)]
                bad = mask & ((safe < 0) | (safe >= arr.size))
            if bad.any():
                raise IndexError(f"Load from {buf!r} out of bounds at lane {int(np.argmax(bad))}")
            v = widen(raw, dt)
            self.env[nm] = Val(v, "f" if dt in FLOATS else "i")

    def st_Write(self, st, mask) -> None:
        """compile.py:1346-1382: one narrowing at the store; ``atomic`` is a reduction add."""
        out = st.output
        dt = _dt(st.value_dtype)
        lin = np.broadcast_to(np.asarray(self.linear(out, st.index), dtype=np.int64), mask.shape)
        shared = out in self.smem
        for i, nm in enumerate(st.values):
            val = self.env[nm]
            v = np.broadcast_to(np.asarray(val.v), mask.shape)
            idx = lin + i
            sel = np.nonzero(mask)[0]
            if shared:
                arr = self.smem[out]
                if len(sel) and ((idx[sel] < 0).any() or (idx[sel] >= arr.shape[1]).any()):
                    raise IndexError(f"Write to {out!r} out of bounds")
                if st.atomic:
                    np.add.at(arr, (self.bslot[sel], idx[sel]), v[sel].astype(arr.dtype))
                else:
                    arr[self.bslot[sel], idx[sel]] = narrow(v[sel], dt)
            else:
                arr = self.buf[out]
                if len(sel) and ((idx[sel] < 0).any() or (idx[sel] >= arr.size).any()):
                    raise IndexError(f"Write to {out!r} out of bounds")
                if st.atomic:
                    if dt in ("f16", "bf16", "f64"):
                        raise ValueError("atomic 16/64-bit write unsupported")    # compile.py:1359-1366
                    if dt == "f32":
                        np.add.at(arr, idx[sel], np.asarray(v[sel], np.float32))
                    else:
                        acc = arr.astype(np.int64)
                        np.add.at(acc, idx[sel], np.asarray(v[sel], np.int64))
                        arr[:] = _wrap(acc)
                else:
                    arr[idx[sel]] = narrow(v[sel], dt)

    def st_ZeroPrologue(self, st, mask) -> None:
        """compile.py:1401-1447: the grid zeroes ``words`` 32-bit words of ``dst``."""
        if st.dst in self.zeroed:
            return
        self.zeroed.add(st.dst)
        words = int(st.words or 0)
        arr = self.buf[st.dst]
        arr.view(np.uint8)[: words * 4] = 0

    def st_CpAsyncCopy(self, st, mask) -> None:
        """compile.py:1449-1471: dst = stripe base + the lane's (row, col); ``nbytes`` per lane."""
        if str(getattr(st, "swizzle", "NONE") or "NONE").upper() != "NONE":
            raise ValueError("swizzled cp.async is not part of the reference semantics")
        if getattr(st, "valid", None) is not None:
            raise ValueError("predicated cp.async is not part of the reference semantics")
        ext, sdt = self.smem_decl[st.smem]
        lin = np.asarray(self.linear(st.smem, st.smem_index), dtype=np.int64)
        if st.lane_index is not None:
            cols = ext[-1]
            l0 = np.asarray(self.ival(st.lane_index[0]), dtype=np.int64)
            l1 = np.asarray(self.ival(st.lane_index[1]), dtype=np.int64)
            lin = lin + l0 * cols + l1
        lin = np.broadcast_to(lin, mask.shape)
        src = np.broadcast_to(np.asarray(self.linear(st.src, st.src_index), dtype=np.int64), mask.shape)
        n = int(st.nbytes) // _BYTES[sdt]
        sel = np.nonzero(mask)[0]
        sm = self.smem[st.smem]
        g = self.buf[st.src]
        for i in range(n):
            d = lin[sel] + i
            s = src[sel] + i
            if (s < 0).any() or (s >= g.size).any() or (d < 0).any() or (d >= sm.shape[1]).any():
                raise IndexError("cp.async out of bounds")
            sm[self.bslot[sel], d] = g[s]

    def st_WarpShuffle(self, st, mask) -> None:
        """compile.py:1627-1654: butterfly all-reduce, or an inclusive scan with identity 0."""
        states = list(st.state)
        others = list(getattr(st, "state_b", None) or ())
        length = int(getattr(st, "length", 32) or 32)
        prefix = bool(getattr(st, "prefix", False))
        if self.T % 32:
            raise ValueError("warp shuffles need whole warps")
        lane = self.lane_in_warp
        base = np.arange(len(lane)) - lane
        off = 1 if prefix else length // 2
        while (off < length) if prefix else (off >= 1):
            for i, nm in enumerate(states):
                cur = self.env[nm]
                vals = np.broadcast_to(np.asarray(cur.v), mask.shape)
                if prefix:
                    src = lane - off
                    ok = src >= 0
                    got = vals[base + np.where(ok, src, lane)]
                    zero = np.zeros((), dtype=got.dtype)
                    got = np.where(ok, got, zero)
                else:
                    got = vals[base + (lane ^ off)]
                self.env[others[i] if i < len(others) else f"{nm}__o"] = Val(got, cur.k)
            for a in getattr(st, "combine_states", None) or ():
                self.st_Assign(a, mask)
            off = off * 2 if prefix else off // 2

    def st_WarpBroadcast(self, st, mask) -> None:
        """The last lane of each ``length``-lane group broadcast to its group (compile.py:1656-1668,
        which documents this meaning; its emitted ``shfl.idx`` only matches it for length 32)."""
        length = int(getattr(st, "length", 32) or 32)
        lane = self.lane_in_warp
        base = np.arange(len(lane)) - lane
        src = (lane & ~(length - 1)) | (length - 1)
        for nm in st.state:
            cur = self.env[nm]
            vals = np.broadcast_to(np.asarray(cur.v), mask.shape)
            self.env[nm] = Val(vals[base + src], cur.k)

    def st_TreeHalve(self, st, mask) -> None:
        """compile.py:1670-1708: halving tree over ``bufs[0:length]``; everyone reads ``bufs[0]``."""
        bufs = list(st.bufs)
        states = list(st.state)
        others = list(getattr(st, "state_b", None) or ())
        length = int(st.length)
        tid = getattr(st, "tid_var", "warp") or "warp"
        treg = self.env[tid] if tid in self.env else self.env["warp"]
        t = np.broadcast_to(np.asarray(treg.v, dtype=np.int64), mask.shape)
        s = length // 2
        while s >= 1:
            act = mask & (t < s)
            slots = []
            for i, (buf, nm) in enumerate(zip(bufs, states)):
                arr = self.smem[buf]
                ia = np.clip(np.where(act, t, 0), 0, arr.shape[1] - 1)
                ib = np.clip(np.where(act, t + s, 0), 0, arr.shape[1] - 1)
                a = widen(arr[self.bslot, ia], self.smem_decl[buf][1])
                b = widen(arr[self.bslot, ib], self.smem_decl[buf][1])
                kind = self.env[nm].k
                self.env[nm] = Val(a, kind)
                self.env[others[i] if i < len(others) else f"{nm}__o"] = Val(b, kind)
                slots.append((buf, nm, ia))
            for a in getattr(st, "combine_states", None) or ():
                self.st_Assign(a, act)
            sel = np.nonzero(act)[0]
            for buf, nm, ia in slots:
                arr = self.smem[buf]
                v = np.broadcast_to(np.asarray(self.env[nm].v), mask.shape)
                arr[self.bslot[sel], ia[sel]] = narrow(v[sel], self.smem_decl[buf][1])
            s //= 2
        for buf, nm in zip(bufs, states):
            arr = self.smem[buf]
            kind = self.env[nm].k
            self.env[nm] = Val(widen(arr[self.bslot, 0], self.smem_decl[buf][1]), kind)

    # -- expressions ----------------------------------------------------------------------

    def ival(self, e):
        """An integer operand (compile.py:580-592)."""
        if isinstance(e, bool):
            return int(e)
        if isinstance(e, int):
            return e
        if type(e).__name__ == "Dim":
            return int(e.value)
        if isinstance(e, str):
            return self.env[e].v
        v = self.expr(e)
        return _cast(v, "i32").v if v.k == "f" else v.v

    def linear(self, buf: str, index):
        """Row-major element offset of a coordinate list, exactly as compile.py:594-615."""
        shape = self.shapes[buf] if buf in self.shapes else self.smem_decl[buf][0]
        parts = list(index)
        if not parts:
            return 0
        if len(parts) == len(shape) and len(shape) > 1:
            acc = np.asarray(self.ival(parts[0]), dtype=np.int64)
            for i in range(1, len(parts)):
                if shape[i] == 1 and i == len(parts) - 1:
                    continue
                acc = acc * shape[i] + np.asarray(self.ival(parts[i]), dtype=np.int64)
            return _wrap(acc)
        if len(parts) == 1:
            return self.ival(parts[0])
        acc = np.asarray(self.ival(parts[0]), dtype=np.int64)
        for p in parts[1:]:
            acc = acc * shape[-1] + np.asarray(self.ival(p), dtype=np.int64)
        return _wrap(acc)

    def value(self, a) -> Val:
        """An SSA name or an expression (compile.py:1229-1237)."""
        if isinstance(a, str):
            if a in self.env:
                return self.env[a]
            raise KeyError(f"unknown SSA name {a!r}")
        return self.expr(a)

    def expr(self, e) -> Val:
        cls = type(e).__name__
        if cls == "Var":
            if e.name not in self.env:
                raise KeyError(f"unknown variable {e.name!r}")
            return self.env[e.name]
        if cls == "Literal":
            t = _dt(getattr(e, "dtype", "int"))
            if t in FLOATS:
                return Val(np.float32(float(e.value)), "f")
            return Val(np.int32(int(e.value)), "i")
        if cls == "Dim":
            return Val(np.int32(int(e.value)), "i")
        if isinstance(e, bool):
            return Val(np.int32(int(e)), "i")
        if isinstance(e, int):
            return Val(np.int32(e), "i")
        if isinstance(e, float):
            return Val(np.float32(e), "f")
        if cls == "BinaryExpr":
            return self.binary(e)
        if cls == "TernaryExpr":
            c = _cast(self.expr(e.cond), "pred").v
            a = self.expr(e.if_true)
            b = self.expr(e.if_false)
            kind = "f" if "f" in (a.k, b.k) else a.k
            if kind == "f":
                a, b = _cast(a, "f32"), _cast(b, "f32")
            return Val(np.where(c, a.v, b.v), kind)
        if cls == "FlatIndex":
            return Val(self.linear(e.buffer, e.index), "i")
        if cls == "CastExpr":
            return _cast(self.expr(e.expr), _dt(e.dtype))
        if cls == "Builtin":
            if e.name in ("threadIdx.x", "tid.x"):
                return Val(self.tid, "i")
            if e.name == "blockIdx.x":
                return Val(_wrap(self.blk), "i")
            raise ValueError(f"unsupported builtin {e.name!r}")
        if cls == "FuncCallExpr":
            return self.elementwise(e.name, [self.expr(a) for a in e.args])
        raise ValueError(f"unsupported expression {cls}")

    def binary(self, e) -> Val:
        """compile.py:744-798."""
        op = e.op
        lt = self.expr(e.left)
        rt = self.expr(e.right)
        if lt.k == "f" or rt.k == "f":
            a = _cast(lt, "f32").v
            b = _cast(rt, "f32").v
            if op in EXPR_F:
                with np.errstate(all="ignore"):
                    return Val(np.asarray(BINARY_F[EXPR_F[op]](a, b), np.float32), "f")
            if op in ("add", "subtract", "multiply", "divide", "maximum", "minimum"):
                with np.errstate(all="ignore"):
                    return Val(np.asarray(BINARY_F[op](a, b), np.float32), "f")
            if op in EXPR_CMP:
                return Val(EXPR_CMP[op](a, b), "p")
            raise ValueError(f"unsupported float binary op {op!r}")
        if op in EXPR_I:
            return Val(np.asarray(BINARY_I[EXPR_I[op]](lt.v, rt.v)).astype(np.int32), "i")
        if op in ("add", "subtract", "multiply", "divide", "modulo") or op in BINARY_I:
            return Val(np.asarray(BINARY_I[op](lt.v, rt.v)).astype(np.int32), "i")
        if op in EXPR_CMP:
            return Val(EXPR_CMP[op](lt.v, rt.v), "p")
        if op in ("&&", "and"):
            return Val(np.logical_and(lt.v, rt.v), "p")
        if op in ("||", "or"):
            return Val(np.logical_or(lt.v, rt.v), "p")
        raise ValueError(f"unsupported int binary op {op!r}")

    def elementwise(self, name: str, args: list) -> Val:
        """compile.py:863-978: numpy-ufunc-named ops on f32, s32 or predicates."""
        data = [a for a in args if a.k != "p"]
        kind = data[0].k if data else (args[0].k if args else "f")
        if name in COMPARE and len(args) == 2:
            if kind == "f":
                return Val(COMPARE[name](_cast(args[0], "f32").v, _cast(args[1], "f32").v), "p")
            return Val(COMPARE[name](args[0].v, args[1].v), "p")
        if name in ("logical_and", "logical_or") and len(args) == 2:
            a, b = _cast(args[0], "pred").v, _cast(args[1], "pred").v
            return Val(np.logical_and(a, b) if name == "logical_and" else np.logical_or(a, b), "p")
        if name == "logical_not" and len(args) == 1:
            return Val(np.logical_not(_cast(args[0], "pred").v), "p")
        if name in ("isnan", "isinf") and len(args) == 1:
            return Val((np.isnan if name == "isnan" else np.isinf)(args[0].v), "p")
        if name in ("copy", "bitcast") and len(args) == 1:
            return Val(args[0].v, kind)
        if kind != "f":
            if name in BINARY_I and len(args) == 2:
                return Val(np.asarray(BINARY_I[name](args[0].v, args[1].v)).astype(np.int32), "i")
            if len(args) == 1:
                un = {"negative": np.negative, "neg": np.negative, "absolute": np.abs, "abs": np.abs,
                      "bitwise_not": np.invert, "invert": np.invert}
                if name in un:
                    return Val(_wrap(un[name](np.asarray(args[0].v, np.int64))), "i")
                if name == "positive":
                    return args[0]
                if name == "square":
                    return Val(_wrap(np.asarray(args[0].v, np.int64) ** 2), "i")
            if name == "where" and len(args) == 3:
                return Val(np.where(_cast(args[0], "pred").v, args[1].v, args[2].v).astype(np.int32), "i")
            raise ValueError(f"unsupported int elementwise {name!r}")
        vals = [_cast(a, "f32").v if a.k != "p" else a.v for a in args]
        with np.errstate(all="ignore"):
            if name in ("where", "select") and len(args) == 3:
                return Val(np.where(_cast(args[0], "pred").v, vals[1], vals[2]).astype(np.float32), "f")
            if len(args) == 2 and name in BINARY_F:
                return Val(np.asarray(BINARY_F[name](vals[0], vals[1]), np.float32), "f")
            if len(args) == 1 and name in UNARY_F:
                return Val(np.asarray(UNARY_F[name](vals[0]), np.float32), "f")
        raise ValueError(f"unsupported elementwise op {name!r}")


def run_graph(graph, buffers: dict, grid: int, block: int, blocks=None) -> dict:
    """Interpret the graph's (single) kernel over ``buffers``; returns the same dict."""
    Interpreter(graph).run(buffers, grid, block, blocks=blocks)
    return buffers
