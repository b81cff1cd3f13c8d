"""Promotion of IR ``CpAsyncCopy`` stripes to TMA tile loads with an mbarrier per commit group.

The reference lowers every ``CpAsyncCopy`` to one ``cp.async`` per thread (compile.py:1449-1471): each
lane moves 16 (or 4 / 8) bytes of a stripe from global memory into its slot of a shared buffer, and
``CpAsyncCommit`` / ``CpAsyncWait(n)`` group and wait for them (compile.py:1473-1478).  When the lanes
of a block together copy one dense box — lane (r, c) moves the elements at source row origin_row + r,
columns origin_col + c .. + chunk-1, into shared row r, columns c .. — the whole stripe is a single
``cp.async.bulk.tensor`` issued by thread 0, completing on an mbarrier instead of a cp.async group.

:func:`plan` decides this for a kernel, for all of its copies or none:

* the block's threads are the Tile's last axis (its extent is the block size), every copy, commit
  and wait sits under block-uniform control flow, and the shared index does not depend on the thread;
* for every thread t of the block, under several random values of everything that is uniform
  (the other Tile axes and loop counters), the lane coordinates (r_t, c_t) and the source index are
  evaluated from the IR: the source index minus (0, .., r_t, c_t) must be the same for every thread
  (the box origin), thread 0 must have r = c = 0, and the lanes' chunks must cover the box
  [H rows, W columns] exactly once, with W the shared buffer's row length;
* TMA's rules: 1-256 rows and columns, W x element size a multiple of 16 bytes, source row strides
  a multiple of 16 bytes, 2-5 source dimensions, the same element type on both sides.

The emitter then proves the two alignments TMA needs from its affine forms (the origin column and the
shared offset are multiples of 16 bytes); if it cannot, it compiles the kernel again without the
promotion.  A wrong promotion can only give wrong data, never a fault: TMA fills coordinates outside
the tensor with zeros, and the shared destination is the IR's own buffer.
"""
from __future__ import annotations

import random
from dataclasses import dataclass

from ..ir import dim_int, dt_bytes, dt_name


class NotPromotable(Exception):
    """The kernel's copies stay cp.async (the reason is the message)."""


@dataclass
class StripePlan:
    """One promoted copy: TMA box ``[W, H, 1, ...]`` (innermost first) over ``src``."""

    src: str
    tmap: int                  # index into the kernel's tensor maps
    rows: int                  # H
    cols: int                  # W (elements)
    elem_bytes: int

    @property
    def box_bytes(self) -> int:
        return self.rows * self.cols * self.elem_bytes


def _trunc_div(a: int, b: int) -> int:
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


class _Eval:
    """Integer evaluation of IR index expressions (the truncating C semantics of compile.py:274-275)."""

    def __init__(self, lets: dict, env: dict):
        self.lets = lets
        self.env = env

    def __call__(self, e):
        if isinstance(e, bool):
            return int(e)
        if isinstance(e, int):
            return e
        if isinstance(e, float) and e == int(e):
            return int(e)
        if isinstance(e, str):
            return self.var(e)
        k = type(e).__name__
        if k == "Var":
            return self.var(e.name)
        if k == "Dim":
            return dim_int(e)
        if k == "Literal":
            v = e.value
            if isinstance(v, (int, bool)) or (isinstance(v, float) and v == int(v)):
                return int(v)
            raise NotPromotable(f"non-integer literal {v!r} in an index")
        if k == "BinaryExpr":
            a, b = self(e.left), self(e.right)
            op = e.op
            if op == "+":
                return a + b
            if op == "-":
                return a - b
            if op == "*":
                return a * b
            if op == "/":
                if b == 0:
                    raise NotPromotable("division by zero in an index")
                return _trunc_div(a, b)
            if op == "%":
                if b == 0:
                    raise NotPromotable("remainder by zero in an index")
                return a - _trunc_div(a, b) * b
            raise NotPromotable(f"operator {op!r} in an index")
        raise NotPromotable(f"{k} in an index")

    def var(self, name):
        if name in self.env:
            return self.env[name]
        if name in self.lets:
            v = self(self.lets[name])
            self.env[name] = v
            return v
        raise NotPromotable(f"index variable {name!r} not known")


def _names(e, out: set) -> set:
    """Variable names an expression reads."""
    if isinstance(e, str):
        out.add(e)
        return out
    k = type(e).__name__
    if k == "Var":
        out.add(e.name)
    elif k == "Builtin":
        out.add("%" + e.name)
    elif k == "BinaryExpr":
        _names(e.left, out)
        _names(e.right, out)
    elif k in ("TernaryExpr",):
        for f in ("cond", "if_true", "if_false"):
            _names(getattr(e, f), out)
    elif k in ("CastExpr",):
        _names(e.expr, out)
    elif k == "FuncCallExpr":
        for x in e.args:
            _names(x, out)
    return out


@dataclass
class _Site:
    st: object
    lets: dict
    uniform: dict              # uniform name -> (lo, hi) range for sampling


def plan(body, block: int | None, shapes: dict, dtypes: dict, smem: dict, samples: int = 3) -> dict | None:
    """The promotion plan of a kernel body: ``{"copies": {id(st): StripePlan}, "tmaps": [...],
    "nbar": N}``, or None when the kernel has no ``CpAsyncCopy`` or they must stay cp.async."""
    try:
        return _plan(body, block, shapes, dtypes, smem, samples)
    except NotPromotable:
        return None


def _plan(body, block, shapes, dtypes, smem, samples):
    tiles = [st for st in body if type(st).__name__ == "Tile"]
    copies_anywhere = []

    def find(stmts):
        for st in stmts or ():
            if type(st).__name__ == "CpAsyncCopy":
                copies_anywhere.append(st)
            find(getattr(st, "body", None))
            find(getattr(st, "else_body", None))
    find(body)
    if not copies_anywhere:
        return None
    if not block or len(tiles) != 1:
        raise NotPromotable("copies outside a single Tile, or no block size")
    tile = tiles[0]
    axes = list(tile.axes)
    if not axes or dim_int(axes[-1].extent) != block:
        raise NotPromotable("the Tile's last axis is not the block's threads")
    thread_axis = axes[-1].name
    uniform0 = {a.name: (0, dim_int(a.extent) - 1) for a in axes[:-1]}
    sites: list[_Site] = []
    waits: list[int] = []

    def thread_dep(e, lets, dep):
        for n in _names(e, set()):
            if n.startswith("%") or n in dep or n in ("lane", "warp"):
                return True
        return False

    def visit(stmts, lets, dep, uniform):
        lets = dict(lets)
        dep = set(dep)
        for st in stmts or ():
            k = type(st).__name__
            if k == "Let":
                lets[st.name] = st.value
                if thread_dep(st.value, lets, dep):
                    dep.add(st.name)
            elif k in ("Loop", "StridedLoop"):
                ax = st.axis
                ends = [getattr(st, f, None) for f in ("start", "step", "end")]
                loop_dep = any(x is not None and thread_dep(x, lets, dep) for x in ends)
                inner_dep = dep | ({ax.name} if loop_dep else set())
                u = dict(uniform)
                if not loop_dep:
                    u[ax.name] = (0, max(0, dim_int(ax.extent) - 1))
                visit(st.body, lets, inner_dep, u if not loop_dep else uniform)
                if loop_dep and _has_async(st.body):
                    raise NotPromotable("a copy under a thread-dependent loop")
            elif k == "Cond":
                if thread_dep(st.cond, lets, dep) and (_has_async(st.body) or _has_async(getattr(st, "else_body", None))):
                    raise NotPromotable("a copy under a thread-dependent condition")
                visit(st.body, lets, dep, uniform)
                visit(getattr(st, "else_body", None), lets, dep, uniform)
            elif k == "CpAsyncCopy":
                if any(thread_dep(x, lets, dep) for x in st.smem_index):
                    raise NotPromotable("a shared index that depends on the thread")
                sites.append(_Site(st, lets, dict(uniform)))
            elif k == "CpAsyncWait":
                waits.append(int(getattr(st, "group", 0) or 0))
            elif k in ("Tile",):
                raise NotPromotable("nested Tile")

    visit(tile.body, {}, {thread_axis}, uniform0)
    rng = random.Random(20250314)
    tmaps: list[dict] = []
    plans: dict[int, StripePlan] = {}
    for site in sites:
        st = site.st
        if str(getattr(st, "swizzle", "NONE") or "NONE").upper() != "NONE" or getattr(st, "valid", None) is not None:
            raise NotPromotable("a swizzled or predicated copy")
        lane = getattr(st, "lane_index", None)
        if lane is None or len(lane) != 2:
            raise NotPromotable("a copy without (row, column) lane coordinates")
        src = st.src
        if src not in shapes or st.smem not in smem:
            raise NotPromotable("unknown source or shared buffer")
        sdt = smem[st.smem][1]
        gdt = dtypes[src]
        es = dt_bytes(gdt)
        if dt_bytes(sdt) != es or dt_name(sdt) != dt_name(gdt):
            raise NotPromotable("source and shared buffer of different element types")
        nbytes = int(st.nbytes)
        if nbytes % es:
            raise NotPromotable("a chunk that is not whole elements")
        chunk = nbytes // es
        shape = shapes[src]
        if not 2 <= len(shape) <= 5 or len(st.src_index) != len(shape):
            raise NotPromotable("TMA takes 2-5 source dimensions")
        row_len = smem[st.smem][0][-1]
        box = None
        for s_ in range(samples):
            env = {name: rng.randint(lo, hi) for name, (lo, hi) in site.uniform.items()}
            origin = None
            cells = set()
            rows_seen = 0
            for t in range(block):
                ev = _Eval(site.lets, {**env, thread_axis: t})
                r, c = ev(lane[0]), ev(lane[1])
                sidx = [ev(x) for x in st.src_index]
                if t == 0 and (r != 0 or c != 0):
                    raise NotPromotable("thread 0 is not at the box origin")
                o = tuple(sidx[:-2]) + (sidx[-2] - r, sidx[-1] - c)
                if origin is None:
                    origin = o
                elif o != origin:
                    raise NotPromotable("the lanes do not copy one box")
                if r < 0 or c < 0 or c % chunk:
                    raise NotPromotable("a lane outside the box grid")
                key = (r, c // chunk)
                if key in cells:
                    raise NotPromotable("two lanes copy the same chunk")
                cells.add(key)
                rows_seen = max(rows_seen, r + 1)
            H = rows_seen
            W = (max(c for _, c in cells) + 1) * chunk
            if len(cells) != H * (W // chunk):
                raise NotPromotable("the lanes leave holes in the box")
            if box is None:
                box = (H, W)
            elif box != (H, W):
                raise NotPromotable("the box changes with the block")
        H, W = box
        if W != row_len:
            raise NotPromotable("the shared rows are wider than the box")
        if not (1 <= H <= 256 and 1 <= W <= 256) or (W * es) % 16:
            raise NotPromotable("the box breaks TMA's size rules")
        # byte strides of the source's dimensions 1.. counted from the innermost (TMA's order)
        strides = []
        acc = es
        for d in reversed(shape[1:]):
            acc *= d
            strides.append(acc)
        if any(s % 16 for s in strides):
            raise NotPromotable("a source row stride that is not a multiple of 16 bytes")
        spec = {"tensor": src, "dtype": dt_name(gdt), "dims": list(reversed(shape)), "strides": strides,
                "box": [W, H] + [1] * (len(shape) - 2), "swizzle": "none", "l2promo": 2}
        tm = next((i for i, t in enumerate(tmaps) if {k: v for k, v in t.items() if k != "name"} == spec), None)
        if tm is None:                             # one descriptor per (source, box)
            tm = len(tmaps)
            tmaps.append({"name": f"tm{tm}", **spec})
        plans[id(st)] = StripePlan(src, tm, H, W, es)
    return {"copies": plans, "tmaps": tmaps, "nbar": max(waits + [0]) + 1}


def _has_async(stmts) -> bool:
    for st in stmts or ():
        if type(st).__name__ in ("CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait"):
            return True
        if _has_async(getattr(st, "body", None)) or _has_async(getattr(st, "else_body", None)):
            return True
    return False
