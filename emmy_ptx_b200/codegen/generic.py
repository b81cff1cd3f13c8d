"""Statement-at-a-time lowering of one Emmy KernelOp to sm_100a PTX (the CUDA-core path).

Each IR construct has its own template (reference counterparts cited per method).  What is
B200-specific about it, compared with the reference's sm_89 emitter:

* global/shared traffic uses the widest vector the index *provably* allows — up to 256-bit
  ``ld.global.v8.b32`` on sm_100 — with 16-bit floats moved as packed ``b32`` words and
  widened/narrowed with bit operations / ``cvt.rn.bf16x2.f32`` instead of one ``ld.b16`` per
  element (compile.py:1178-1182, 1257-1260);
* read-only inputs go through the non-coherent path (``ld.global.nc``);
* integer index math is symbolic (:mod:`.affine`), so coordinates cancel, constants land in the
  address immediate and invariant address arithmetic is emitted in loop preheaders;
* ``WarpShuffle`` reductions whose combine is a single commutative op use ``redux.sync``;
  ``TreeHalve`` becomes one shared-memory read plus a butterfly over the warp (no per-level
  barriers), bit-identical to the halving tree for commutative combines;
* flat grid-stride loops are unrolled by four with a remainder loop so several 16/32-byte loads
  are in flight per thread; ``Select`` is a ``selp`` chain instead of a branch chain.
"""
from __future__ import annotations

import math
import os

from ..ir import dim_int, dt_name, dt_bytes, IRError, walk
from .affine import Affine, Atom, reg_atom, div_const, rem_const, recombine, INT_MAX
from .ptx import PtxBuilder, f32_imm
from . import mathlib

FLOATS = ("f16", "bf16", "f32", "f64")
INTS = ("i32", "int", "u32", "i64", "u64")
BOOLS = ("bool", "bool8", "i1", "u8", "i8")
LOG2E = 1.4426950408889634


class Unsupported(IRError):
    """The IR uses a construct this backend refuses (the reference raises SystemExit too)."""


class TmaNotProvable(Exception):
    """A promoted stripe's TMA alignment could not be proved: the kernel is built again with
    ``cp.async`` (``tma_stripes=False``)."""


TMA_BARS = "__tmabar"                # the shared mbarriers of the promoted commit groups
TMA_WAIT_LIMIT = 40000               # bounded try_wait polls with a 0.1 ms hint: < ~4 s
TMA_WAIT_HINT_NS = 100000
ERR_TMA_WAIT = 41                    # status word: a commit group's TMA loads never completed


class Sym:
    """A bound IR value: ``f32`` (operand string), ``pred`` (register) or ``s32`` (Affine)."""

    __slots__ = ("kind", "op", "aff")

    def __init__(self, kind: str, op: str | None = None, aff: Affine | None = None):
        self.kind = kind
        self.op = op
        self.aff = aff

    def __repr__(self):
        return f"Sym({self.kind}, {self.op if self.aff is None else self.aff})"


def _wrap32(v: int) -> int:
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= (1 << 31) else v


class KernelEmitter:
    """Lower one KernelOp.  ``kmeta`` is its ``meta.json`` kernel record (may be None)."""

    def __init__(self, graph, node, kmeta: dict | None = None, prefix: str = "", options: dict | None = None):
        self.g = graph
        self.node = node
        self.op = node.op
        self.name = self.op.name
        self.kmeta = kmeta or {}
        self.prefix = prefix
        self.opts = dict(options or {})
        self.b = PtxBuilder()
        self.syms: dict[str, Sym] = {}
        self.shapes: dict[str, tuple] = {}
        self.dtypes: dict[str, str] = {}
        self.smem: dict[str, tuple] = {}         # name -> (extents, dtype, align)
        self.smem_off: dict[str, int] = {}
        self.params: list[str] = []
        self.preg: dict[str, str] = {}           # param -> b64 global base register
        self.palign: dict[str, int] = {}         # param -> base alignment the code relies on
        self.sbase: dict[str, str] = {}          # smem buffer -> b32 shared-window base register
        self.written: set[str] = set()
        self.dyn_smem = 0
        # programmatic dependent launch is opt-in: on the benchmark kernels it measured no better
        # than plain stream order, and slower for the one-wave softmax
        self.pdl = bool(self.opts.get("pdl", os.environ.get("EMMY_B200_PDL", "0") == "1"))
        self.uses_tid_const = False

    # ---- set-up (compile.py:476-519) ---------------------------------------------------
    def prepare(self) -> None:
        for nd in self.g.nodes.values():
            for v in nd.outputs:
                self.shapes[v.name] = tuple(int(x) for x in v.shape)
                self.dtypes[v.name] = dt_name(v.dtype)
        order = list(self.node.inputs) + [v.name for v in self.node.outputs]
        self.params = list(self.kmeta.get("arg_order", order))
        self._scan(self.op.body)
        block = self.kmeta.get("block") or []
        grid = self.kmeta.get("grid") or []
        self.T = int(block[0]) if block and not os.environ.get("PTX_NO_MAXNTID") else None
        if block and len(block) > 1 and any(int(x) != 1 for x in block[1:]):
            self.T = None                      # 2-D/3-D blocks: keep %ntid.x
        self.G = int(grid[0]) if grid else None
        if grid and len(grid) > 1 and any(int(x) != 1 for x in grid[1:]):
            self.G = None
        self.exchange = self.opts.get("exchange")
        if self.exchange:
            # the multi-GPU sum's exchange as this kernel's epilogue (kernels/peer_sum.py): it needs the
            # grid size (the block that finishes last runs it) and the one-element partial to publish
            x = self.exchange
            if not self.G or not self.T:
                raise Unsupported("the fused exchange needs a 1-D grid and block from the launch meta")
            if x.get("partial") not in self.params or self.shapes.get(x["partial"], (0,)) not in ((1,), ()):
                raise Unsupported(f"the fused exchange needs a one-element output, not {x.get('partial')!r}")
            if x.get("dtype") not in ("f32", "i32") or dt_name(self.dtypes[x["partial"]]) != x["dtype"]:
                raise Unsupported("the fused exchange adds an f32 or i32 partial of the output's type")
        # outputs that accumulate in a scratch the kernel zeroes itself (option ``self_zeroing``; the
        # fused exchange's partial always does): see _last_block_epilogue
        self.acc_outs: dict[str, int] = {}
        if self.opts.get("self_zeroing") or self.exchange:
            self.acc_outs = self._self_zeroing_outputs()
            if self.exchange and self.exchange["partial"] not in self.acc_outs:
                raise Unsupported("the fused exchange needs a partial that only atomic adds write")
        self.err = None
        self.tma = None
        if self.opts.get("tma_stripes", True) is not False and self.T:
            from . import tma_stripes
            self.tma = tma_stripes.plan(self.op.body, self.T, self.shapes, self.dtypes, self.smem)
            if self.tma is not None:
                # one 8-byte mbarrier per commit group that can be in flight
                self.smem[TMA_BARS] = ((2 * self.tma["nbar"],), "i32", 16)
        self._plan_smem()

    def _self_zeroing_outputs(self) -> dict:
        """Byte offsets in the accumulator scratch of the outputs that can skip the zeroing before the
        launch: listed in ``zero_outputs``, written only by atomic adds (scalar 32-bit, the only atomic
        writes the emitter makes), never read by the kernel, at most 32 elements (warp 0 of the last
        block moves them), and a 1-D launch whose grid size is known.  Word 0 of the scratch is the
        block ticket; the accumulators start at byte 16, each 16-byte aligned."""
        if not self.G or not self.T:
            return {}
        cand = [n for n in (self.kmeta.get("zero_outputs") or []) if n in self.params]
        stmts = []
        walk(self.op.body, stmts.append)
        out_of = set()                           # outputs some statement disqualifies
        for st in stmts:
            cls = type(st).__name__
            if cls == "Write" and not getattr(st, "atomic", False):
                out_of.add(st.output)
            elif cls == "Load":
                out_of.add(st.input)
            elif cls == "CpAsyncCopy":
                out_of.add(st.src)
        out, off = {}, 16
        for n in (c for c in cand if c not in out_of):
            elems = 1
            for x in self.shapes.get(n, (0,)):
                elems *= int(x)
            if not 1 <= elems <= 32 or dt_name(self.dtypes[n]) not in ("f32", "i32", "u32"):
                continue
            out[n] = off
            off += (4 * elems + 15) // 16 * 16
        return out

    def _scan(self, body) -> None:
        for st in body or ():
            cls = type(st).__name__
            if cls == "Smem":
                ext = tuple(dim_int(x) for x in st.extents)
                self.smem[st.name] = (ext, dt_name(st.dtype), int(getattr(st, "align", 0) or 0))
            elif cls == "Write":
                self.written.add(st.output)
            elif cls == "ZeroPrologue":
                self.written.add(st.dst)
            self._scan(getattr(st, "body", None))
            self._scan(getattr(st, "else_body", None))

    def _plan_smem(self) -> None:
        """Byte layout of every shared buffer: each aligned to max(align, 16) — 1024 when the
        buffer is large enough to be a swizzled tensor-core operand — with one dynamic pool when
        the total passes the 48 KiB static limit (compile.py:506-519, 1739-1747).  Sizes are
        exact bytes per dtype (the reference declares 16-bit buffers as 32-bit elements)."""
        off = 0
        for name, (ext, dt, align) in self.smem.items():
            n = 1
            for e in ext:
                n *= e
            nbytes = n * dt_bytes(dt)
            al = max(align or 0, 16)
            off = (off + al - 1) // al * al
            self.smem_off[name] = off
            off += nbytes
        self.smem_total = off
        if off > 227 * 1024:
            raise Unsupported(f"shared memory {off} B exceeds the 227 KiB per-block limit of sm_100")
        self.dyn = off > 48 * 1024
        self.dyn_smem = off if self.dyn else 0

    def sym_name(self, s: str) -> str:
        return f"{self.prefix}{s}"

    # ---- prologue (compile.py:542-577) -------------------------------------------------
    def prologue(self) -> None:
        b = self.b
        for name in self.params:
            r = b.reg("b64")
            b.emit(f"ld.param.u64 {r}, [p_{name}];")
            b.emit(f"cvta.to.global.u64 {r}, {r};")
            self.preg[name] = r
            self.palign[name] = 16
        if self.pdl:
            # programmatic dependent launch: this grid may be scheduled while the previous kernel
            # in the stream is still running; wait for it (and its memory) before the first global
            # access, then let the next kernel's grid be scheduled onto SMs as they free up
            b.emit("griddepcontrol.wait;")
            b.emit("griddepcontrol.launch_dependents;")
        tid = b.reg("b32")
        b.emit(f"mov.u32 {tid}, %tid.x;")
        ctaid = b.reg("b32")
        b.emit(f"mov.u32 {ctaid}, %ctaid.x;")
        T = self.T
        gmax = (self.G - 1) if self.G else INT_MAX
        if T:
            self.tid = Affine.of(reg_atom(tid, 0, T - 1))
            self.ctaid = Affine.of(reg_atom(ctaid, 0, gmax))
            self.gid = self.ctaid.scale(T) + self.tid
        else:
            ntid = b.reg("b32")
            b.emit(f"mov.u32 {ntid}, %ntid.x;")
            gid = b.reg("b32")
            b.emit(f"mad.lo.s32 {gid}, {ctaid}, {ntid}, {tid};")
            self.tid = Affine.of(reg_atom(tid, 0, 1023))
            self.ctaid = Affine.of(reg_atom(ctaid, 0, gmax))
            self.gid = Affine.of(reg_atom(gid, 0, INT_MAX))
        self.syms["lane"] = Sym("s32", aff=rem_const(self.tid, 32))
        self.syms["warp"] = Sym("s32", aff=div_const(self.tid, 32))
        # shared bases once, in the prologue: a base first taken inside a divergent branch would
        # be undefined on the threads that skipped it (README.md:45-47, compile.py:564-577)
        for name in self.smem:
            r = b.reg("b32")
            if self.dyn:
                b.emit(f"mov.u32 {r}, {self.sym_name('smem_pool')};")
                if self.smem_off[name]:
                    b.emit(f"add.u32 {r}, {r}, {self.smem_off[name]};")
            else:
                b.emit(f"mov.u32 {r}, {self.sym_name(name)};")
            self.sbase[name] = r
        if self.tma is not None:
            self._tma_prologue(tid)
        if self.exchange:
            self.xch, self.peers = b.reg("b64"), b.reg("b64")
            for r, nm in ((self.xch, "p_xch"), (self.peers, "p_peers")):
                b.emit(f"ld.param.u64 {r}, [{nm}];")
                b.emit(f"cvta.to.global.u64 {r}, {r};")
            if self.err is None:
                self.err = b.reg("b64")
                b.emit(f"ld.param.u64 {self.err}, [p_err];")
                b.emit(f"cvta.to.global.u64 {self.err}, {self.err};")
        if self.acc_outs:
            # the atomic adds of these outputs go to their accumulators in the scratch; the output
            # pointers are kept for the last block's stores
            self.acc = b.reg("b64")
            b.emit(f"ld.param.u64 {self.acc}, [p_acc];")
            b.emit(f"cvta.to.global.u64 {self.acc}, {self.acc};")
            self.real_out = {}
            for n, off in self.acc_outs.items():
                r = b.reg("b64")
                b.emit(f"add.s64 {r}, {self.acc}, {off};")
                self.real_out[n] = self.preg[n]
                self.preg[n] = r
                self.palign[n] = 16
            self.tid_reg = tid

    # ---- integers -------------------------------------------------------------------------
    def mat(self, aff) -> str:
        """An integer operand: an immediate, or a register holding the affine value."""
        if isinstance(aff, int):
            return str(_wrap32(aff))
        if aff.is_const():
            return str(_wrap32(aff.c))
        a = aff.single_atom()
        if a is not None:
            return self.mat_atom(a)
        key = ("aff", aff.key)
        mutable = aff.mutable()
        if not mutable:
            hit = self.b.lookup(key)
            if hit is not None:
                return hit
        depth = None if mutable else aff.depth()
        terms = sorted(aff.terms.items(), key=lambda t: (t[1] < 0, repr(t[0].key)))
        acc = None
        for atom, k in terms:
            x = self.mat_atom(atom)
            if acc is None:
                if k == 1:
                    acc = x
                    continue
                r = self.b.reg("b32")
                if k == -1:
                    self.b.emit(f"neg.s32 {r}, {x};", depth)
                else:
                    self.b.emit(f"mul.lo.s32 {r}, {x}, {_wrap32(k)};", depth)
                acc = r
                continue
            r = self.b.reg("b32")
            if k == 1:
                self.b.emit(f"add.s32 {r}, {acc}, {x};", depth)
            elif k == -1:
                self.b.emit(f"sub.s32 {r}, {acc}, {x};", depth)
            else:
                self.b.emit(f"mad.lo.s32 {r}, {x}, {_wrap32(k)}, {acc};", depth)
            acc = r
        if aff.c:
            r = self.b.reg("b32")
            self.b.emit(f"add.s32 {r}, {acc}, {_wrap32(aff.c)};", depth)
            acc = r
        if not mutable:
            self.b.remember(key, acc, depth)
        return acc

    def mat_atom(self, a: Atom) -> str:
        if a.kind == "reg":
            return a.reg
        key = ("atom", a.key)
        if not a.mutable:
            hit = self.b.lookup(key)
            if hit is not None:
                return hit
        depth = None if a.mutable else a.depth
        num = self.mat(a.num)
        r = self.b.reg("b32")
        pow2 = a.d & (a.d - 1) == 0
        nn = a.num.nonneg()
        if a.kind == "div":
            if nn and pow2:
                self.b.emit(f"shr.u32 {r}, {num}, {a.d.bit_length() - 1};", depth)
            elif nn:
                self.b.emit(f"div.u32 {r}, {num}, {a.d};", depth)
            else:
                self.b.emit(f"div.s32 {r}, {num}, {a.d};", depth)
        else:
            if nn and pow2:
                self.b.emit(f"and.b32 {r}, {num}, {a.d - 1};", depth)
            elif nn:
                self.b.emit(f"rem.u32 {r}, {num}, {a.d};", depth)
            else:
                self.b.emit(f"rem.s32 {r}, {num}, {a.d};", depth)
        if not a.mutable:
            self.b.remember(key, r, depth)
        return r

    def reg_of(self, aff: Affine) -> str:
        """Like :meth:`mat` but always a register (for operands that cannot be immediates)."""
        x = self.mat(aff)
        if x.startswith("%"):
            return x
        r = self.b.reg("b32")
        self.b.emit(f"mov.b32 {r}, {x};")
        return r

    def new_int(self, reg: str, lo=None, hi=None, mutable=False) -> Affine:
        return Affine.of(reg_atom(reg, lo, hi, depth=self.b.depth, mutable=mutable))

    # ---- operand access ------------------------------------------------------------------
    def ival(self, e) -> Affine:
        """An integer operand as an affine form (compile.py:580-592)."""
        if isinstance(e, bool):
            return Affine.const(int(e))
        if isinstance(e, int):
            return Affine.const(e)
        if type(e).__name__ == "Dim":
            return Affine.const(dim_int(e))
        if isinstance(e, Affine):
            return e
        s = self.value(e) if isinstance(e, str) else self.expr(e)
        return self.to_int(s)

    def to_int(self, s: Sym) -> Affine:
        if s.kind == "s32":
            return s.aff
        if s.kind == "pred":
            r = self.b.reg("b32")
            self.b.emit(f"selp.b32 {r}, 1, 0, {s.op};")
            return self.new_int(r, 0, 1)
        if s.kind == "f32":
            r = self.b.reg("b32")
            self.b.emit(f"cvt.rzi.s32.f32 {r}, {s.op};")
            return self.new_int(r)
        raise Unsupported(f"cannot use {s.kind} as an integer")

    def to_f32(self, s: Sym) -> str:
        if s.kind == "f32":
            return s.op
        if s.kind == "s32":
            if s.aff.is_const():
                return f32_imm(float(s.aff.c))
            r = self.b.reg("f32")
            self.b.emit(f"cvt.rn.f32.s32 {r}, {self.mat(s.aff)};")
            return r
        if s.kind == "pred":
            r = self.b.reg("f32")
            self.b.emit(f"selp.f32 {r}, 0f3F800000, 0f00000000, {s.op};")
            return r
        raise Unsupported(f"cannot use {s.kind} as f32")

    def to_pred(self, s: Sym) -> str:
        if s.kind == "pred":
            return s.op
        p = self.b.reg("pred")
        if s.kind == "f32":
            self.b.emit(f"setp.ne.f32 {p}, {s.op}, 0f00000000;")
        else:
            self.b.emit(f"setp.ne.s32 {p}, {self.reg_of(s.aff)}, 0;")
        return p

    def freg(self, op: str) -> str:
        """An f32 operand in a register (for instructions that take no immediate)."""
        if op.startswith("%"):
            return op
        r = self.b.reg("f32")
        self.b.emit(f"mov.b32 {r}, {op};")
        return r

    def value(self, a) -> Sym:
        """An SSA name or an expression (compile.py:1229-1237)."""
        if isinstance(a, str):
            s = self.syms.get(a)
            if s is None:
                raise Unsupported(f"unknown SSA name {a!r}")
            return s
        return self.expr(a)

    # ---- expressions (compile.py:682-855) --------------------------------------------------
    def expr(self, e) -> Sym:
        cls = type(e).__name__
        if cls == "Var":
            s = self.syms.get(e.name)
            if s is None:
                raise Unsupported(f"unknown variable {e.name!r}")
            return s
        if cls == "Literal":
            t = dt_name(getattr(e, "dtype", "int"))
            if t in FLOATS:
                return Sym("f32", op=f32_imm(float(e.value)))
            if t in BOOLS and t != "u8":
                p = self.b.reg("pred")
                self.b.emit(f"setp.ne.s32 {p}, {1 if e.value else 0}, 0;")
                return Sym("pred", op=p)
            return Sym("s32", aff=Affine.const(int(e.value)))
        if cls == "Dim":
            return Sym("s32", aff=Affine.const(dim_int(e)))
        if isinstance(e, bool):
            return Sym("s32", aff=Affine.const(int(e)))
        if isinstance(e, int):
            return Sym("s32", aff=Affine.const(e))
        if isinstance(e, float):
            return Sym("f32", op=f32_imm(e))
        if cls == "BinaryExpr":
            return self.binary(e.op, self.expr(e.left), self.expr(e.right))
        if cls == "TernaryExpr":
            c = self.to_pred(self.expr(e.cond))
            a = self.expr(e.if_true)
            b = self.expr(e.if_false)
            return self.select(c, a, b)
        if cls == "FlatIndex":
            return Sym("s32", aff=self.linear(e.buffer, e.index))
        if cls == "CastExpr":
            return self.cast(self.expr(e.expr), dt_name(e.dtype))
        if cls == "Builtin":
            if e.name in ("threadIdx.x", "tid.x"):
                return Sym("s32", aff=self.tid)
            if e.name in ("blockIdx.x", "ctaid.x"):
                return Sym("s32", aff=self.ctaid)
            raise Unsupported(f"unsupported builtin {e.name!r}")
        if cls == "FuncCallExpr":
            return self.elementwise(e.name, [self.expr(a) for a in e.args])
        raise Unsupported(f"unsupported expression {cls}")

    def select(self, p: str, a: Sym, b: Sym) -> Sym:
        if a.kind == "f32" or b.kind == "f32":
            r = self.b.reg("f32")
            self.b.emit(f"selp.f32 {r}, {self.to_f32(a)}, {self.to_f32(b)}, {p};")
            return Sym("f32", op=r)
        if a.kind == "pred" and b.kind == "pred":
            r = self.b.reg("pred")
            t1, t2 = self.b.reg("pred"), self.b.reg("pred")
            self.b.emit(f"and.pred {t1}, {p}, {a.op};")
            self.b.emit(f"not.pred {t2}, {p};")
            self.b.emit(f"and.pred {t2}, {t2}, {b.op};")
            self.b.emit(f"or.pred {r}, {t1}, {t2};")
            return Sym("pred", op=r)
        r = self.b.reg("b32")
        self.b.emit(f"selp.b32 {r}, {self.mat(self.to_int(a))}, {self.mat(self.to_int(b))}, {p};")
        return Sym("s32", aff=self.new_int(r))

    _CMP = {"==": "eq", "!=": "ne", "<": "lt", "<=": "le", ">": "gt", ">=": "ge"}
    _SWAP = {"eq": "eq", "ne": "ne", "lt": "gt", "le": "ge", "gt": "lt", "ge": "le"}

    def compare(self, cmp: str, a: Sym, b: Sym, isfloat: bool) -> Sym:
        p = self.b.reg("pred")
        if isfloat:
            x, y = self.to_f32(a), self.to_f32(b)
            if not x.startswith("%"):
                x, y, cmp = y, x, self._SWAP[cmp]
            self.b.emit(f"setp.{cmp}.f32 {p}, {self.freg(x)}, {y};")
            return Sym("pred", op=p)
        ia, ib = self.to_int(a), self.to_int(b)
        if ia.is_const() and ib.is_const():
            v = {"eq": ia.c == ib.c, "ne": ia.c != ib.c, "lt": ia.c < ib.c, "le": ia.c <= ib.c,
                 "gt": ia.c > ib.c, "ge": ia.c >= ib.c}[cmp]
            self.b.emit(f"setp.ne.s32 {p}, {1 if v else 0}, 0;")
            return Sym("pred", op=p)
        if ia.is_const():
            ia, ib, cmp = ib, ia, self._SWAP[cmp]
        self.b.emit(f"setp.{cmp}.s32 {p}, {self.reg_of(ia)}, {self.mat(ib)};")
        return Sym("pred", op=p)

    def binary(self, op: str, lt: Sym, rt: Sym) -> Sym:
        """compile.py:744-798: float if either side is float, else integer / predicate."""
        if lt.kind == "f32" or rt.kind == "f32":
            fop = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide"}.get(op, op)
            if fop in ("add", "subtract", "multiply", "divide", "maximum", "minimum"):
                return self.fbin(fop, self.to_f32(lt), self.to_f32(rt))
            if op in self._CMP:
                return self.compare(self._CMP[op], lt, rt, True)
            raise Unsupported(f"unsupported float binary op {op!r}")
        if op in self._CMP:
            return self.compare(self._CMP[op], lt, rt, False)
        if op in ("&&", "and", "||", "or") and (lt.kind == "pred" or rt.kind == "pred"):
            p = self.b.reg("pred")
            ins = "and" if op in ("&&", "and") else "or"
            self.b.emit(f"{ins}.pred {p}, {self.to_pred(lt)}, {self.to_pred(rt)};")
            return Sym("pred", op=p)
        iop = {"+": "add", "-": "subtract", "*": "multiply", "/": "divide", "%": "modulo",
               "&": "bitwise_and", "|": "bitwise_or", "^": "bitwise_xor", "<<": "left_shift",
               ">>": "right_shift", "&&": "bitwise_and", "||": "bitwise_or"}.get(op, op)
        return self.ibin(iop, self.to_int(lt), self.to_int(rt))

    def ibin(self, op: str, a: Affine, b: Affine) -> Sym:
        """Integer ops: affine where exact, one instruction otherwise (compile.py:87-125, 266-335)."""
        if op == "add":
            return Sym("s32", aff=a + b)
        if op == "subtract":
            return Sym("s32", aff=a - b)
        if op == "multiply":
            if b.is_const():
                return Sym("s32", aff=a.scale(b.c))
            if a.is_const():
                return Sym("s32", aff=b.scale(a.c))
        if op in ("divide",) and b.is_const() and b.c > 0:
            return Sym("s32", aff=div_const(a, b.c))
        if op in ("modulo", "remainder", "fmod") and b.is_const() and b.c > 0:
            return Sym("s32", aff=rem_const(a, b.c))
        if op == "left_shift" and b.is_const() and 0 <= b.c < 31:
            return Sym("s32", aff=a.scale(1 << b.c))
        if op == "right_shift" and b.is_const() and a.nonneg() and 0 <= b.c < 31:
            return Sym("s32", aff=div_const(a, 1 << b.c))
        if op == "bitwise_and" and b.is_const() and a.nonneg() and b.c > 0 and (b.c + 1) & b.c == 0:
            return Sym("s32", aff=rem_const(a, b.c + 1))
        if a.is_const() and b.is_const():
            x, y = a.c, b.c
            fold = {"multiply": lambda: x * y, "bitwise_and": lambda: x & y, "bitwise_or": lambda: x | y,
                    "bitwise_xor": lambda: x ^ y, "maximum": lambda: max(x, y), "minimum": lambda: min(x, y),
                    "left_shift": lambda: x << y, "right_shift": lambda: x >> y}
            if op in fold:
                return Sym("s32", aff=Affine.const(_wrap32(fold[op]())))
        ins = {"multiply": "mul.lo.s32", "divide": "div.s32", "modulo": "rem.s32", "remainder": "rem.s32",
               "fmod": "rem.s32", "maximum": "max.s32", "minimum": "min.s32", "bitwise_and": "and.b32",
               "bitwise_or": "or.b32", "bitwise_xor": "xor.b32", "and": "and.b32", "or": "or.b32",
               "xor": "xor.b32", "left_shift": "shl.b32", "right_shift": "shr.s32"}.get(op)
        if ins is None:
            raise Unsupported(f"unsupported int op {op!r}")
        r = self.b.reg("b32")
        self.b.emit(f"{ins} {r}, {self.reg_of(a)}, {self.mat(b)};")
        return Sym("s32", aff=self.new_int(r))

    def fbin(self, op: str, x: str, y: str) -> Sym:
        ins = {"add": "add.f32", "subtract": "sub.f32", "multiply": "mul.f32", "divide": "div.rn.f32",
               "maximum": "max.f32", "minimum": "min.f32"}[op]
        if op == "divide" and self.opts.get("fast_div"):
            ins = "div.full.f32"       # option: the 2-ulp division instead of IEEE round-to-nearest
        r = self.b.reg("f32")
        if not x.startswith("%") and not y.startswith("%"):
            x = self.freg(x)
        elif not x.startswith("%"):
            if op in ("add", "multiply", "maximum", "minimum"):
                x, y = y, x
            else:
                x = self.freg(x)
        self.b.emit(f"{ins} {r}, {x}, {y};")
        return Sym("f32", op=r)

    def cast(self, s: Sym, want: str) -> Sym:
        """compile.py:806-845."""
        if want in FLOATS:
            if s.kind == "f32":
                return s
            return Sym("f32", op=self.to_f32(s))
        if want in BOOLS + ("pred",):
            if s.kind == "pred":
                return s
            if want == "u8" or want == "i8":
                return Sym("s32", aff=self.to_int(s))
            return Sym("pred", op=self.to_pred(s))
        if want in INTS:
            if s.kind == "pred":
                return s                  # a predicate bound to an int name stays a predicate (compile.py:816)
            return Sym("s32", aff=self.to_int(s))
        raise Unsupported(f"unsupported cast {s.kind} -> {want}")

    def elementwise(self, name: str, args: list[Sym]) -> Sym:
        """numpy-ufunc-named elementwise ops (compile.py:863-978)."""
        data = [a for a in args if a.kind != "pred"]
        isfloat = (data[0].kind == "f32") if data else False
        if name in mathlib.COMPARISONS and len(args) == 2:
            return self.compare(mathlib.COMPARISONS[name], args[0], args[1], isfloat)
        if name in ("logical_and", "logical_or") and len(args) == 2:
            p = self.b.reg("pred")
            self.b.emit(f"{'and' if name == 'logical_and' else 'or'}.pred {p}, "
                        f"{self.to_pred(args[0])}, {self.to_pred(args[1])};")
            return Sym("pred", op=p)
        if name == "logical_not" and len(args) == 1:
            p = self.b.reg("pred")
            self.b.emit(f"not.pred {p}, {self.to_pred(args[0])};")
            return Sym("pred", op=p)
        if name in ("isnan", "isinf") and len(args) == 1:
            p = self.b.reg("pred")
            self.b.emit(f"testp.{'notanumber' if name == 'isnan' else 'infinite'}.f32 {p}, "
                        f"{self.freg(self.to_f32(args[0]))};")
            return Sym("pred", op=p)
        if name in ("copy", "bitcast", "positive") and len(args) == 1:
            return args[0]
        if name in ("where", "select") and len(args) == 3:
            return self.select(self.to_pred(args[0]), args[1], args[2])
        if not isfloat:
            if len(args) == 2:
                return self.ibin(name, self.to_int(args[0]), self.to_int(args[1]))
            if len(args) == 1:
                a = self.to_int(args[0])
                if name in ("negative", "neg"):
                    return Sym("s32", aff=-a)
                if name == "square":
                    return self.ibin("multiply", a, a) if not a.is_const() else Sym("s32", aff=Affine.const(a.c * a.c))
                ins = {"absolute": "abs.s32", "abs": "abs.s32", "bitwise_not": "not.b32", "invert": "not.b32"}.get(name)
                if ins:
                    r = self.b.reg("b32")
                    self.b.emit(f"{ins} {r}, {self.reg_of(a)};")
                    return Sym("s32", aff=self.new_int(r))
            raise Unsupported(f"unsupported int elementwise {name!r}")
        xs = [self.to_f32(a) for a in args]
        if len(xs) == 2 and name in ("add", "subtract", "multiply", "divide", "maximum", "minimum"):
            return self.fbin(name, xs[0], xs[1])
        fn = mathlib.UNARY.get(name) if len(xs) == 1 else mathlib.BINARY.get(name)
        if fn is None:
            raise Unsupported(f"unsupported elementwise op {name!r}")
        return Sym("f32", op=fn(mathlib.Ops(self.b, self.freg, ftz=bool(self.opts.get("approx_ftz"))), *xs))

    # ---- indexing (compile.py:594-679) -----------------------------------------------------
    def linear(self, buf: str, index) -> Affine:
        """Row-major element offset exactly as compile.py:594-615 defines it."""
        if buf in self.shapes:
            shape = self.shapes[buf]
        elif buf in self.smem:
            shape = self.smem[buf][0]
        else:
            raise Unsupported(f"unknown buffer {buf!r}")
        parts = list(index)
        if not parts:
            return Affine.const(0)
        if len(parts) == len(shape) and len(shape) > 1:
            acc = self.ival(parts[0])
            for i in range(1, len(parts)):
                if shape[i] == 1 and i == len(parts) - 1:
                    continue
                acc = acc.scale(shape[i]) + self.ival(parts[i])
            return recombine(acc)
        if len(parts) == 1:
            return recombine(self.ival(parts[0]))
        acc = self.ival(parts[0])
        for p in parts[1:]:
            acc = acc.scale(shape[-1]) + self.ival(p)
        return recombine(acc)

    def global_addr(self, buf: str, lin: Affine, esize: int):
        """(base register, byte immediate): the variable part via ``mad.wide``, the constant part
        left for the instruction's ``[reg+imm]`` operand."""
        var = lin.without_const()
        imm = lin.c * esize
        if buf not in self.preg:
            raise Unsupported(f"buffer {buf!r} is not a kernel parameter")
        base = self.preg[buf]
        if var.is_const():
            return base, imm
        key = ("gaddr", buf, var.key, esize)
        mutable = var.mutable()
        if not mutable:
            hit = self.b.lookup(key)
            if hit is not None:
                return hit, imm
        depth = None if mutable else var.depth()
        v = self.mat(var)
        r = self.b.reg("b64")
        op = "mad.wide.u32" if var.nonneg() else "mad.wide.s32"
        self.b.emit(f"{op} {r}, {v}, {esize}, {base};", depth)
        if not mutable:
            self.b.remember(key, r, depth)
        return r, imm

    def shared_addr(self, buf: str, lin: Affine, esize: int):
        var = lin.without_const()
        imm = lin.c * esize
        base = self.sbase[buf]
        if var.is_const():
            return base, imm
        key = ("saddr", buf, var.key, esize)
        mutable = var.mutable()
        if not mutable:
            hit = self.b.lookup(key)
            if hit is not None:
                return hit, imm
        depth = None if mutable else var.depth()
        v = self.mat(var)
        r = self.b.reg("b32")
        self.b.emit(f"mad.lo.s32 {r}, {v}, {esize}, {base};", depth)
        if not mutable:
            self.b.remember(key, r, depth)
        return r, imm

    @staticmethod
    def addr(base: str, imm: int) -> str:
        if imm == 0:
            return f"[{base}]"
        return f"[{base}+{imm}]"                     # a negative offset is written +-N

    def _base_align(self, buf: str, shared: bool) -> int:
        if shared:
            off = self.smem_off[buf]
            al = 16
            while al < 1024 and off % (al * 2) == 0:
                al *= 2
            return al
        return 32

    def _vec_plan(self, lin: Affine, n: int, esize: int, buf: str, shared: bool, global_max: int = 32):
        """Split n consecutive elements into (first element, count) chunks, each a power-of-two
        byte size whose alignment the index provably guarantees."""
        base_al = self._base_align(buf, shared)
        maxb = 16 if shared else global_max
        chunks = []
        i = 0
        while i < n:
            best = 1
            for cnt in (16, 8, 4, 2):
                nbytes = cnt * esize
                if cnt > n - i or nbytes > maxb or nbytes < 4 or nbytes > base_al:
                    continue
                if (lin + i).scale(esize).divisible_by(nbytes):
                    best = cnt
                    break
            chunks.append((i, best))
            i += best
        return chunks

    # ---- statements ------------------------------------------------------------------------
    def stmts(self, body) -> None:
        for st in body or ():
            fn = getattr(self, "st_" + type(st).__name__, None)
            if fn is None:
                raise Unsupported(f"unsupported statement {type(st).__name__}")
            fn(st)

    def st_Smem(self, st) -> None:
        pass                                                   # planned up front (compile.py:1384-1388)

    def st_Tile(self, st) -> None:
        """compile.py:1135-1157: guard ``gid < ncells``; coordinates row major, last axis fastest."""
        ext = [dim_int(a.extent) for a in st.axes]
        total = 1
        for e in ext:
            total *= e
        end = self.b.label("_end")
        lo, hi = self.gid.range()
        guarded = hi is None or hi >= total
        if guarded:
            p = self.b.reg("pred")
            self.b.emit(f"setp.ge.s32 {p}, {self.reg_of(self.gid)}, {total};")
            self.b.emit(f"@{p} bra {end};")
        self.b.push_scope()
        rest = self.gid
        for i, ax in enumerate(st.axes):
            inner = 1
            for e in ext[i + 1:]:
                inner *= e
            if i == len(ext) - 1:
                self.syms[ax.name] = Sym("s32", aff=rest)
            else:
                self.syms[ax.name] = Sym("s32", aff=div_const(rest, inner))
                rest = rem_const(rest, inner)
        self.stmts(st.body)
        self.b.pop_scope()
        self.b.place(end)

    def _load_type(self, st) -> str:
        if getattr(st, "dtype", None) is not None:
            return dt_name(st.dtype)
        if st.input in self.smem:
            return self.smem[st.input][1]
        return self.dtypes.get(st.input, "f32")

    def st_Load(self, st) -> None:
        """compile.py:1159-1204, with packed vector traffic."""
        names = list(st.names)
        buf = st.input
        t = self._load_type(st)
        shared = buf in self.smem
        lin = self.linear(buf, st.index)
        if t in BOOLS:
            for i, nm in enumerate(names):
                base, imm = (self.shared_addr if shared else self.global_addr)(buf, lin + i, 1)
                r = self.b.reg("b32")
                self.b.emit(f"ld.{'shared' if shared else 'global'}.u8 {r}, {self.addr(base, imm)};")
                self.syms[nm] = Sym("s32", aff=self.new_int(r, 0, 255))
            return
        if t == "f64":
            for i, nm in enumerate(names):
                base, imm = (self.shared_addr if shared else self.global_addr)(buf, lin + i, 8)
                d = self.b.reg("b64")
                self.b.emit(f"ld.{'shared' if shared else 'global'}.f64 {d}, {self.addr(base, imm)};")
                r = self.b.reg("f32")
                self.b.emit(f"cvt.rn.f32.f64 {r}, {d};")   # narrowed in the register (compile.py:1183-1193)
                self.syms[nm] = Sym("f32", op=r)
            return
        esize = dt_bytes(t)
        space = "shared" if shared else ("global.nc" if buf not in self.written else "global")
        if not shared and buf not in self.written:
            space += self._load_hint()
        if not shared:
            self.palign[buf] = max(self.palign.get(buf, 16), 16)
        for first, cnt in self._vec_plan(lin, len(names), esize, buf, shared):
            base, imm = (self.shared_addr if shared else self.global_addr)(buf, lin + first, esize)
            if not shared and cnt * esize == 32:
                self.palign[buf] = 32
            if esize == 4:
                regs = [self.b.reg("f32" if t in FLOATS else "b32") for _ in range(cnt)]
                vec = "" if cnt == 1 else f".v{cnt}"
                ty = "f32" if t in FLOATS else ("u32" if t == "u32" else "s32")
                dst = regs[0] if cnt == 1 else "{" + ", ".join(regs) + "}"
                self.b.emit(f"ld.{space}{vec}.{ty} {dst}, {self.addr(base, imm)};")
                for k, r in enumerate(regs):
                    nm = names[first + k]
                    self.syms[nm] = Sym("f32", op=r) if t in FLOATS else Sym("s32", aff=self.new_int(r))
            elif esize == 2:
                if cnt == 1:
                    h = self.b.reg("b16")
                    self.b.emit(f"ld.{space}.b16 {h}, {self.addr(base, imm)};")
                    r = self.b.reg("f32")
                    self.b.emit(f"cvt.f32.{t} {r}, {h};")
                    self.syms[names[first]] = Sym("f32", op=r)
                    continue
                words = [self.b.reg("b32") for _ in range(cnt // 2)]
                vec = "" if len(words) == 1 else f".v{len(words)}"
                dst = words[0] if len(words) == 1 else "{" + ", ".join(words) + "}"
                self.b.emit(f"ld.{space}{vec}.b32 {dst}, {self.addr(base, imm)};")
                for k, w in enumerate(words):
                    lo_nm, hi_nm = names[first + 2 * k], names[first + 2 * k + 1]
                    self.syms[lo_nm] = Sym("f32", op=self._unpack(w, t, 0))
                    self.syms[hi_nm] = Sym("f32", op=self._unpack(w, t, 1))
            else:
                raise Unsupported(f"unsupported load element size {esize}")

    def _load_hint(self) -> str:
        """Cache qualifiers for read-only global vector loads (opt-in): ``ld_no_l1`` adds
        ``.L1::no_allocate`` (streamed data never re-read through L1), ``ld_prefetch`` adds
        ``.L2::64B`` / ``.L2::128B`` / ``.L2::256B`` (the L2 fetches that many bytes per miss)."""
        hint = ""
        if self.opts.get("ld_no_l1"):
            hint += ".L1::no_allocate"
        pf = self.opts.get("ld_prefetch")
        if pf:
            if int(pf) not in (64, 128, 256):
                raise Unsupported(f"ld_prefetch must be 64, 128 or 256, not {pf!r}")
            hint += f".L2::{int(pf)}B"
        return hint

    def _store_hint(self) -> str:
        """A cache operator for global stores (opt-in ``st_cop``: ``cs`` streams the line past the
        caches, ``wt`` writes through)."""
        cop = self.opts.get("st_cop")
        if not cop:
            return ""
        if cop not in ("cs", "wt", "wb", "cg"):
            raise Unsupported(f"st_cop must be one of cs, wt, wb, cg, not {cop!r}")
        return "." + cop

    def _unpack(self, word: str, t: str, half: int) -> str:
        """One 16-bit float of a packed word, widened to f32 (exact)."""
        r = self.b.reg("f32")
        if t == "bf16":
            if half == 0:
                self.b.emit(f"shl.b32 {r}, {word}, 16;")
            else:
                self.b.emit(f"and.b32 {r}, {word}, -65536;")
            return r
        lo, hi = self.b.reg("b16"), self.b.reg("b16")
        self.b.emit(f"mov.b32 {{{lo}, {hi}}}, {word};")
        self.b.emit(f"cvt.f32.f16 {r}, {hi if half else lo};")
        return r

    def st_Write(self, st) -> None:
        """compile.py:1346-1382: one narrowing at the store; ``atomic`` is ``red.add``."""
        out = st.output
        values = [self.value(v) for v in st.values]
        t = dt_name(st.value_dtype)
        shared = out in self.smem
        lin = self.linear(out, st.index)
        space = "shared" if shared else "global"
        addr_fn = self.shared_addr if shared else self.global_addr
        if getattr(st, "atomic", False):
            if t in ("f16", "bf16", "f64"):
                raise Unsupported(f"atomic {t} write unsupported")
            if len(values) != 1:
                raise Unsupported("atomic vector write unsupported")
            base, imm = addr_fn(out, lin, dt_bytes(t))
            if t in FLOATS:
                self.b.emit(f"red.{space}.add.f32 {self.addr(base, imm)}, {self.freg(self.to_f32(values[0]))};")
            else:
                ty = "u32" if t == "u32" else "s32"
                self.b.emit(f"red.{space}.add.{ty} {self.addr(base, imm)}, {self.reg_of(self.to_int(values[0]))};")
            return
        if t in BOOLS:
            for i, v in enumerate(values):
                base, imm = addr_fn(out, lin + i, 1)
                x = self.to_int(v) if v.kind != "pred" else self.to_int(v)
                self.b.emit(f"st.{space}.u8 {self.addr(base, imm)}, {self.reg_of(x)};")
            return
        if t == "f64":
            for i, v in enumerate(values):
                base, imm = addr_fn(out, lin + i, 8)
                d = self.b.reg("b64")
                self.b.emit(f"cvt.f64.f32 {d}, {self.freg(self.to_f32(v))};")
                self.b.emit(f"st.{space}.f64 {self.addr(base, imm)}, {d};")
            return
        esize = dt_bytes(t)
        if not shared:
            space += self._store_hint()
        for first, cnt in self._vec_plan(lin, len(values), esize, out, shared):
            base, imm = addr_fn(out, lin + first, esize)
            if not shared and cnt * esize == 32:
                self.palign[out] = 32
            chunk = values[first:first + cnt]
            if esize == 4:
                if t in FLOATS:
                    regs = [self.to_f32(v) for v in chunk]
                    ty = "f32"
                else:
                    regs = [self.mat(self.to_int(v)) for v in chunk]
                    ty = "u32" if t == "u32" else "s32"
                vec = "" if cnt == 1 else f".v{cnt}"
                src = regs[0] if cnt == 1 else "{" + ", ".join(regs) + "}"
                self.b.emit(f"st.{space}{vec}.{ty} {self.addr(base, imm)}, {src};")
            elif esize == 2:
                if cnt == 1:
                    h = self.b.reg("b16")
                    self.b.emit(f"cvt.rn.{t}.f32 {h}, {self.freg(self.to_f32(chunk[0]))};")
                    self.b.emit(f"st.{space}.b16 {self.addr(base, imm)}, {h};")
                    continue
                words = []
                for k in range(cnt // 2):
                    w = self.b.reg("b32")
                    lo = self.freg(self.to_f32(chunk[2 * k]))
                    hi = self.freg(self.to_f32(chunk[2 * k + 1]))
                    self.b.emit(f"cvt.rn.{t}x2.f32 {w}, {hi}, {lo};")
                    words.append(w)
                vec = "" if len(words) == 1 else f".v{len(words)}"
                src = words[0] if len(words) == 1 else "{" + ", ".join(words) + "}"
                self.b.emit(f"st.{space}{vec}.b32 {self.addr(base, imm)}, {src};")
            else:
                raise Unsupported(f"unsupported store element size {esize}")

    def st_Assign(self, st) -> None:
        """compile.py:1206-1227."""
        opname = getattr(st.op, "name", None) or str(st.op)
        args = [self.value(a) for a in st.args]
        res = self.elementwise(opname, args)
        want = dt_name(st.dtype) if getattr(st, "dtype", None) is not None else None
        if want in ("bool", "bool8", "i1"):
            res = Sym("pred", op=self.to_pred(res))
        elif want in ("f16", "bf16", "f32", "f64") and res.kind != "f32":
            res = self.cast(res, want)
        elif want in INTS and res.kind == "f32":
            res = self.cast(res, want)
        self.syms[st.name] = res

    def st_Let(self, st) -> None:
        """compile.py:1262-1274."""
        t = dt_name(st.dtype)
        val = st.value
        if type(val).__name__ == "FlatIndex":
            self.syms[st.name] = Sym("s32", aff=self.linear(val.buffer, val.index))
            return
        self.syms[st.name] = self.cast(self.expr(val), t)

    def _seed_reg(self, name: str, dt: str, ident) -> None:
        if dt in FLOATS:
            r = self.b.reg("f32")
            self.b.emit(f"mov.b32 {r}, {f32_imm(float(ident))};")
            self.syms[name] = Sym("f32", op=r)
        else:
            r = self.b.reg("b32")
            self.b.emit(f"mov.b32 {r}, {int(ident)};")
            self.syms[name] = Sym("s32", aff=Affine.of(reg_atom(r, depth=self.b.depth, mutable=True)))

    def st_Init(self, st) -> None:
        """compile.py:1276-1286: a fresh register holding the identity."""
        self._seed_reg(st.name, dt_name(st.dtype), st.identity)

    @staticmethod
    def accum_identity(st):
        """compile.py:1288-1294: the seed is the op's identity; ``base`` only redirects the fold."""
        op = st.op
        if getattr(op, "has_identity", False) and getattr(op, "identity", None) is not None:
            return op.identity
        return {"add": 0.0, "multiply": 1.0, "maximum": -math.inf, "minimum": math.inf}.get(
            getattr(op, "name", ""), 0.0)

    def _accums(self, body, out):
        for st in body or ():
            cls = type(st).__name__
            if cls == "Accum":
                out.append(st)
            elif cls in ("StridedLoop", "Loop"):
                continue
            else:
                self._accums(getattr(st, "body", None), out)
                self._accums(getattr(st, "else_body", None), out)
        return out

    def hoist_accums(self, body) -> None:
        """compile.py:1296-1310: seed not-yet-bound accumulators in front of the loop."""
        for st in self._accums(body, []):
            if st.name in self.syms:
                continue
            self._seed_reg(st.name, dt_name(st.dtype), self.accum_identity(st))

    def st_Accum(self, st) -> None:
        """compile.py:1328-1344: ``acc = op(base or acc, value)``, in place."""
        opname = getattr(st.op, "name", "") or str(st.op)
        acc = self.syms[st.name]
        val = self.value(st.value)
        base = getattr(st, "base", None)
        left = self.value(base) if base is not None and base != st.name else acc
        if acc.kind == "f32":
            ins = {"add": "add.f32", "subtract": "sub.f32", "multiply": "mul.f32", "divide": "div.rn.f32",
                   "maximum": "max.f32", "minimum": "min.f32"}.get(opname)
            if ins is None:
                raise Unsupported(f"unsupported accumulator op {opname!r}")
            x, y = self.to_f32(left), self.to_f32(val)
            if not x.startswith("%"):
                x = self.freg(x)
            self.b.emit(f"{ins} {acc.op}, {x}, {y};")
            return
        ins = {"add": "add.s32", "subtract": "sub.s32", "multiply": "mul.lo.s32", "maximum": "max.s32",
               "minimum": "min.s32", "bitwise_and": "and.b32", "bitwise_or": "or.b32",
               "bitwise_xor": "xor.b32"}.get(opname)
        if ins is None:
            raise Unsupported(f"unsupported int accumulator op {opname!r}")
        areg = acc.aff.single_atom().reg
        self.b.emit(f"{ins} {areg}, {self.reg_of(self.to_int(left))}, {self.mat(self.to_int(val))};")

    def st_Select(self, st) -> None:
        """compile.py:1498-1520: first true branch wins, the last is the catch-all — as a selp chain."""
        brs = list(st.branches)
        res = self.value(brs[-1].value)
        for br in reversed(brs[:-1]):
            p = self.to_pred(self.expr(br.select))
            res = self.select(p, self.value(br.value), res)
        if res.kind == "f32" and not res.op.startswith("%"):
            res = Sym("f32", op=self.freg(res.op))
        self.syms[st.name] = res

    def st_Cond(self, st) -> None:
        """compile.py:1480-1496."""
        p = self.to_pred(self.expr(st.cond))
        other = self.b.label("_else")
        self.b.emit(f"@!{p} bra {other};")
        self.b.push_scope()
        self.stmts(st.body)
        self.b.pop_scope()
        if getattr(st, "else_body", None):
            end = self.b.label("_endif")
            self.b.emit(f"bra {end};")
            self.b.place(other)
            self.b.push_scope()
            self.stmts(st.else_body)
            self.b.pop_scope()
            self.b.place(end)
        else:
            self.b.place(other)

    def st_Sync(self, st) -> None:
        """compile.py:1390-1399."""
        if getattr(st, "warp", False):
            self.b.emit("bar.warp.sync -1;")
        elif getattr(st, "count", None):
            self.b.emit(f"bar.sync {int(getattr(st, 'barrier_id', 0) or 0)}, {int(st.count)};")
        else:
            self.b.emit(f"bar.sync {int(getattr(st, 'barrier_id', 0) or 0)};")

    # ---- CpAsyncCopy stripes promoted to TMA (codegen/tma_stripes.py) ------------------------
    def _tma_prologue(self, tid: str) -> None:
        """Tensor-map parameter addresses, the status word, the commit groups' mbarriers (thread 0
        initialises them; one block barrier publishes the initialisation) and the group counter."""
        b = self.b
        self.tma_regs = []
        for spec in self.tma["tmaps"]:
            r = b.reg("b64")
            b.emit(f"mov.u64 {r}, p_{spec['name']};")
            b.emit(f"cvta.param.u64 {r}, {r};")
            self.tma_regs.append(r)
        self.err = b.reg("b64")
        b.emit(f"ld.param.u64 {self.err}, [p_err];")
        b.emit(f"cvta.to.global.u64 {self.err}, {self.err};")
        self.t0 = b.reg("pred")
        b.emit(f"setp.eq.u32 {self.t0}, {tid}, 0;")
        skip = b.label("_tmainit")
        b.emit(f"@!{self.t0} bra {skip};")
        bars = self.sbase[TMA_BARS]
        for i in range(self.tma["nbar"]):
            b.emit(f"mbarrier.init.shared::cta.b64 [{bars}+{8 * i}], 1;")
        b.emit("fence.mbarrier_init.release.cluster;")
        b.place(skip)
        b.emit("bar.sync 0;")
        self.grp = b.reg("b32")
        b.emit(f"mov.u32 {self.grp}, 0;")

    def _last_block_epilogue(self) -> None:
        """Self-zeroing accumulators, and the multi-GPU sum's exchange fused after the reduction.

        Every block meets at a barrier (its atomic adds are issued); thread 0 releases them and takes a
        ticket (word 0 of the accumulator scratch).  In the block whose ticket is the last, warp 0
        resets the ticket, acquires the other blocks' adds, takes each accumulator with an atomic
        exchange against 0 (so the scratch is zero again for the next launch) and stores it to the
        output.  With the exchange option it then runs the peer exchange (kernels/peer_sum.py), which
        replaces this rank's partial in the output by the rank-ordered total of every rank's."""
        b, x = self.b, self.exchange
        end = b.label("_xend")
        lane, w, tk = b.reg("b32"), b.reg("b32"), b.reg("b32")
        pw, p0, plast = b.reg("pred"), b.reg("pred"), b.reg("pred")
        b.emit("bar.sync 0;")
        b.emit(f"and.b32 {lane}, {self.tid_reg}, 31;")
        b.emit(f"shr.u32 {w}, {self.tid_reg}, 5;")
        b.emit(f"setp.ne.u32 {pw}, {w}, 0;")
        b.emit(f"@{pw} bra {end};")
        b.emit(f"setp.eq.u32 {p0}, {lane}, 0;")
        b.emit(f"mov.u32 {tk}, 0;")
        b.emit(f"@{p0} fence.acq_rel.gpu;")
        b.emit(f"@{p0} atom.global.add.u32 {tk}, [{self.acc}], 1;")
        b.emit(f"shfl.sync.idx.b32 {tk}, {tk}, 0, 31, -1;")
        b.emit(f"setp.ne.u32 {plast}, {tk}, {self.G - 1};")
        b.emit(f"@{plast} bra {end};")
        b.emit(f"@{p0} st.global.u32 [{self.acc}], 0;")
        b.emit("fence.acq_rel.gpu;")
        for n, off in self.acc_outs.items():
            elems = 1
            for d in self.shapes[n]:
                elems *= int(d)
            skip = b.label("_accdone")
            pin, a_acc, a_out, v = b.reg("pred"), b.reg("b64"), b.reg("b64"), b.reg("b32")
            b.emit(f"setp.ge.u32 {pin}, {lane}, {elems};")
            b.emit(f"@{pin} bra {skip};")
            b.emit(f"mul.wide.u32 {a_acc}, {lane}, 4;")
            b.emit(f"add.s64 {a_out}, {a_acc}, {self.real_out[n]};")
            b.emit(f"add.s64 {a_acc}, {a_acc}, {self.preg[n]};")
            b.emit(f"atom.global.exch.b32 {v}, [{a_acc}], 0;")
            b.emit(f"st.global.b32 [{a_out}], {v};")
            b.place(skip)
        b.emit("bar.warp.sync -1;")
        if x:
            from ..kernels import peer_sum
            peer_sum.emit_exchange(lambda line: b.place(line[:-1]) if line.endswith(":") else b.emit(line),
                                   b.reg, lambda tag: b.label("_" + tag), lane, self.real_out[x["partial"]],
                                   self.xch, self.peers, self.err, int(x["rank"]), int(x["world"]), x["dtype"])
        b.place(end)

    def _tma_bar(self, group: str) -> str:
        """The shared address of the mbarrier of commit group ``group`` (a register)."""
        b = self.b
        slot, bar = b.reg("b32"), b.reg("b32")
        b.emit(f"rem.u32 {slot}, {group}, {self.tma['nbar']};")
        b.emit(f"mad.lo.u32 {bar}, {slot}, 8, {self.sbase[TMA_BARS]};")
        return bar

    def _reg32(self, aff) -> str:
        m = self.mat(aff)
        if m.startswith("%"):
            return m
        r = self.b.reg("b32")
        self.b.emit(f"mov.b32 {r}, {m};")
        return r

    def _tma_copy(self, st, sp) -> None:
        """One TMA tile load of the whole stripe, issued by thread 0 into the current group's
        mbarrier: the box origin is the source index less the lane's (row, col), the destination
        the stripe's shared base.  TMA wants the origin's innermost coordinate and the shared
        address on 16-byte boundaries; both are proved here or the kernel is built without TMA."""
        b = self.b
        es = sp.elem_bytes
        unit = 16 // es
        lin = self.linear(st.smem, st.smem_index)
        idx = [self.ival(x) for x in st.src_index]
        idx[-2] = recombine(idx[-2] - self.ival(st.lane_index[0]))
        idx[-1] = recombine(idx[-1] - self.ival(st.lane_index[1]))
        if not lin.divisible_by(unit) or not idx[-1].divisible_by(unit) or self.smem_off[st.smem] % 16:
            raise TmaNotProvable(f"cannot prove the 16-byte alignment of the {st.src!r} stripe")
        coords = [self._reg32(c) for c in reversed(idx)]
        base, imm = self.shared_addr(st.smem, lin, es)
        dst = b.reg("b32")
        b.emit(f"add.u32 {dst}, {base}, {imm};")
        bar = self._tma_bar(self.grp)
        rank = len(idx)
        t0 = self.t0
        b.emit(f"@{t0} fence.proxy.async.shared::cta;")
        b.emit(f"@{t0} mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [{bar}], {sp.box_bytes};")
        b.emit(f"@{t0} cp.async.bulk.tensor.{rank}d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
               f"[{dst}], [{self.tma_regs[sp.tmap]}, {{{', '.join(coords)}}}], [{bar}];")

    def st_CpAsyncCopy(self, st) -> None:
        """compile.py:1449-1471: stripe base plus the lane's (row, col); 16 B ``.cg``, 4/8 B ``.ca``.
        A kernel whose stripes each form one dense box issues them as TMA tile loads instead."""
        if self.tma is not None:
            self._tma_copy(st, self.tma["copies"][id(st)])
            return
        if str(getattr(st, "swizzle", "NONE") or "NONE").upper() != "NONE":
            raise Unsupported(f"unsupported cp.async swizzle {st.swizzle}")
        if getattr(st, "valid", None) is not None:
            raise Unsupported("predicated cp.async unsupported")
        ext, sdt, _ = self.smem[st.smem]
        lin = self.linear(st.smem, st.smem_index)
        lane = getattr(st, "lane_index", None)
        if lane is not None:
            lin = lin + self.ival(lane[0]).scale(ext[-1]) + self.ival(lane[1])
        es = dt_bytes(sdt)
        sbase, simm = self.shared_addr(st.smem, lin, es)
        gbase, gimm = self.global_addr(st.src, self.linear(st.src, st.src_index), dt_bytes(self.dtypes[st.src]))
        nbytes = int(st.nbytes)
        if nbytes == 16:
            self.b.emit(f"cp.async.cg.shared.global {self.addr(sbase, simm)}, {self.addr(gbase, gimm)}, 16;")
        elif nbytes in (4, 8):
            self.b.emit(f"cp.async.ca.shared.global {self.addr(sbase, simm)}, {self.addr(gbase, gimm)}, {nbytes};")
        else:
            raise Unsupported(f"unsupported cp.async size {nbytes}")

    def st_CpAsyncCommit(self, st) -> None:
        if self.tma is not None:
            # thread 0's arrival closes the group: its mbarrier phase completes once every TMA byte
            # of the group has landed (at once for a group that issued no copy)
            bar = self._tma_bar(self.grp)
            self.b.emit(f"@{self.t0} mbarrier.arrive.shared::cta.b64 _, [{bar}];")
            self.b.emit(f"add.u32 {self.grp}, {self.grp}, 1;")
            return
        self.b.emit("cp.async.commit_group;")

    def st_CpAsyncWait(self, st) -> None:
        n = int(getattr(st, "group", 0) or 0)
        if self.tma is None:
            self.b.emit(f"cp.async.wait_group {n};")
            return
        # every thread waits (bounded) for group g = committed - 1 - n: its mbarrier's phase g / nbar
        b = self.b
        g, ph, cnt = b.reg("b32"), b.reg("b32"), b.reg("b32")
        pz, pw, pq = b.reg("pred"), b.reg("pred"), b.reg("pred")
        done, top = b.label("_tmaw"), b.label("_tmawl")
        b.emit(f"sub.s32 {g}, {self.grp}, {n + 1};")
        b.emit(f"setp.lt.s32 {pz}, {g}, 0;")
        b.emit(f"@{pz} bra {done};")
        bar = self._tma_bar(g)
        b.emit(f"div.u32 {ph}, {g}, {self.tma['nbar']};")
        b.emit(f"and.b32 {ph}, {ph}, 1;")
        b.emit(f"mov.u32 {cnt}, 0;")
        b.place(top)
        b.emit(f"mbarrier.try_wait.parity.shared::cta.b64 {pw}, [{bar}], {ph}, {TMA_WAIT_HINT_NS};")
        b.emit(f"@{pw} bra {done};")
        b.emit(f"add.u32 {cnt}, {cnt}, 1;")
        b.emit(f"setp.lt.u32 {pq}, {cnt}, {TMA_WAIT_LIMIT};")
        b.emit(f"@{pq} bra {top};")
        b.emit(f"st.global.u32 [{self.err}], {ERR_TMA_WAIT};")
        b.place(done)

    def st_ZeroPrologue(self, st) -> None:
        """compile.py:1401-1447: the whole grid zeroes ``words`` 32-bit words, grid stride."""
        dst = st.dst
        words = int(getattr(st, "words", 0) or 0)
        if dst not in self.preg:
            raise Unsupported(f"zero-prologue target {dst!r} is not a kernel parameter")
        if words <= 0:
            return
        b = self.b
        r = {k: b.reg("b32") for k in ("nx", "gx", "i", "stride")}
        b.emit(f"mov.u32 {r['nx']}, %ntid.x;")
        b.emit(f"mov.u32 {r['gx']}, %nctaid.x;")
        b.emit(f"mul.lo.u32 {r['stride']}, {r['nx']}, {r['gx']};")
        b.emit(f"mad.lo.u32 {r['i']}, {self.reg_of(self.ctaid)}, {r['nx']}, {self.reg_of(self.tid)};")
        top, end = b.label("_zp"), b.label("_zpend")
        p = b.reg("pred")
        b.place(top)
        b.emit(f"setp.ge.u32 {p}, {r['i']}, {words};")
        b.emit(f"@{p} bra {end};")
        a = b.reg("b64")
        b.emit(f"mad.wide.u32 {a}, {r['i']}, 4, {self.preg[dst]};")
        b.emit(f"st.global.u32 [{a}], 0;")
        b.emit(f"add.u32 {r['i']}, {r['i']}, {r['stride']};")
        b.emit(f"bra {top};")
        b.place(end)

    # ---- loops (compile.py:1525-1618) ---------------------------------------------------------
    _FLAT = {"Load", "Write", "Assign", "Accum", "Let", "Init", "CpAsyncCopy", "CpAsyncCommit", "CpAsyncWait"}

    def _flat(self, body) -> bool:
        """compile.py:1525-1534: straight-line bodies only (no nested loop, branch or barrier)."""
        return all(type(s).__name__ in self._FLAT for s in body)

    def _loop(self, st, start: Affine, step: Affine, end: Affine, unroll_full: int = 0) -> None:
        self.hoist_accums(st.body)
        name = st.axis.name
        if unroll_full:
            for i in range(unroll_full):
                self.syms[name] = Sym("s32", aff=Affine.const(i))
                self.stmts(st.body)
            return
        b = self.b
        slo, shi = start.range()
        elo, ehi = end.range()
        step_c = step.c if step.is_const() else None
        lo = slo if (slo is not None and step_c is not None and step_c > 0) else None
        hi = (ehi - 1) if (ehi is not None and step_c is not None and step_c > 0) else None
        if lo is not None and hi is not None and hi < lo:
            hi = lo
        cur = b.reg("b32")
        b.emit(f"mov.b32 {cur}, {self.mat(start)};")
        unroll = 0
        if step_c is not None and step_c > 0 and self._flat(st.body) and not self.opts.get("no_unroll"):
            has_load = any(type(s).__name__ in ("Load", "CpAsyncCopy") for s in st.body)
            unroll = int(self.opts.get("unroll", 4)) if has_load else 0
            if elo is not None and slo is not None and ehi is not None and shi is not None:
                trips = (ehi - slo + step_c - 1) // step_c
                if trips < 2 * unroll:
                    unroll = 0
        exit_l = b.label("_lexit")
        endop = self.mat(end)

        def body_pass(counter: Affine):
            self.syms[name] = Sym("s32", aff=counter)
            self.stmts(st.body)

        if unroll > 1:
            rem_l = b.label("_lrem")
            p = b.reg("pred")
            span = (unroll - 1) * step_c
            last = b.reg("b32")
            b.emit(f"add.s32 {last}, {cur}, {span};")
            # the preheader (hoisted loop invariants) sits before the zero-trip guard, so what it
            # defines exists on every path past the loop, including the one that skips it
            b.open_loop()
            b.emit(f"setp.ge.s32 {p}, {last}, {endop};")
            b.emit(f"@{p} bra {rem_l};")
            top = b.label("_lu")
            b.place(top)
            ctr = Affine.of(reg_atom(cur, lo, hi, depth=b.depth))
            for u in range(unroll):
                body_pass(ctr + u * step_c)
            b.close_loop()
            b.emit(f"add.s32 {cur}, {cur}, {unroll * step_c};")
            b.emit(f"add.s32 {last}, {cur}, {span};")
            q = b.reg("pred")
            b.emit(f"setp.lt.s32 {q}, {last}, {endop};")
            b.emit(f"@{q} bra {top};")
            b.place(rem_l)
        p = b.reg("pred")
        b.open_loop()
        b.emit(f"setp.ge.s32 {p}, {cur}, {endop};")
        b.emit(f"@{p} bra {exit_l};")
        top = b.label("_l")
        b.place(top)
        body_pass(Affine.of(reg_atom(cur, lo, hi, depth=b.depth)))
        b.close_loop()
        stepop = self.mat(step)
        b.emit(f"add.s32 {cur}, {cur}, {stepop};")
        q = b.reg("pred")
        b.emit(f"setp.lt.s32 {q}, {cur}, {endop};")
        b.emit(f"@{q} bra {top};")
        b.place(exit_l)
        self.syms[name] = Sym("s32", aff=Affine.of(reg_atom(cur, depth=b.depth, mutable=True)))

    def st_StridedLoop(self, st) -> None:
        lim = st.end if getattr(st, "end", None) is not None else st.axis.extent
        self._loop(st, self.ival(st.start), self.ival(st.step), self.ival(lim))

    def st_Loop(self, st) -> None:
        lim_v = st.end if getattr(st, "end", None) is not None else st.axis.extent
        lim = self.ival(lim_v)
        full = 0
        if getattr(st, "unroll", False) and lim.is_const() and 1 < lim.c <= 128 and self._flat(st.body):
            full = lim.c
        self._loop(st, Affine.const(0), Affine.const(1), lim, unroll_full=full)

    # ---- warp and block reductions ---------------------------------------------------------
    def _single_op_combine(self, st, states, others):
        """The op name when the combine program is ``s_i = op(s_i, other_i)`` for each state."""
        comb = list(getattr(st, "combine_states", None) or ())
        if len(comb) != len(states):
            return None
        op = None
        for a, s, o in zip(comb, states, others):
            nm = getattr(a.op, "name", None) or str(a.op)
            args = list(a.args)
            if a.name != s or len(args) != 2 or not all(isinstance(x, str) for x in args):
                return None
            if set(args) != {s, o}:
                return None
            if op is not None and nm != op:
                return None
            op = nm
        return op

    def _bind_others(self, states, st):
        others = list(getattr(st, "state_b", None) or ())
        return [others[i] if i < len(others) else f"{nm}__o" for i, nm in enumerate(states)]

    def _shfl(self, mode: str, val: Sym, b_op, c_op: str) -> Sym:
        """One ``shfl.sync`` of a value of any kind (predicates travel as 0/1)."""
        if val.kind == "f32":
            src = self.freg(val.op)
            r = self.b.reg("f32")
            self.b.emit(f"shfl.sync.{mode}.b32 {r}, {src}, {b_op}, {c_op}, -1;")
            return Sym("f32", op=r)
        src = self.reg_of(self.to_int(val))
        r = self.b.reg("b32")
        self.b.emit(f"shfl.sync.{mode}.b32 {r}, {src}, {b_op}, {c_op}, -1;")
        return Sym("s32", aff=self.new_int(r))

    def st_WarpShuffle(self, st) -> None:
        """compile.py:1627-1654: butterfly all-reduce (or ``redux.sync``), or an inclusive scan."""
        states = list(st.state)
        others = self._bind_others(states, st)
        length = int(getattr(st, "length", 32) or 32)
        prefix = bool(getattr(st, "prefix", False))
        if length & (length - 1) or not 1 <= length <= 32:
            raise Unsupported(f"warp shuffle length {length}")
        op = None if prefix else self._single_op_combine(st, states, others)
        if op is not None and length == 32 and not self.opts.get("no_redux"):
            kinds = {self.syms[s].kind for s in states}
            ok = {("add", "s32"), ("maximum", "s32"), ("minimum", "s32"), ("bitwise_and", "s32"),
                  ("bitwise_or", "s32"), ("bitwise_xor", "s32"), ("maximum", "f32"), ("minimum", "f32")}
            if len(kinds) == 1 and (op, kinds.copy().pop()) in ok:
                kind = kinds.pop()
                rop = {"add": "add", "maximum": "max", "minimum": "min", "bitwise_and": "and",
                       "bitwise_or": "or", "bitwise_xor": "xor"}[op]
                for s in states:
                    v = self.syms[s]
                    if kind == "f32":
                        r = self.b.reg("f32")
                        self.b.emit(f"redux.sync.{rop}.f32 {r}, {self.freg(v.op)}, -1;")
                        self.syms[s] = Sym("f32", op=r)
                    else:
                        r = self.b.reg("b32")
                        ty = "s32" if rop in ("add", "max", "min") else "b32"
                        self.b.emit(f"redux.sync.{rop}.{ty} {r}, {self.reg_of(v.aff)}, -1;")
                        self.syms[s] = Sym("s32", aff=self.new_int(r))
                return
        off = 1 if prefix else length // 2
        while (off < length) if prefix else (off >= 1):
            for s, o in zip(states, others):
                v = self.syms[s]
                if prefix:
                    # lane i takes lane i-off; lanes below the segment get 0 (compile.py:1642-1648)
                    got = self._shfl("up", v, off, "0", )
                    lanev = self.syms["lane"].aff
                    p = self.b.reg("pred")
                    self.b.emit(f"setp.ge.s32 {p}, {self.reg_of(lanev)}, {off};")
                    zero = Sym("f32", op="0f00000000") if v.kind == "f32" else Sym("s32", aff=Affine.const(0))
                    got = self.select(p, got, zero)
                else:
                    got = self._shfl("bfly", v, off, "31")
                self.syms[o] = got
            for a in getattr(st, "combine_states", None) or ():
                self.st_Assign(a)
            off = off * 2 if prefix else off // 2

    def st_WarpBroadcast(self, st) -> None:
        """The last lane of each ``length`` group, to the whole group (compile.py:1656-1668 states
        this meaning; the segment mask here makes it hold for lengths below 32 too)."""
        length = int(getattr(st, "length", 32) or 32)
        if length & (length - 1) or not 1 <= length <= 32:
            raise Unsupported(f"warp broadcast length {length}")
        c = ((32 - length) << 8) | (length - 1)
        for nm in st.state:
            self.syms[nm] = self._shfl("idx", self.syms[nm], length - 1, str(c))

    def st_TreeHalve(self, st) -> None:
        """compile.py:1670-1708.  For at most 32 power-of-two slots of 32-bit data: every warp reads
        all slots once and reduces them with a butterfly — lane 0's combine order equals the
        halving tree's, so the result is the tree's; with a non-commutative combine lane 0's value
        is broadcast.  Otherwise the tree itself, one barrier per level."""
        bufs = list(getattr(st, "bufs", ()))
        states = list(st.state)
        others = self._bind_others(states, st)
        length = int(st.length)
        if length < 1:
            raise Unsupported("TreeHalve length must be positive")
        kinds = [self.syms[s].kind for s in states]
        types = [self.smem[bf][1] for bf in bufs]
        one_pass = (length & (length - 1) == 0 and length <= 32 and all(dt_bytes(t) == 4 for t in types)
                    and not self.opts.get("tree_barriers"))
        if not one_pass:
            return self._tree_levels(st, bufs, states, others, length)
        lane = self.syms["lane"].aff
        idx = rem_const(lane, length) if length < 32 else lane
        for bf, s, t in zip(bufs, states, types):
            base, imm = self.shared_addr(bf, idx, 4)
            if t in FLOATS:
                r = self.b.reg("f32")
                self.b.emit(f"ld.shared.f32 {r}, {self.addr(base, imm)};")
                self.syms[s] = Sym("f32", op=r)
            else:
                r = self.b.reg("b32")
                self.b.emit(f"ld.shared.b32 {r}, {self.addr(base, imm)};")
                self.syms[s] = Sym("s32", aff=self.new_int(r))
        off = length // 2
        while off >= 1:
            for s, o in zip(states, others):
                self.syms[o] = self._shfl("bfly", self.syms[s], off, "31")
            for a in getattr(st, "combine_states", None) or ():
                self.st_Assign(a)
            off //= 2
        op = self._single_op_combine(st, states, others)
        if op not in ("add", "multiply", "maximum", "minimum", "bitwise_and", "bitwise_or", "bitwise_xor"):
            for s in states:
                self.syms[s] = self._shfl("idx", self.syms[s], 0, "31")

    def _tree_levels(self, st, bufs, states, others, length) -> None:
        tid = getattr(st, "tid_var", "warp") or "warp"
        treg = self.syms[tid].aff if tid in self.syms else self.syms["warp"].aff
        bar = int(getattr(st, "barrier_id", 0) or 0)
        cnt = getattr(st, "barrier_count", None)
        s = length // 2
        while s >= 1:
            p = self.b.reg("pred")
            self.b.emit(f"setp.lt.s32 {p}, {self.reg_of(treg)}, {s};")
            skip = self.b.label("_tskip")
            self.b.emit(f"@!{p} bra {skip};")
            self.b.push_scope()
            slots = []
            for bf, nm, o in zip(bufs, states, others):
                t = self.smem[bf][1]
                ty = "f32" if t in FLOATS else "s32"
                a_base, a_imm = self.shared_addr(bf, treg, 4)
                b_base, b_imm = self.shared_addr(bf, treg + s, 4)
                ra = self.b.reg("f32" if ty == "f32" else "b32")
                rb = self.b.reg("f32" if ty == "f32" else "b32")
                self.b.emit(f"ld.shared.{ty} {ra}, {self.addr(a_base, a_imm)};")
                self.b.emit(f"ld.shared.{ty} {rb}, {self.addr(b_base, b_imm)};")
                mk = (lambda r: Sym("f32", op=r)) if ty == "f32" else (lambda r: Sym("s32", aff=self.new_int(r)))
                self.syms[nm] = mk(ra)
                self.syms[o] = mk(rb)
                slots.append((a_base, a_imm, nm, ty))
            for a in getattr(st, "combine_states", None) or ():
                self.st_Assign(a)
            for a_base, a_imm, nm, ty in slots:
                v = self.syms[nm]
                src = self.freg(v.op) if ty == "f32" else self.reg_of(v.aff)
                self.b.emit(f"st.shared.{ty} {self.addr(a_base, a_imm)}, {src};")
            self.b.pop_scope()
            self.b.place(skip)
            self.b.emit(f"bar.sync {bar}, {int(cnt)};" if cnt else f"bar.sync {bar};")
            s //= 2
        for bf, nm in zip(bufs, states):
            t = self.smem[bf][1]
            if t in FLOATS:
                r = self.b.reg("f32")
                self.b.emit(f"ld.shared.f32 {r}, [{self.sbase[bf]}];")
                self.syms[nm] = Sym("f32", op=r)
            else:
                r = self.b.reg("b32")
                self.b.emit(f"ld.shared.s32 {r}, [{self.sbase[bf]}];")
                self.syms[nm] = Sym("s32", aff=self.new_int(r))

    # ---- whole kernel ------------------------------------------------------------------------
    def build(self) -> dict:
        self.prepare()
        self.prologue()
        self.stmts(self.op.body)
        if self.acc_outs:
            self._last_block_epilogue()
        body, decls = self.b.lines(), self.b.reg_decls()
        if self.opts.get("regalloc", os.environ.get("EMMY_B200_REGALLOC", "1") != "0"):
            from .regalloc import allocate
            from .ptx import REG_CLASSES
            body, counts = allocate(body)
            by_prefix = {pre[1:]: ty for pre, ty in REG_CLASSES.values()}
            decls = [f"\t.reg {by_prefix[c]} %{c}<{k + 1}>;" for c, k in sorted(counts.items())]
        extra = []
        if self.exchange:
            extra += [{"name": "__xch", "kind": "buffer", "param": "p_xch"},
                      {"name": "__peers", "kind": "buffer", "param": "p_peers"}]
        acc_name, acc_words = f"{self.prefix}{self.name}__acc", 0
        if self.acc_outs:
            # the accumulator scratch: the runtime allocates it zeroed once; every launch leaves it zero
            acc_words = max(16 + 4 * 32, max(self.acc_outs.values()) + 4 * 32) // 4
            extra.append({"name": acc_name, "kind": "buffer", "param": "p_acc"})
        if self.tma is not None or self.exchange:
            extra.append({"name": "__err", "kind": "errword"})
        return {
            "name": self.name,
            "params": list(self.params),
            "body": body,
            "decls": decls,
            "smem": [(self.sym_name(n), self.smem_off[n], self.smem[n]) for n in self.smem],
            "smem_total": self.smem_total,
            "dyn": self.dyn,
            "dyn_smem": self.dyn_smem,
            "pool_name": self.sym_name("smem_pool"),
            "block": self.kmeta.get("block") or [],
            "grid": self.kmeta.get("grid") or [],
            "reqntid": self.T,
            "align": dict(self.palign),
            "zero_outputs": [n for n in (self.kmeta.get("zero_outputs") or []) if n not in self.acc_outs],
            "pdl": self.pdl,
            **({"tmaps": self.tma["tmaps"]} if self.tma is not None else {}),
            **({"extra": extra} if extra else {}),
            **({"scratch": [{"name": acc_name, "dtype": "i32", "shape": [acc_words], "zeroed": True}],
                "self_zeroing": sorted(self.acc_outs)} if self.acc_outs else {}),
            **({"exchange": dict(self.exchange)} if self.exchange else {}),
        }
