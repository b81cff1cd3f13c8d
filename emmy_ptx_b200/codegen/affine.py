"""Symbolic 32-bit integer values: affine forms over atoms, with range-aware div/mod rewriting.

Every integer the IR computes (coordinates, loop counters, index arithmetic) is held as
``sum(coef * atom) + const`` until an instruction actually needs it in a register.  That lets
the emitter

* cancel terms (a Tile decode ``i * C + 8 * (gid - i * C / 8)`` collapses to ``8 * gid``),
* move the constant part of an address into the ``[reg + imm]`` operand of the load/store,
* prove vector alignment (every coefficient and the constant divisible by the width), and
* decide where a value may be computed (the outermost loop preheader it is invariant in).

Integer semantics are those of the reference emitter: 32-bit wrap-around ``add``/``mul``
(exact modulo 2**32, so re-association is exact), truncating ``div``/``rem`` (compile.py:274-275).
A quotient or remainder by a constant becomes a lazy :class:`Atom`; the rewrite rules below
only fire when value ranges prove them exact, otherwise the plain ``div.s32``/``rem.s32`` is kept.
"""
from __future__ import annotations

from math import gcd

INT_MIN, INT_MAX = -(1 << 31), (1 << 31) - 1


class Atom:
    """A leaf of an affine form.

    kind ``reg``: a value already in a register (``reg`` set); ``div``/``rem``: the truncating
    quotient/remainder of an affine numerator by a positive constant, materialised on demand.
    ``lo``/``hi`` bound the value (None = unknown).  ``depth`` is the loop depth of the innermost
    loop whose body defines it; ``mutable`` registers (loop counters are not, accumulators are)
    are never cached or hoisted.
    """

    __slots__ = ("kind", "key", "lo", "hi", "depth", "reg", "num", "d", "mutable")

    def __init__(self, kind, key, lo=None, hi=None, depth=0, reg=None, num=None, d=None, mutable=False):
        self.kind = kind
        self.key = key
        self.lo = lo
        self.hi = hi
        self.depth = depth
        self.reg = reg
        self.num = num
        self.d = d
        self.mutable = mutable

    def __hash__(self):
        return hash(self.key)

    def __eq__(self, other):
        return isinstance(other, Atom) and self.key == other.key

    def __lt__(self, other):
        return _order(self.key) < _order(other.key)

    def __repr__(self):
        if self.kind == "reg":
            return self.reg
        return f"({self.num!r} {'/' if self.kind == 'div' else '%'} {self.d})"


def _order(key):
    return repr(key)


def reg_atom(reg: str, lo=None, hi=None, depth=0, mutable=False) -> Atom:
    return Atom("reg", ("reg", reg), lo, hi, depth, reg=reg, mutable=mutable)


class Affine:
    """``sum(terms[atom] * atom) + c`` with integer coefficients."""

    __slots__ = ("terms", "c")

    def __init__(self, terms=None, c: int = 0):
        self.terms = {a: k for a, k in (terms or {}).items() if k}
        self.c = int(c)

    # -- construction -------------------------------------------------------------------
    @staticmethod
    def const(c: int) -> "Affine":
        return Affine({}, c)

    @staticmethod
    def of(atom: Atom, k: int = 1) -> "Affine":
        return Affine({atom: k}, 0)

    def is_const(self) -> bool:
        return not self.terms

    def single_atom(self):
        """The atom when this form is exactly ``1 * atom``, else None."""
        if self.c == 0 and len(self.terms) == 1:
            (a, k), = self.terms.items()
            if k == 1:
                return a
        return None

    @property
    def key(self):
        return (tuple(sorted(((a.key, k) for a, k in self.terms.items()), key=lambda t: _order(t[0]))), self.c)

    def __add__(self, o):
        o = _aff(o)
        t = dict(self.terms)
        for a, k in o.terms.items():
            t[a] = t.get(a, 0) + k
        return Affine(t, self.c + o.c)

    __radd__ = __add__

    def __neg__(self):
        return Affine({a: -k for a, k in self.terms.items()}, -self.c)

    def __sub__(self, o):
        return self + (-_aff(o))

    def __rsub__(self, o):
        return _aff(o) - self

    def scale(self, k: int) -> "Affine":
        return Affine({a: c * k for a, c in self.terms.items()}, self.c * k)

    def without_const(self) -> "Affine":
        return Affine(self.terms, 0)

    # -- analysis -----------------------------------------------------------------------
    def range(self):
        """(lo, hi) over the atoms' ranges, or (None, None) when any atom is unbounded."""
        lo = hi = self.c
        for a, k in self.terms.items():
            if a.lo is None or a.hi is None:
                return None, None
            if k > 0:
                lo += k * a.lo
                hi += k * a.hi
            else:
                lo += k * a.hi
                hi += k * a.lo
        return lo, hi

    def nonneg(self) -> bool:
        lo, _ = self.range()
        return lo is not None and lo >= 0

    def depth(self) -> int:
        return max((a.depth for a in self.terms), default=0)

    def mutable(self) -> bool:
        return any(a.mutable for a in self.terms)

    def divisible_by(self, n: int) -> bool:
        """True when every value this form takes is a multiple of ``n``."""
        if self.c % n:
            return False
        return all(k % n == 0 for k in self.terms.values())

    def coef_gcd(self) -> int:
        g = 0
        for k in self.terms.values():
            g = gcd(g, abs(k))
        return g

    def __repr__(self):
        parts = [f"{k}*{a!r}" for a, k in sorted(self.terms.items(), key=lambda t: _order(t[0].key))]
        if self.c or not parts:
            parts.append(str(self.c))
        return " + ".join(parts)


def recombine(a: Affine) -> Affine:
    """Fold ``k*d*(X/d) + k*(X%d)`` back into ``k*X`` (exact for X >= 0), repeatedly.

    A row-major decode followed by re-linearisation produces exactly these pairs; folding them
    removes the division and remainder from the emitted code altogether."""
    changed = True
    while changed:
        changed = False
        divs = {(at.num.key, at.d): at for at in a.terms if at.kind == "div"}
        for at, k in list(a.terms.items()):
            if at.kind != "rem" or not at.num.nonneg():
                continue
            dv = divs.get((at.num.key, at.d))
            if dv is None or a.terms.get(dv, 0) != k * at.d:
                continue
            t = dict(a.terms)
            del t[at]
            del t[dv]
            a = Affine(t, a.c) + at.num.scale(k)
            changed = True
            break
    return a


def _aff(x) -> Affine:
    if isinstance(x, Affine):
        return x
    if isinstance(x, int):
        return Affine.const(x)
    if isinstance(x, Atom):
        return Affine.of(x)
    raise TypeError(f"not an integer form: {x!r}")


def _trunc_div(a: int, b: int) -> int:
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def _split_for(num: Affine, d: int):
    """Find c | d with num = c*X + R, X a form over some terms, 0 <= R < c and X >= 0.

    Returns (c, X, R) for the largest such c, or None.  Used by both div and rem:
    floor((c*X + R) / (c*k)) = floor(X / k) and (c*X + R) % (c*k) = c*(X % k) + R.
    """
    if not num.nonneg():
        return None
    cands = sorted({abs(k) for k in num.terms.values()} | ({abs(num.c)} if num.c else set()), reverse=True)
    for c in cands:
        if c <= 1 or d % c:
            continue
        big = {a: k // c for a, k in num.terms.items() if k % c == 0}
        rest = Affine({a: k for a, k in num.terms.items() if k % c}, 0)
        cbig = (num.c // c) * c if num.c >= 0 else 0
        rest = rest + (num.c - cbig)
        X = Affine(big, cbig // c)
        lo, hi = rest.range()
        if lo is None or lo < 0 or hi >= c:
            continue
        if not X.nonneg():
            continue
        return c, X, rest
    return None


def div_const(num, d: int) -> Affine:
    """``num / d`` (truncating) for a positive constant ``d``, simplified when ranges allow."""
    num = _aff(num)
    if d <= 0:
        raise ValueError("division by a non-positive constant is not an affine rewrite")
    if d == 1:
        return num
    if num.is_const():
        return Affine.const(_trunc_div(num.c, d))
    if num.nonneg():
        lo, hi = num.range()
        if hi < d:
            return Affine.const(0)
        # exact part: terms whose coefficient is a multiple of d
        exact = {a: k // d for a, k in num.terms.items() if k % d == 0}
        rest = Affine({a: k for a, k in num.terms.items() if k % d}, num.c % d)
        exact_c = num.c // d
        E = Affine(exact, exact_c)
        if exact and E.nonneg() and rest.nonneg():
            rlo, rhi = rest.range()
            if rhi < d:
                return E
            return E + div_const(rest, d)
        sp = _split_for(num, d)
        if sp is not None:
            c, X, _R = sp
            return div_const(X, d // c)
        a = num.single_atom()
        if a is not None and a.kind == "div" and a.num.nonneg():
            return div_const(a.num, a.d * d)
    lo, hi = num.range()
    atom = Atom("div", ("div", num.key, d),
                lo=None if lo is None else _trunc_div(lo, d), hi=None if hi is None else _trunc_div(hi, d),
                depth=num.depth(), num=num, d=d, mutable=num.mutable())
    return Affine.of(atom)


def rem_const(num, d: int) -> Affine:
    """``num % d`` (sign of the dividend) for a positive constant ``d``."""
    num = _aff(num)
    if d <= 0:
        raise ValueError("remainder by a non-positive constant is not an affine rewrite")
    if d == 1:
        return Affine.const(0)
    if num.is_const():
        return Affine.const(num.c - _trunc_div(num.c, d) * d)
    if num.nonneg():
        lo, hi = num.range()
        if hi < d:
            return num
        # drop every term that is a multiple of d
        red = Affine({a: k for a, k in num.terms.items() if k % d}, num.c % d)
        if red.nonneg():
            rlo, rhi = red.range()
            if rhi < d:
                return red
        sp = _split_for(num, d)
        if sp is not None:
            c, X, R = sp
            return rem_const(X, d // c).scale(c) + R
        if red.nonneg() and len(red.terms) < len(num.terms):
            num = red
    lo, hi = num.range()
    if lo is not None and lo >= 0:
        rl, rh = 0, min(d - 1, hi)
    elif hi is not None and hi <= 0:
        rl, rh = max(-(d - 1), lo), 0
    else:
        rl, rh = -(d - 1), d - 1
    atom = Atom("rem", ("rem", num.key, d), lo=rl, hi=rh, depth=num.depth(), num=num, d=d,
                mutable=num.mutable())
    return Affine.of(atom)
