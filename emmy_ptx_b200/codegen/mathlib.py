"""Elementwise float math for the CUDA-core path, built on the hardware ``ex2``/``lg2``.

Each function takes an :class:`Ops` and f32 operands (registers or ``0f…`` immediates) and
returns the result register.  The formulas are the reference's (compile.py:937-1111), which in
turn are textbook: ``exp(x) = 2^(x*log2 e)``, ``log(x) = log2(x)*ln 2``, ``tanh(x) = 1 - 2/(e^2x+1)``,
``sigmoid(x) = 1/(1+2^(-x*log2 e))`` and ``erf`` by Abramowitz & Stegun 7.1.26.  No vendor
math-library code or constants are involved: the only transcendental instructions are the PTX
``ex2.approx.f32``/``lg2.approx.f32``/``sin.approx``/``cos.approx``/``rsqrt.approx``.
"""
from __future__ import annotations

from .ptx import f32_imm

LOG2E = 1.4426950408889634
LN2 = 0.6931471805599453
LOG10_2 = 0.30102999566398120

COMPARISONS = {"greater": "gt", "less": "lt", "greater_equal": "ge", "less_equal": "le",
               "equal": "eq", "not_equal": "ne"}


class Ops:
    """Instruction helpers over a :class:`~.ptx.PtxBuilder` (first operands forced to registers)."""

    def __init__(self, b, freg, ftz: bool = False):
        self.b = b
        self.freg = freg
        self.ftz = ftz          # option approx_ftz: ex2/lg2 flush subnormal inputs and results to zero

    _FTZ = {"ex2.approx.f32": "ex2.approx.ftz.f32", "lg2.approx.f32": "lg2.approx.ftz.f32"}

    @staticmethod
    def c(v: float) -> str:
        return f32_imm(v)

    def un(self, ins: str, x: str) -> str:
        if self.ftz:
            ins = self._FTZ.get(ins, ins)
        r = self.b.reg("f32")
        self.b.emit(f"{ins} {r}, {self.freg(x)};")
        return r

    def bin(self, ins: str, x: str, y: str) -> str:
        r = self.b.reg("f32")
        self.b.emit(f"{ins} {r}, {self.freg(x)}, {y};")
        return r

    def fma(self, x: str, y: str, z: str) -> str:
        r = self.b.reg("f32")
        self.b.emit(f"fma.rn.f32 {r}, {self.freg(x)}, {y}, {z};")
        return r

    def selp(self, x: str, y: str, p: str) -> str:
        r = self.b.reg("f32")
        self.b.emit(f"selp.f32 {r}, {x}, {y}, {p};")
        return r

    def setp(self, cmp: str, x: str, y: str) -> str:
        p = self.b.reg("pred")
        self.b.emit(f"setp.{cmp}.f32 {p}, {self.freg(x)}, {y};")
        return p

    # composite helpers
    def exp(self, x):
        return self.un("ex2.approx.f32", self.bin("mul.f32", x, self.c(LOG2E)))

    def lg2(self, x):
        return self.un("lg2.approx.f32", x)

    def rcp(self, x):
        return self.un("rcp.rn.f32", x)


def _sigmoid(o: Ops, x):
    return o.rcp(o.bin("add.f32", o.un("ex2.approx.f32", o.bin("mul.f32", x, o.c(-LOG2E))), o.c(1.0)))


def _tanh(o: Ops, x):
    e2 = o.un("ex2.approx.f32", o.bin("mul.f32", x, o.c(2.0 * LOG2E)))
    q = o.bin("div.rn.f32", o.c(2.0), o.bin("add.f32", e2, o.c(1.0)))
    return o.bin("sub.f32", o.c(1.0), q)


def _erf(o: Ops, x):
    """Abramowitz & Stegun 7.1.26 (|error| < 1.5e-7) with the sign bit restored."""
    ax = o.un("abs.f32", x)
    t = o.rcp(o.fma(ax, o.c(0.3275911), o.c(1.0)))
    poly = o.c(1.061405429)
    for k in (-1.453152027, 1.421413741, -0.284496736, 0.254829592):
        poly = o.fma(poly, t, o.c(k))
    series = o.bin("mul.f32", poly, t)
    tail = o.bin("mul.f32", series, o.exp(o.bin("mul.f32", o.bin("mul.f32", ax, ax), o.c(-1.0))))
    y = o.bin("sub.f32", o.c(1.0), tail)
    sgn = o.b.reg("b32")
    o.b.emit(f"and.b32 {sgn}, {o.freg(x)}, -2147483648;")
    r = o.b.reg("f32")
    o.b.emit(f"or.b32 {r}, {y}, {sgn};")
    return r


def _gelu(o: Ops, x):
    inner = _erf(o, o.bin("mul.f32", x, o.c(0.7071067811865476)))
    return o.bin("mul.f32", o.bin("mul.f32", x, o.c(0.5)), o.bin("add.f32", inner, o.c(1.0)))


def _gelu_tanh(o: Ops, x):
    x3 = o.bin("mul.f32", o.bin("mul.f32", x, x), x)
    inner = o.bin("mul.f32", o.bin("add.f32", x, o.bin("mul.f32", x3, o.c(0.044715))), o.c(0.7978845608028654))
    return o.bin("mul.f32", o.bin("mul.f32", x, o.c(0.5)), o.bin("add.f32", _tanh(o, inner), o.c(1.0)))


def _softplus(o: Ops, x):
    ax = o.un("abs.f32", x)
    e = o.exp(o.bin("mul.f32", ax, o.c(-1.0)))
    lg = o.bin("mul.f32", o.lg2(o.bin("add.f32", e, o.c(1.0))), o.c(LN2))
    return o.bin("add.f32", o.bin("max.f32", x, o.c(0.0)), lg)


def _sign(o: Ops, x):
    pos = o.setp("gt", x, o.c(0.0))
    nz = o.setp("ne", x, o.c(0.0))
    one = o.selp(o.c(1.0), o.c(-1.0), pos)
    return o.selp(one, o.c(0.0), nz)


def _fmod(o: Ops, x, y):
    q = o.bin("div.rn.f32", x, y)
    tr = o.un("cvt.rzi.f32.f32", q)
    return o.bin("sub.f32", x, o.bin("mul.f32", tr, y))


UNARY = {
    "relu": lambda o, x: o.bin("max.f32", x, o.c(0.0)),
    "neg": lambda o, x: o.un("neg.f32", x), "negative": lambda o, x: o.un("neg.f32", x),
    "absolute": lambda o, x: o.un("abs.f32", x), "abs": lambda o, x: o.un("abs.f32", x),
    "fabs": lambda o, x: o.un("abs.f32", x),
    "sqrt": lambda o, x: o.un("sqrt.rn.f32", x), "rsqrt": lambda o, x: o.un("rsqrt.approx.f32", x),
    "reciprocal": lambda o, x: o.un("rcp.rn.f32", x),
    "sin": lambda o, x: o.un("sin.approx.f32", x), "cos": lambda o, x: o.un("cos.approx.f32", x),
    "floor": lambda o, x: o.un("cvt.rmi.f32.f32", x), "ceil": lambda o, x: o.un("cvt.rpi.f32.f32", x),
    "round": lambda o, x: o.un("cvt.rni.f32.f32", x), "rint": lambda o, x: o.un("cvt.rni.f32.f32", x),
    "trunc": lambda o, x: o.un("cvt.rzi.f32.f32", x),
    "exp": lambda o, x: o.exp(x), "exp_fast": lambda o, x: o.exp(x),
    "exp2": lambda o, x: o.un("ex2.approx.f32", x),
    "log": lambda o, x: o.bin("mul.f32", o.lg2(x), o.c(LN2)),
    "ln": lambda o, x: o.bin("mul.f32", o.lg2(x), o.c(LN2)),
    "log2": lambda o, x: o.lg2(x),
    "log10": lambda o, x: o.bin("mul.f32", o.lg2(x), o.c(LOG10_2)),
    "tanh": _tanh, "sigmoid": _sigmoid,
    "silu": lambda o, x: o.bin("mul.f32", x, _sigmoid(o, x)),
    "softplus": _softplus, "gelu": _gelu, "gelu_tanh": _gelu_tanh, "erf": _erf, "sign": _sign,
    "square": lambda o, x: o.bin("mul.f32", x, o.freg(x)),
    "log1p": lambda o, x: o.bin("mul.f32", o.lg2(o.bin("add.f32", x, o.c(1.0))), o.c(LN2)),
    "expm1": lambda o, x: o.bin("sub.f32", o.exp(x), o.c(1.0)),
    "sinh": lambda o, x: o.bin("mul.f32", o.bin("sub.f32", o.exp(x), o.exp(o.bin("mul.f32", x, o.c(-1.0)))), o.c(0.5)),
    "cosh": lambda o, x: o.bin("mul.f32", o.bin("add.f32", o.exp(x), o.exp(o.bin("mul.f32", x, o.c(-1.0)))), o.c(0.5)),
}

BINARY = {
    "power": lambda o, x, y: o.un("ex2.approx.f32", o.bin("mul.f32", o.lg2(x), y)),
    "pow": lambda o, x, y: o.un("ex2.approx.f32", o.bin("mul.f32", o.lg2(x), y)),
    "mod": _fmod, "remainder": _fmod, "fmod": _fmod,
    "floor_divide": lambda o, x, y: o.un("cvt.rmi.f32.f32", o.bin("div.rn.f32", x, y)),
    "hypot": lambda o, x, y: o.un("sqrt.rn.f32", o.bin("add.f32", o.bin("mul.f32", x, o.freg(x)),
                                                       o.bin("mul.f32", y, o.freg(y)))),
}
