"""Shared pieces of the hand-written tensor-core kernels: a small PTX assembler, bounded mbarrier
waits, and the tcgen05 instruction / shared-memory descriptor encodings.

Descriptor bit layouts follow the public sm_100 matrix-descriptor and instruction-descriptor formats
(the same fields CUTLASS's ``cute/arch/mma_sm100_desc.hpp`` names): instruction descriptor bits 4-5
D format, 7-9 / 10-12 A / B format, 15 / 16 A / B major-ness, 17-22 N>>3, 24-28 M>>4; matrix
descriptor bits 0-13 start address>>4, 16-29 leading byte offset>>4, 32-45 stride byte offset>>4,
46-48 the constant 0b001, 61-63 the swizzle mode.
"""
from __future__ import annotations

WAIT_LIMIT = 40000               # bounded polls of try_wait with a 0.1 ms hint: < ~4 s
WAIT_HINT_NS = 100000


def idesc_f16(m: int, n: int, a_mn_major: bool, b_mn_major: bool, half: bool = False) -> int:
    """tcgen05 instruction descriptor, kind::f16, bf16 x bf16 -> f32 (f16 x f16 -> f32 with ``half``;
    the two operands always have the same type)."""
    fmt = 0 if half else 1       # A / B format: 0 f16, 1 bf16
    d = 0
    d |= 1 << 4                  # D format: f32
    d |= fmt << 7                # A format
    d |= fmt << 10               # B format
    d |= (1 if a_mn_major else 0) << 15
    d |= (1 if b_mn_major else 0) << 16
    d |= (n >> 3) << 17
    d |= (m >> 4) << 24
    return d


def smem_desc_hi(lbo: int, sbo: int, swizzle: int = 128) -> int:
    """Bits 16..63 of a shared-memory matrix descriptor (SWIZZLE_128B, or SWIZZLE_64B with
    ``swizzle=64``; version 1); the start address (>>4) is added into bits 0..13 at run time."""
    d = 0
    d |= ((lbo >> 4) & 0x3FFF) << 16
    d |= ((sbo >> 4) & 0x3FFF) << 32
    d |= 1 << 46                 # descriptor version for sm_100
    d |= {128: 2, 64: 4}[swizzle] << 61      # layout type: 2 SWIZZLE_128B, 4 SWIZZLE_64B
    return d


class Asm:
    """Tiny PTX assembler helper: numbered registers per class, labels, lines."""

    def __init__(self):
        self.lines: list[str] = []
        self.n = {"r": 0, "rd": 0, "p": 0, "f": 0}
        self.lab = 0

    def r(self, cls="r"):
        self.n[cls] += 1
        return f"%{cls}{self.n[cls]}"

    def L(self, tag):
        self.lab += 1
        return f"$G{self.lab}_{tag}"

    def __call__(self, line):
        self.lines.append(line if line.endswith(":") else "\t" + line)

    def label(self, name):
        self.lines.append(name + ":")

    def decls(self):
        ty = {"r": ".b32", "rd": ".b64", "p": ".pred", "f": ".f32"}
        return [f"\t.reg {ty[c]} %{c}<{k + 1}>;" for c, k in self.n.items() if k]


def wait_bar(a: Asm, bar: str, parity: str, err: str, code: int, bail: str) -> None:
    """Bounded wait for ``bar`` to complete the phase of ``parity``; on time-out write ``code``
    to the error word and branch to ``bail``."""
    cnt = a.r()
    p = a.r("p")
    q = a.r("p")
    top, done = a.L("w"), a.L("wd")
    a(f"mov.u32 {cnt}, 0;")
    a.label(top)
    a(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar}], {parity}, {WAIT_HINT_NS};")
    a(f"@{p} bra {done};")
    a(f"add.u32 {cnt}, {cnt}, 1;")
    a(f"setp.lt.u32 {q}, {cnt}, {WAIT_LIMIT};")
    a(f"@{q} bra {top};")
    a(f"st.global.u32 [{err}], {code};")
    a(f"bra {bail};")
    a.label(done)


def wait_bar_warp(a: Asm, bar: str, parity: str, err: str, code: int, bail: str) -> None:
    """Like :func:`wait_bar`, for a whole warp: the exit decision is a ``vote.sync.all`` so every lane
    leaves the loop together (the TMEM loads that follow need a converged warp)."""
    cnt = a.r()
    p = a.r("p")
    pa = a.r("p")
    q = a.r("p")
    top, done = a.L("ww"), a.L("wwd")
    a(f"mov.u32 {cnt}, 0;")
    a.label(top)
    a(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar}], {parity}, {WAIT_HINT_NS};")
    a(f"vote.sync.all.pred {pa}, {p}, -1;")
    a(f"@{pa} bra {done};")
    a(f"add.u32 {cnt}, {cnt}, 1;")
    a(f"setp.lt.u32 {q}, {cnt}, {WAIT_LIMIT};")
    a(f"@{q} bra {top};")
    a(f"st.global.u32 [{err}], {code};")
    a(f"bra {bail};")
    a.label(done)
