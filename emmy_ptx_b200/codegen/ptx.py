"""PTX text builder: typed virtual registers, labels, nested code segments and scoped caches.

Code is emitted into a tree of :class:`Segment` lists.  Each open loop owns a *preheader*
segment that sits just before its header; a value that is invariant in a loop is emitted into
the preheader of the outermost loop it is invariant in (loop-invariant code motion at emission
time, no after-the-fact line surgery).  Caches of materialised values are scoped: entering a
branch, an else-branch or a loop body pushes a scope, leaving pops it, so a cached register is
reused only where its definition dominates the use (the soundness rule the reference enforces
by clearing its cache at every merge and back edge, compile.py:1118-1122, 1493-1496, 430-434).
"""
from __future__ import annotations

import struct

# register classes -> (prefix, PTX declaration type)
REG_CLASSES = {
    "pred": ("%p", ".pred"),
    "b16": ("%h", ".b16"),
    "b32": ("%r", ".b32"),
    "f32": ("%f", ".f32"),
    "b64": ("%rd", ".b64"),
}


def f32_imm(v: float) -> str:
    """An f32 immediate operand in PTX's exact hex form."""
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", float(v)))[0]


class Segment(list):
    """A list of PTX lines and nested segments, flattened at the end."""

    def flatten(self, out: list) -> list:
        for item in self:
            if isinstance(item, Segment):
                item.flatten(out)
            else:
                out.append(item)
        return out


class LoopFrame:
    __slots__ = ("pre", "scope_index", "depth")

    def __init__(self, pre: Segment, scope_index: int, depth: int):
        self.pre = pre
        self.scope_index = scope_index
        self.depth = depth


class PtxBuilder:
    """Registers, labels, segments, scopes and loop frames for one kernel body."""

    def __init__(self) -> None:
        self.counts = {c: 0 for c in REG_CLASSES}
        self.root = Segment()
        self.cur = self.root
        self.scopes: list[dict] = [{}]
        self.loops: list[LoopFrame] = []
        self.labels = 0

    # -- registers and labels ------------------------------------------------------------
    def reg(self, cls: str) -> str:
        self.counts[cls] += 1
        return f"{REG_CLASSES[cls][0]}{self.counts[cls]}"

    def label(self, tag: str = "") -> str:
        self.labels += 1
        return f"$L{self.labels}{tag}"

    # -- emission -----------------------------------------------------------------------
    def emit(self, line: str, depth: int | None = None) -> None:
        """Append an instruction at the current point, or into the preheader of the loop at
        ``depth`` (0 = outside every loop: the preheader of the outermost loop)."""
        seg = self.cur
        if depth is not None and depth < len(self.loops):
            seg = self.loops[depth].pre
        seg.append(line if line.endswith(":") else "\t" + line)

    def place(self, label: str) -> None:
        self.cur.append(label + ":")

    @property
    def depth(self) -> int:
        return len(self.loops)

    # -- scoped caches ------------------------------------------------------------------
    def push_scope(self) -> None:
        self.scopes.append({})

    def pop_scope(self) -> None:
        self.scopes.pop()

    def lookup(self, key):
        for sc in reversed(self.scopes):
            hit = sc.get(key)
            if hit is not None:
                return hit
        return None

    def remember(self, key, value, depth: int | None = None) -> None:
        """Cache ``value`` in the scope where its definition point lives."""
        if depth is not None and depth < len(self.loops):
            self.scopes[self.loops[depth].scope_index][key] = value
        else:
            self.scopes[-1][key] = value

    # -- loops ----------------------------------------------------------------------------
    def open_loop(self) -> LoopFrame:
        pre = Segment()
        self.cur.append(pre)
        frame = LoopFrame(pre, len(self.scopes) - 1, len(self.loops))
        self.loops.append(frame)
        self.push_scope()
        return frame

    def close_loop(self) -> None:
        self.pop_scope()
        self.loops.pop()

    def lines(self) -> list[str]:
        return self.root.flatten([])

    def reg_decls(self) -> list[str]:
        out = []
        for cls, n in self.counts.items():
            if n:
                pre, ty = REG_CLASSES[cls]
                out.append(f"\t.reg {ty} {pre}<{n + 1}>;")
        return out
