"""IR -> PTX: the drop-in replacement for the reference's ``Emitter``/``module_text`` pipeline.

``compile_ir`` mirrors compile.py:1802-1813: every KernelOp of the graph becomes one
``.visible .entry``; with several kernels, module-level shared symbols are namespaced
``<kernel>__`` (compile.py:1810-1811).  Before the statement-at-a-time lowering, each kernel is
offered to the pattern lowerings (:mod:`.patterns`): a dense contraction (batched matmul,
attention) that matches is emitted as a tcgen05/TMA kernel instead; anything that does not
match exactly stays on the CUDA-core path.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field
from pathlib import Path

from .ir import Graph, IRError, load_graph, read_meta, kernel_meta
from .codegen.generic import KernelEmitter, TmaNotProvable, Unsupported
from .codegen import module as modwriter


@dataclass
class CompiledModule:
    """PTX text plus the launch record of every entry (see :mod:`.codegen.module`)."""

    ptx: str
    kernels: list[dict] = field(default_factory=list)

    def kernel(self, entry: str | None = None) -> dict:
        if entry is None:
            return self.kernels[0]
        for k in self.kernels:
            if k["entry"] == entry:
                return k
        raise KeyError(entry)


def _use_patterns(options: dict) -> bool:
    if "patterns" in options:
        return bool(options["patterns"])
    return os.environ.get("EMMY_B200_PATTERNS", "1") != "0"


def compile_graph(graph: Graph, meta: dict | None = None, options: dict | None = None) -> CompiledModule:
    options = dict(options or {})
    kernels = graph.kernels()
    if not kernels:
        raise IRError("no KernelOp in this graph")
    multi = len(kernels) > 1
    built = []
    for node in kernels:
        km = kernel_meta(meta, node.op.name)
        prefix = f"{node.op.name}__" if multi else ""
        b = None
        if _use_patterns(options):
            from . import patterns
            b = patterns.try_lower(graph, node, km, prefix, options)
        if b is None:
            try:
                b = KernelEmitter(graph, node, km, prefix, options).build()
            except TmaNotProvable:
                # the stripes' TMA alignment is not provable: the same kernel with cp.async
                b = KernelEmitter(graph, node, km, prefix, {**options, "tma_stripes": False}).build()
        # a lowering may emit several entries for one KernelOp (a pre-pass before the main kernel)
        built.extend(b if isinstance(b, list) else [b])
    text = modwriter.module_text(built)
    return CompiledModule(text, modwriter.parse_records(text))


def compile_ir(source, meta: dict | None = None, options: dict | None = None) -> CompiledModule:
    """Compile IR given as a path (its sibling ``meta.json`` is read, compile.py:525-539), a
    JSON string path, a wire dict, or a loaded :class:`Graph`."""
    ir_path = None
    if isinstance(source, (str, os.PathLike)) and Path(source).exists():
        ir_path = Path(source)
    graph = load_graph(source)
    if meta is None and ir_path is not None:
        meta = read_meta(ir_path)
    return compile_graph(graph, meta, options)


def main(argv: list[str]) -> int:
    """``python compile.py path/to/kernel.ir.json > out.ptx`` (compile.py:1802-1813).

    Exactly one argument, else usage on stderr and exit 1.  PTX goes to stdout as ASCII; any
    unsupported construct is reported on stderr with exit status 1.
    """
    import sys
    if len(argv) != 2:
        sys.exit("usage: python compile.py path/to/kernel.ir.json > out.ptx")
    try:
        mod = compile_ir(argv[1])
    except (IRError, Unsupported) as exc:
        sys.exit(str(exc))
    out = mod.ptx
    out.encode("ascii")
    sys.stdout.write(out)
    return 0
