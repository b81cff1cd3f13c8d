"""``emmy_ptx``: the module entry point of the B200 backend (the reference's package name).

``python -m emmy_ptx kernel.ir.json > out.ptx`` behaves like ``python compile.py``;
``emmy_ptx.compile_ir(graph_or_path)`` returns the PTX text.  The implementation lives in
:mod:`emmy_ptx_b200`.
"""
from emmy_ptx_b200.compiler import compile_ir as _compile_ir, compile_graph, CompiledModule  # noqa: F401
from emmy_ptx_b200.ir import Graph  # noqa: F401


def compile_ir(graph_or_path, meta=None) -> str:
    """PTX text for an IR path (sibling meta.json is read), JSON dict or Graph."""
    return _compile_ir(graph_or_path, meta).ptx
