"""Test-only ``emmy.compiler.graph``: the reference emitter imports ``Graph`` from here
(compile.py:18) and calls ``Graph.from_dict`` (compile.py:1806).  It is this repository's own
loader, so the reference's emitter reads exactly the IR objects this backend reads."""
from emmy_ptx_b200.ir import Graph  # noqa: F401
