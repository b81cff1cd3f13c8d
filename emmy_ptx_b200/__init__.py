"""emmy_ptx_b200: a B200-native (sm_100a) backend for the Emmy kernel IR.

* :mod:`.ir` — ``Graph.from_dict`` and the IR classes (the input contract);
* :mod:`.compiler` — IR -> PTX (``compile_ir``), CUDA-core templates in :mod:`.codegen`,
  tensor-core lowerings in :mod:`.patterns`;
* :mod:`.launcher` / :mod:`.runtime` — the C-ABI launcher (``libemmy_launch.so``) and the
  executable that runs emitted modules on device tensors;
* :mod:`.irgen` — IR for the benchmark configurations; :mod:`.data` — their seeded inputs.
"""
from .compiler import compile_ir, compile_graph, CompiledModule  # noqa: F401
from .ir import Graph  # noqa: F401

__all__ = ["compile_ir", "compile_graph", "CompiledModule", "Graph"]
