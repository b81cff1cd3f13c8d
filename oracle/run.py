"""Run the CPU oracle interpreter on a problem's tensors.

TEST INFRASTRUCTURE ONLY (see oracle/interp.py for the import rule).
"""
from __future__ import annotations

import numpy as np

from .interp import Interpreter


def oracle_outputs(problem, tensors: dict, blocks=None) -> dict:
    """Interpret the problem's IR on CPU copies of ``tensors``; returns output name -> tensor.

    Outputs listed in ``zero_outputs`` start at zero, like the launcher zeroes them; ``blocks``
    restricts execution to a subset of thread blocks (the bounded CPU-baseline sample).  A problem
    with a ``launches`` list (several kernels) runs each kernel in that order with its own grid and
    block, as the graph's launches run in stream order."""
    from emmy_ptx_b200.ir import Graph
    from emmy_ptx_b200.data import to_numpy_storage, from_numpy_storage
    graph = Graph.from_dict(problem.graph)
    bufs = {}
    for a in problem.args:
        arr = to_numpy_storage(tensors[a.name])
        if a.output:
            arr = np.zeros_like(arr)
        bufs[a.name] = arr
    launches = getattr(problem, "launches", None)
    if launches:
        nodes = {nd.op.name: nd for nd in graph.kernels()}
        for entry, grid, block, _zero, _order in launches:
            Interpreter(graph, nodes[entry]).run(bufs, grid, block)
    else:
        Interpreter(graph).run(bufs, problem.grid, problem.block, blocks=blocks)
    out = {}
    for a in problem.outputs:
        out[a.name] = from_numpy_storage(bufs[a.name], a.dtype).reshape(a.shape)
    return out
