"""The Emmy kernel-IR contract: ``Graph.from_dict`` and the statement / expression classes.

The reference backend reads the IR only through ``emmy.compiler.graph.Graph.from_dict``
(compile.py:18, compile.py:1806) and then dispatches on the *class name* of every statement
(compile.py:1129-1133) and expression (compile.py:682-719), reading fields with ``getattr``.
Emmy itself is not vendored, so this module is a loader written from the field list those
``getattr`` sites use.  Any object graph with these class names and fields is a drop-in.

Wire format (this loader's; Emmy's own codec is not available)::

    {"nodes": {name: {"op": "KernelOp" | "InputOp" | "ConstantOp",
                      "op_fields": {...},
                      "inputs": [name, ...],
                      "outputs": [{"name": str, "shape": [int, ...], "dtype": str}]}},
     "inputs": [name, ...], "outputs": [name, ...]}

Inside ``op_fields`` every IR object is a dict whose ``"kind"`` key is its class name
(``{"kind": "Load", "names": [...], ...}``).  Bare ints are integer immediates, bare strings
are SSA names, bare floats are f32 immediates — the same shorthands compile.py accepts
(``as_int`` compile.py:580-592, ``value`` compile.py:1229-1237, ``expr`` compile.py:694-697).
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Any

# Field schema per class: name -> (required fields, optional fields with defaults).
# The field names are the ones the reference emitter reads (compile.py getattr sites).
_STMT = {
    "Tile": (("axes", "body"), {}),                                              # compile.py:1135
    "Load": (("names", "input", "index"), {"dtype": None}),                      # compile.py:1159
    "Write": (("output", "values", "index", "value_dtype"), {"atomic": False}),  # compile.py:1346
    "Assign": (("name", "op", "args"), {"dtype": None}),                         # compile.py:1206
    "Let": (("name", "value", "dtype"), {}),                                     # compile.py:1262
    "Init": (("name", "dtype", "identity"), {}),                                 # compile.py:1276
    "Accum": (("name", "op", "value", "dtype"), {"base": None}),                 # compile.py:1328
    "Select": (("name", "branches"), {}),                                        # compile.py:1498
    "Cond": (("cond", "body"), {"else_body": None}),                             # compile.py:1480
    "Loop": (("axis", "body"), {"end": None, "unroll": False}),                  # compile.py:1588
    "StridedLoop": (("axis", "start", "step", "body"), {"end": None}),           # compile.py:1552
    "WarpShuffle": (("state",), {"state_b": (), "combine_states": (), "length": 32,
                                 "prefix": False}),                              # compile.py:1627
    "WarpBroadcast": (("state",), {"length": 32}),                               # compile.py:1656
    "TreeHalve": (("bufs", "state", "length"), {"state_b": (), "combine_states": (),
                                                "tid_var": "warp", "barrier_id": 0,
                                                "barrier_count": None}),         # compile.py:1670
    "CpAsyncCopy": (("smem", "smem_index", "src", "src_index", "nbytes"),
                    {"lane_index": None, "swizzle": "NONE", "valid": None}),     # compile.py:1449
    "CpAsyncCommit": ((), {}),                                                   # compile.py:1473
    "CpAsyncWait": ((), {"group": 0}),                                           # compile.py:1476
    "Smem": (("name", "extents", "dtype"), {"align": 0}),                        # compile.py:1384
    "Sync": ((), {"warp": False, "count": None, "barrier_id": 0}),               # compile.py:1390
    "ZeroPrologue": (("dst", "words"), {}),                                      # compile.py:1401
}
_EXPR = {
    "Var": (("name",), {}),                                                      # compile.py:685
    "Literal": (("value",), {"dtype": "f32"}),                                   # compile.py:724
    "Dim": (("value",), {}),                                                     # compile.py:692
    "BinaryExpr": (("op", "left", "right"), {}),                                 # compile.py:744
    "TernaryExpr": (("cond", "if_true", "if_false"), {}),                        # compile.py:847
    "FlatIndex": (("buffer", "index"), {}),                                      # compile.py:702
    "CastExpr": (("expr", "dtype"), {}),                                         # compile.py:706
    "Builtin": (("name",), {}),                                                  # compile.py:710
    "FuncCallExpr": (("name", "args"), {}),                                      # compile.py:857
}
_AUX = {
    "Axis": (("name", "extent"), {}),
    "SelectBranch": (("select", "value"), {}),
    # Assign's op (an elementwise implementation) and Accum's op (a reduction with identity).
    "ElementwiseImpl": (("name",), {}),
    "ReduceOp": (("name",), {"identity": None, "has_identity": False}),
}
_OPS = {
    "KernelOp": (("name", "body"), {}),
    "InputOp": ((), {}),
    "ConstantOp": ((), {"value": None}),
}

SCHEMA: dict[str, tuple[tuple[str, ...], dict[str, Any]]] = {**_STMT, **_EXPR, **_AUX, **_OPS}
STATEMENTS = frozenset(_STMT)
EXPRESSIONS = frozenset(_EXPR)


class IRError(ValueError):
    """Malformed IR: a missing field or an unknown class name."""


class IRObject:
    """Base of every loaded IR class.  Fields are plain attributes; ``kind`` is the class name."""

    kind = "IRObject"

    def __init__(self, **fields: Any) -> None:
        self.__dict__.update(fields)

    def __repr__(self) -> str:
        inner = ", ".join(f"{k}={v!r}" for k, v in self.__dict__.items() if k not in ("body", "else_body"))
        return f"{type(self).__name__}({inner})"

    def to_dict(self) -> dict:
        out = {"kind": type(self).__name__}
        for k, v in self.__dict__.items():
            out[k] = _dump(v)
        return out


_CLASSES: dict[str, type] = {}


def ir_class(name: str) -> type:
    """The loaded class for an IR kind (one Python class per name, so ``type(x).__name__`` works)."""
    cls = _CLASSES.get(name)
    if cls is None:
        if name not in SCHEMA:
            raise IRError(f"unknown IR class {name!r}")
        cls = type(name, (IRObject,), {"kind": name})
        _CLASSES[name] = cls
    return cls


def _load(obj: Any) -> Any:
    if isinstance(obj, dict):
        kind = obj.get("kind")
        if kind is None:
            return {k: _load(v) for k, v in obj.items()}
        required, optional = SCHEMA.get(kind, (None, None))
        if required is None:
            raise IRError(f"unknown IR class {kind!r}")
        fields = {}
        for f in required:
            if f not in obj:
                raise IRError(f"{kind} is missing required field {f!r}")
        for k, v in obj.items():
            if k == "kind":
                continue
            fields[k] = _load(v)
        for k, default in optional.items():
            fields.setdefault(k, default)
        return ir_class(kind)(**fields)
    if isinstance(obj, list):
        return [_load(v) for v in obj]
    return obj


def _dump(v: Any) -> Any:
    if isinstance(v, IRObject):
        return v.to_dict()
    if isinstance(v, (list, tuple)):
        return [_dump(x) for x in v]
    if isinstance(v, dict):
        return {k: _dump(x) for k, x in v.items()}
    return v


class Value:
    """One produced tensor: ``name``, ``shape`` (ints) and ``dtype`` (a dtype name)."""

    def __init__(self, name: str, shape, dtype: str) -> None:
        self.name = name
        self.shape = tuple(int(x) for x in shape)
        self.dtype = dtype

    def __repr__(self) -> str:
        return f"Value({self.name!r}, {self.shape}, {self.dtype!r})"


class Node:
    """A graph node: ``op`` (KernelOp / InputOp / ConstantOp), input names and output values."""

    def __init__(self, op: IRObject, inputs, outputs) -> None:
        self.op = op
        self.inputs = list(inputs)
        self.outputs = list(outputs)


class Graph:
    """``nodes`` (name -> Node), graph ``inputs`` and ``outputs`` (names)."""

    def __init__(self, nodes: dict[str, Node], inputs, outputs) -> None:
        self.nodes = nodes
        self.inputs = list(inputs)
        self.outputs = list(outputs)

    @classmethod
    def from_dict(cls, d: dict) -> "Graph":
        """Load the wire dict described in the module docstring (compile.py:1806)."""
        if not isinstance(d, dict) or "nodes" not in d:
            raise IRError("graph dict needs a 'nodes' mapping")
        nodes = {}
        for name, nd in d["nodes"].items():
            kind = nd.get("op")
            if kind not in _OPS:
                raise IRError(f"node {name!r}: unknown op {kind!r}")
            fields = dict(nd.get("op_fields") or {})
            fields["kind"] = kind
            op = _load(fields)
            outs = [Value(o["name"], o.get("shape", ()), o.get("dtype", "f32")) for o in nd.get("outputs") or []]
            nodes[name] = Node(op, nd.get("inputs") or [], outs)
        return cls(nodes, d.get("inputs") or [], d.get("outputs") or [])

    def to_dict(self) -> dict:
        nodes = {}
        for name, nd in self.nodes.items():
            fields = {k: _dump(v) for k, v in nd.op.__dict__.items()}
            nodes[name] = {
                "op": type(nd.op).__name__,
                "op_fields": fields,
                "inputs": list(nd.inputs),
                "outputs": [{"name": v.name, "shape": list(v.shape), "dtype": v.dtype} for v in nd.outputs],
            }
        return {"nodes": nodes, "inputs": list(self.inputs), "outputs": list(self.outputs)}

    def kernels(self) -> list[Node]:
        """Every KernelOp node, in graph order (compile.py:1807)."""
        return [n for n in self.nodes.values() if type(n.op).__name__ == "KernelOp"]

    def values(self) -> dict[str, Value]:
        out = {}
        for nd in self.nodes.values():
            for v in nd.outputs:
                out[v.name] = v
        return out


def load_graph(path_or_dict) -> Graph:
    """A Graph from a path to IR JSON, a JSON string, a wire dict, or a Graph."""
    if isinstance(path_or_dict, Graph):
        return path_or_dict
    if isinstance(path_or_dict, dict):
        return Graph.from_dict(path_or_dict)
    p = Path(path_or_dict)
    return Graph.from_dict(json.loads(p.read_text()))


def read_meta(ir_path) -> dict | None:
    """The sibling ``meta.json`` of an IR file, if any (compile.py:525-539, localrun.py:148)."""
    if ir_path is None:
        return None
    mpath = Path(ir_path).parent / "meta.json"
    if not mpath.exists():
        return None
    try:
        return json.loads(mpath.read_text())
    except (OSError, ValueError):
        return None


def kernel_meta(meta: dict | None, entry: str) -> dict | None:
    """The ``kernels[]`` record whose ``entry`` is this kernel's name (compile.py:536-538)."""
    if not meta:
        return None
    for k in meta.get("kernels", []):
        if k.get("entry") == entry:
            return k
    return None


# ---- dtype names (compile.py:28-53) ------------------------------------------------------

_DT_ALIASES = {
    "float32": "f32", "float16": "f16", "float64": "f64", "int32": "i32", "int64": "i64",
    "float": "f32", "double": "f64", "half": "f16", "int": "i32", "bfloat16": "bf16",
}
_DT_BYTES = {"f16": 2, "bf16": 2, "f32": 4, "f64": 8, "i32": 4, "int": 4, "i64": 8, "u32": 4, "u64": 8,
             "bool": 1, "bool8": 1, "i1": 1, "u8": 1, "i8": 1}


def dt_name(dt) -> str:
    """Canonical dtype name (``float32`` -> ``f32``), as compile.py:32-39."""
    n = getattr(dt, "name", None)
    if n is None:
        n = str(dt)
    return _DT_ALIASES.get(n, n)


def dt_bytes(dt) -> int:
    n = dt_name(dt)
    if n not in _DT_BYTES:
        raise IRError(f"unsupported dtype {n!r}")
    return _DT_BYTES[n]


def is_float_dt(dt) -> bool:
    return dt_name(dt) in ("f16", "bf16", "f32", "f64")


def dim_int(d) -> int:
    """An integer extent from an int or a ``Dim`` (compile.py:56-58)."""
    return int(getattr(d, "value", d))


def walk(body, fn) -> None:
    """Call ``fn`` on every statement, depth first, including nested bodies."""
    for st in body or ():
        fn(st)
        walk(getattr(st, "body", None), fn)
        walk(getattr(st, "else_body", None), fn)
