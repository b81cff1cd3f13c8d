"""CPU oracle (b): torch-CPU evaluation of each configuration's *source expression*, in float64.

TEST INFRASTRUCTURE ONLY (see oracle/interp.py for the import rule).  These are the expressions
the five benchmark IRs are lowered from; they are independent of the IR and of the interpreter,
so agreement between ``interp`` and these functions pins both the hand-authored IR and the
interpreter's restatement of the reference semantics.
"""
from __future__ import annotations

import math


def softmax(x):
    import torch
    return torch.softmax(x.double(), dim=-1)


def array_sum(x):
    import torch
    if x.dtype == torch.int32:
        return x.long().sum().reshape(1)
    return x.double().sum().reshape(1)


def fused(a, b, c, d):
    import torch
    return torch.relu(a.double() * b.double() + c.double()) * torch.exp(d.double())


def bmm(A, B):
    import torch
    return torch.bmm(A.double(), B.double())


def attention(Q, K, V, causal=True, scale=None):
    import torch
    q, k, v = Q.double(), K.double(), V.double()
    d = q.shape[-1]
    s = (q @ k.transpose(-1, -2)) * (scale if scale is not None else 1.0 / math.sqrt(d))
    if causal:
        n = s.shape[-1]
        mask = torch.ones(n, n, dtype=torch.bool).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    return torch.softmax(s, dim=-1) @ v


def reference(problem, tensors: dict):
    """The float64 source-expression result for a problem, keyed by output name."""
    fam = problem.family
    if fam == "softmax":
        return {"y": softmax(tensors["x"])}
    if fam == "sum":
        return {"out": array_sum(tensors["x"])}
    if fam == "fused":
        return {"y": fused(tensors["a"], tensors["b"], tensors["c"], tensors["d"])}
    if fam == "bmm":
        return {"C": bmm(tensors["A"], tensors["B"])}
    if fam == "attention":
        return {"O": attention(tensors["Q"], tensors["K"], tensors["V"], problem.params.get("causal", True),
                               problem.params.get("scale"))}
    raise ValueError(f"no source expression for family {fam!r}")
