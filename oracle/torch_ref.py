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


def attention(Q, K, V, causal=True, scale=None, mask=None):
    """SDPA in float64; ``mask`` is a boolean [S, S] tensor, True where the key takes part."""
    import torch
    q, k, v = Q.double(), K.double(), V.double()
    d = q.shape[-1]
    s = (q @ k.transpose(-1, -2)) * (scale if scale is not None else 1.0 / math.sqrt(d))
    if causal:
        n = s.shape[-1]
        s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    if mask is not None:
        s = s.masked_fill(~mask.bool(), float("-inf"))
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
    if fam == "corpus":
        return CORPUS[problem.params["expr"]](tensors, problem.params)
    raise ValueError(f"no source expression for family {fam!r}")


# ---- the coverage corpus (emmy_ptx_b200/corpus.py): each kernel's torch source expression ----------


def _rmsnorm(t, p):
    import torch
    x = t["x"].double()
    return {"y": x / torch.sqrt((x * x).mean(-1, keepdim=True) + p["eps"]) * t["w"].double()}


def _layernorm(t, p):
    import torch
    x = t["x"].double()
    return {"y": torch.nn.functional.layer_norm(x, (x.shape[-1],), t["g"].double(), t["b"].double(), p["eps"])}


def _intops(t, p):
    import torch
    x, y = t["x"].long(), t["y"].long()
    q = torch.div(x, 3, rounding_mode="trunc")
    r = x - q * 3
    return {"z": torch.where(x > 4, x & y, (x | y) - 3), "s": torch.sign(x), "w": torch.maximum(q, r) + (y << 2),
            "bd": torch.where(x > 10, 2, torch.where(x > 0, 1, 0))}


def _mathzoo(t, p):
    import torch
    F = torch.nn.functional
    x, z = t["x"].double(), t["z"].double()
    p1 = x.abs() + 0.5
    cols = [torch.tanh(x), torch.sigmoid(x), F.silu(x), F.softplus(x), torch.erf(x), x.abs(), 1 / x,
            torch.sign(x), x * x, torch.floor(x), torch.log(p1), torch.log2(p1), torch.rsqrt(p1),
            torch.pow(p1, z), torch.floor(x / p1), torch.fmod(x, p1),
            torch.maximum(x, z), torch.minimum(x, z)]
    return {"y": torch.stack(cols, 1).reshape(-1)}


def _chain(t, p):
    import torch
    prod = t["a"].double() * t["b"].double()
    return {"t": prod, "y": torch.relu(prod + t["c"].double())}


def _where_pos(t, p):
    import torch
    x = t["x"].double()
    return {"mask": (x > 0).to(torch.uint8), "y": torch.where(x > 0, x, torch.zeros_like(x))}


def _cond(t, p):
    import torch
    x = t["x"].double()
    return {"y": torch.where(x >= 0, torch.sqrt(x.clamp_min(0)), -0.5 * x)}


def _gelu(t, p):
    import torch
    x = t["x"].double()
    return {"y": torch.nn.functional.gelu(x), "yt": torch.nn.functional.gelu(x, approximate="tanh")}


def _exprs(t, p):
    import torch
    x = t["x"].double()
    rows, cols = x.shape
    r = torch.arange(rows, dtype=torch.float64)[:, None]
    c = torch.arange(cols, dtype=torch.float64)[None, :]
    w = (r * cols + c).float().double() * 0.01
    tt = torch.where(c < 32, x, torch.zeros_like(x)) + w
    e = 0.5 * torch.exp(x)
    pa = (x > 0) & (c < 48)
    return {"y": torch.where(~pa, e, tt)}


def _special(t, p):
    """The special-value kernel in float64, under the PTX rules the IR lowers to: max/min return the
    non-NaN operand, comparisons with NaN are false (including NaN != NaN)."""
    import torch
    x = t["x"].double()
    nan = torch.isnan(x)
    return {"relu": torch.where(nan, torch.zeros_like(x), x.clamp_min(0.0)),
            "mn": torch.where(nan, torch.ones_like(x), x.clamp_max(1.0)),
            "ex": torch.exp(x), "lg": torch.log(x), "sq": torch.sqrt(x), "rc": 1.0 / x,
            "wh": torch.where(x > 0, x, -torch.ones_like(x)),
            "nanm": nan.to(torch.uint8), "nem": torch.zeros_like(x, dtype=torch.uint8),
            "xb": x * 2.0}


def _special16(t, p):
    """The 16-bit special-value kernel in float64 (max returns the non-NaN operand)."""
    import torch
    xb, xh = t["xb"].double(), t["xh"].double()
    nan = torch.isnan(xb)
    return {"yb": torch.where(nan, torch.zeros_like(xb), xb.clamp_min(0.0)), "yh": xh * 2.0,
            "nanb": nan.to(torch.uint8)}


CORPUS = {
    "special": _special,
    "special16": _special16,
    "rmsnorm": _rmsnorm,
    "layernorm": _layernorm,
    "logsoftmax": lambda t, p: {"y": __import__("torch").log_softmax(t["x"].double(), -1)},
    "colsum": lambda t, p: {"out": t["x"].double().sum(0)},
    "midsum": lambda t, p: {"out": t["x"].double().sum(1)},
    "tri": lambda t, p: {"y": t["x"].double().cumsum(0)},
    "cumsum": lambda t, p: {"y": t["x"].double().cumsum(-1)},
    "intops": _intops,
    "gelu_f16": _gelu,
    "mask": _where_pos,
    # f64 buffers are computed in f32 registers by the reference (narrowed at the load)
    "f64": lambda t, p: {"y": (t["x"].float() * 2.5 + 1.0).double()},
    "cond": _cond,
    "mathzoo": _mathzoo,
    "hypot": lambda t, p: {"y": __import__("torch").hypot(t["x"].double(), t["z"].double())},
    "exprs": _exprs,
    "chain": _chain,
    "hist": lambda t, p: {"hist": __import__("torch").bincount(t["x"].long() % p["bins"], minlength=p["bins"])},
    "bcast3d": lambda t, p: {"y": __import__("torch").relu(t["x"].double() * t["w"].double()[:, None, None]
                                                           + t["bias"].double()[None, None, :])},
    "minmax": lambda t, p: {"mx": t["x"].double().amax(-1), "mn": t["x"].double().amin(-1)},
    "softmax3d": lambda t, p: {"y": __import__("torch").softmax(t["x"].double(), -1)},
    "argmax": lambda t, p: {"idx": t["x"].double().argmax(-1), "cnt": (t["x"].double() > p["thresh"]).sum(-1)},
    "varstd": lambda t, p: {"var": t["x"].double().var(-1), "std": t["x"].double().std(-1)},
    "groupnorm": lambda t, p: {"y": __import__("torch").nn.functional.group_norm(t["x"].double(), p["groups"],
                                                                                 eps=p["eps"])},
    "pad": lambda t, p: {"y": __import__("torch").nn.functional.pad(t["x"].double(), (p["left"], p["right"]))},
    "logsumexp": lambda t, p: {"y": __import__("torch").logsumexp(t["x"].double(), -1)},
    "matmul": lambda t, p: {"C": t["A"].double() @ t["B"].double()},
    "softmax_mid": lambda t, p: {"y": __import__("torch").softmax(t["x"].double(), 1)},
    "scanprod": lambda t, p: {"cm": __import__("torch").cummax(t["x"].double(), -1).values,
                              "pr": t["x"].double().prod(-1)},
    # torch's posinf / neginf defaults for a float32 tensor: the largest finite f32 and its negative
    "sdpa": lambda t, p: {"O": attention(t["Q"], t["K"], t["V"], p["causal"], p["scale"],
                                         t["M"] if p.get("mask") else None)},
    "nan_to_num": lambda t, p: {"y": __import__("torch").nan_to_num(t["x"]).double()},
    "logaddexp": lambda t, p: {"y": __import__("torch").logaddexp(t["a"].double(), t["b"].double())},
    "elu_selu": lambda t, p: {"elu": __import__("torch").nn.functional.elu(t["x"].double()),
                              "selu": __import__("torch").nn.functional.selu(t["x"].double())},
    "any": lambda t, p: {"out": (t["x"].double() > p["thresh"]).any(-1).to(__import__("torch").uint8)},
    "l2norm": lambda t, p: {"y": __import__("torch").nn.functional.normalize(t["x"].double(), dim=-1,
                                                                             eps=p["eps"])},
}
