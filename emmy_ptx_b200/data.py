"""Seeded synthetic inputs for a :class:`~.irgen.Problem` (the benchmark's data source).

Inputs are drawn on the CPU in fp32 from ``torch.Generator().manual_seed(crc32(name) ^ 1234)``
(the per-tensor seed rule of tools/oracle.py:191) and then cast, so the host oracle and the GPU
see identical bits.  Outputs start as zeros.
"""
from __future__ import annotations

import math

import numpy as np

TORCH_DTYPE = {}


def torch_dtype(dt: str):
    import torch
    return {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "i32": torch.int32,
            "f64": torch.float64, "u8": torch.uint8}[dt]


def make_tensor(spec, device="cpu", seed_offset: int = 0):
    """One argument tensor, drawn from the spec's distribution (or zeros for outputs)."""
    import torch
    shape = tuple(spec.shape)
    if spec.output or spec.dist[0] == "zeros":
        return torch.zeros(shape, dtype=torch_dtype(spec.dtype), device=device)
    g = torch.Generator().manual_seed((spec.seed + seed_offset) & 0x7FFFFFFFFFFFFFFF)
    kind = spec.dist[0]
    if kind == "normal":
        t = torch.randn(shape, generator=g, dtype=torch.float32) * float(spec.dist[1])
    elif kind == "uniform":
        lo, hi = spec.dist[1], spec.dist[2]
        t = torch.rand(shape, generator=g, dtype=torch.float32) * (hi - lo) + lo
    elif kind == "randint":
        t = torch.randint(int(spec.dist[1]), int(spec.dist[2]), shape, generator=g, dtype=torch.int32)
    elif kind == "special":
        # normal values with IEEE special and boundary values at fixed positions (flat index i):
        # NaN, +inf, -inf, +0, a magnitude whose exp overflows, and a small negative number
        t = torch.randn(shape, generator=g, dtype=torch.float32) * float(spec.dist[1])
        flat = t.reshape(-1)
        i = torch.arange(flat.numel())
        for mod, rem, val in ((17, 3, math.nan), (23, 5, math.inf), (29, 7, -math.inf), (31, 11, 0.0),
                              (37, 13, 1e30), (41, 17, -1e-3)):
            flat[(i % mod) == rem] = val
    else:
        raise ValueError(f"unknown distribution {spec.dist!r}")
    t = t.to(torch_dtype(spec.dtype))
    return t.to(device) if device != "cpu" else t


def make_inputs(problem, device="cpu", seed_offset: int = 0) -> dict:
    """Every argument of the problem as a tensor: seeded inputs, zeroed outputs."""
    return {a.name: make_tensor(a, device, seed_offset) for a in problem.args}


def to_numpy_storage(t) -> np.ndarray:
    """A flat numpy array in the oracle's storage format (16-bit floats as raw uint16 bits)."""
    import torch
    t = t.detach().cpu().contiguous().reshape(-1)
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def from_numpy_storage(a: np.ndarray, dt: str):
    """The inverse of :func:`to_numpy_storage`."""
    import torch
    if dt in ("bf16", "f16"):
        return torch.from_numpy(a.view(np.int16).copy()).view(torch_dtype(dt))
    return torch.from_numpy(a.copy())
