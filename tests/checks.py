"""Tolerance policy shared by the parity tests (the bars the benchmark configurations state).

* integer and byte outputs (including predicates stored as u8): bit-exact;
* f32 fused / softmax / reduction outputs: relative 1e-5 (elementwise, with an absolute floor of
  1e-5 of the tensor's largest magnitude for entries near zero);
* f32 matmul / attention outputs: relative 1e-4 of max(|ref|, rms(ref)) — a K-term dot product's
  rounding error scales with the operands' norms, so entries that cancel to near zero are held to
  the tensor's typical magnitude;
* bf16 outputs: within one bf16 unit in the last place of the reference value (2**-7 relative)
  plus 1e-6 absolute — bf16 keeps 8 significant bits, so two correct f32 computations that differ
  in the last f32 bits can round to neighbouring bf16 values;
* bf16 attention from the tensor-core kernel: one bf16 unit of max(|ref|, rms of the query row).
  The kernel rounds the softmax weights P for the PV product (the tensor core multiplies operands of
  one type: f16 P with an f16 copy of V, 2**-12 relative, or P as two bf16 parts with bf16 V, 2**-14),
  which moves each term slightly before the f32 accumulation; an output element that happens to
  cancel to near zero is held to its row's magnitude (rows that attend to few keys have large outputs
  and the least averaging of that rounding).
"""
from __future__ import annotations

import torch

BF16_REL = 2.0 ** -7


def atol_for(problem) -> float:
    """An absolute floor for the coverage kernels (their ``atol``, 1e-6): approximate hardware math
    (ex2/lg2/rsqrt ``.approx``) near a zero of the function leaves an absolute error of a few f32
    units of 1.0, which no relative bound covers."""
    return problem.atol if problem.family == "corpus" else 0.0


def rtol_for(problem) -> float:
    """1e-4 for contractions (the batched matmul, attention and a coverage kernel marked as a
    contraction), 1e-5 for everything else."""
    if problem.family in ("bmm", "attention") or problem.params.get("contraction"):
        return 1e-4
    return 1e-5


def rms_floor_for(problem) -> bool:
    return problem.family == "attention" or bool(problem.params.get("attention"))


def compare(got: torch.Tensor, ref: torch.Tensor, dtype: str, rtol: float, what: str = "",
            rms_floor: bool = False, atol: float = 0.0) -> dict:
    g = got.detach().cpu()
    r = ref.detach().cpu()
    assert g.shape == r.shape, f"{what}: shape {tuple(g.shape)} vs {tuple(r.shape)}"
    if r.numel() == 0:
        return {"max_abs": 0.0}
    if dtype in ("i32", "i64", "u32", "u8", "i8", "bool"):
        eq = torch.equal(g.long(), r.long())
        assert eq, f"{what}: integer result differs: {g.reshape(-1)[:4].tolist()} vs {r.reshape(-1)[:4].tolist()}"
        return {"max_abs": 0.0}
    g = g.double()
    r = r.double()
    # special values must match exactly: NaN where the reference has NaN, the same infinities
    bad_nan = torch.isnan(g) != torch.isnan(r)
    assert not bad_nan.any(), f"{what}: NaN at {int(bad_nan.sum())} positions differs, first {int(bad_nan.reshape(-1).nonzero()[0])}"
    inf = torch.isinf(r)
    bad_inf = (torch.isinf(g) != inf) | (inf & (g != r))
    assert not bad_inf.any(), f"{what}: infinities differ at {int(bad_inf.sum())} positions"
    fin = torch.isfinite(r)
    err = (g - r).abs()
    err = torch.where(fin, err, torch.zeros_like(err))
    scale = r[fin].abs().max().item() if fin.any() else 0.0
    if dtype in ("bf16", "f16"):
        rel = BF16_REL if dtype == "bf16" else 2.0 ** -10
        if rms_floor:
            row_rms = torch.where(fin, r, torch.zeros_like(r)).pow(2).mean(dim=-1, keepdim=True).sqrt()
            bound = rel * torch.maximum(r.abs(), row_rms) + 1e-6
        else:
            bound = rel * r.abs() + 1e-6
    elif rtol >= 1e-4:
        rms = r[fin].pow(2).mean().sqrt().item() if fin.any() else 0.0
        bound = rtol * torch.clamp(r.abs(), min=rms) + 1e-30
    else:
        bound = rtol * r.abs() + rtol * 1e-5 * scale + 1e-30
    bound = bound + atol
    bad = err > bound
    n_bad = int(bad.sum().item())
    worst = int(torch.argmax((err / bound).reshape(-1)).item())
    assert n_bad == 0, (f"{what}: {n_bad}/{g.numel()} outside tolerance; worst at {worst}: "
                        f"got {g.reshape(-1)[worst].item()!r} want {r.reshape(-1)[worst].item()!r}")
    return {"max_abs": float(err.max().item()) if err.numel() else 0.0, "scale": scale}
