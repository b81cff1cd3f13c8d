"""Clock64 timeline of the tensor-core attention: where each 64-row key/value block's cycles go.

This is the package's tracing tool: a user-run probe of a kernel's pipeline. Nothing on the compile or
launch path imports it, and the kernel carries the stamps only when it is built with ``trace=True``.

``python -m emmy_ptx_b200.timeline [--no-pingpong] [--bf16]`` runs config 5 (causal bf16 attention
[8, 32, 4096, 128]) once untraced for timing, then once with the kernel's trace option
(``attention_entry(..., trace=True)``: one u64 ``clock64`` stamp per event per kv block per CTA, taken
by one thread of each role) and prints per-event intervals (median, 10th and 90th percentile over
the steady-state blocks 4..55 of the longest CTAs).  Events per block: the issuers' iteration start,
K_(j+1) arrived, S(j+1) issued, V_j arrived, P_0(j) seen, PV_0 issued, P_1(j) seen, PV_1 issued; per
softmax tile: S ready, S loaded, row max, format known, MUFU turn taken, exps done, P stores issued,
P written.  The stamps cost a few percent of the kernel's speed (both timings are printed).
"""
from __future__ import annotations

import argparse
import json

import numpy as np

ISSUER = ["iteration start", "K(j+1) arrived", "S(j+1) issued", "V(j) arrived", "P0(j) seen", "PV0 issued",
          "P1(j) seen", "PV1 issued"]


def summarise(tr: np.ndarray, t_of_cta: np.ndarray) -> dict:
    """Interval statistics from a trace array [ctas, 66, 24] (see ``tc_attention.trace_events``)."""
    tr = tr.astype(np.int64)
    out = {"per_cta": {}, "intervals": {}}
    dur = tr[:, 65, 1] - tr[:, 65, 0]
    for tt in sorted(set(int(x) for x in t_of_cta)):
        d = dur[t_of_cta == tt]
        blocks = 4 * tt + 4
        out["per_cta"][f"t={tt} ({blocks} blocks)"] = {"cta_kclk": float(d.mean() / 1e3),
                                                       "clk_per_block": float(d.mean() / blocks)}
    tmax = int(t_of_cta.max())
    sel = np.where(t_of_cta == tmax)[0]
    hi = min(4 * tmax + 4 - 8, 56)
    r = np.concatenate([tr[c, 4:hi] for c in sel]).astype(np.float64)
    n = np.concatenate([tr[c, 5:hi + 1] for c in sel]).astype(np.float64)

    def put(name, x):
        out["intervals"][name] = {"median": float(np.median(x)), "p10": float(np.percentile(x, 10)),
                                  "p90": float(np.percentile(x, 90))}
    put("issuer 0 iteration", n[:, 0] - r[:, 0])
    for k in range(7):
        put(f"issuer: {ISSUER[k]} -> {ISSUER[k + 1]}", r[:, k + 1] - r[:, k])
    for ti, b in ((0, 8), (1, 16)):
        put(f"softmax {ti}: S ready -> loaded", r[:, b + 1] - r[:, b])
        put(f"softmax {ti}: loaded -> row max", r[:, b + 2] - r[:, b + 1])
        put(f"softmax {ti}: row max -> format known", r[:, b + 3] - r[:, b + 2])
        put(f"softmax {ti}: format known -> turn taken", r[:, b + 7] - r[:, b + 3])
        put(f"softmax {ti}: turn taken -> exps done", r[:, b + 4] - r[:, b + 7])
        put(f"softmax {ti}: exps done -> P stores issued", r[:, b + 5] - r[:, b + 4])
        put(f"softmax {ti}: P stores issued -> P written", r[:, b + 6] - r[:, b + 5])
        put(f"softmax {ti}: P written -> next S ready", n[:, b] - r[:, b + 6])
    put("P0(j) written -> issuer 0 sees it", r[:, 4] - r[:, 14])
    put("P1(j) written -> issuer 1 sees it", r[:, 6] - r[:, 22])
    return out


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--no-pingpong", action="store_true")
    ap.add_argument("--bf16", action="store_true", help="bf16 hi + lo P for every block (no value pre-pass)")
    ap.add_argument("--out", default=None, help="also write the summary as JSON here")
    args = ap.parse_args()
    import torch
    from . import irgen
    from .compiler import compile_graph
    from .ir import Graph
    from .kernels import tc_attention
    from .runtime import Executable
    p = irgen.attention_ir()
    shp = (p.params["batch"], p.params["heads"], p.params["seq"], p.params["dim"])
    flop = 4.0 * shp[0] * shp[1] * shp[3] * shp[2] * (shp[2] + 1) / 2
    g = torch.Generator(device="cuda").manual_seed(1)
    t = {n: torch.randn(shp, device="cuda", generator=g).to(torch.bfloat16) for n in "QKV"}
    t["O"] = torch.empty(shp, device="cuda", dtype=torch.bfloat16)
    res = {}
    for trace in (False, True):
        opts = {"attn_trace": trace, "attn_pingpong": not args.no_pingpong, "attn_half": not args.bf16}
        mod = compile_graph(Graph.from_dict(p.graph), p.meta(), opts)
        grid = mod.kernels[-1]["grid"][0]
        if trace:
            t["__trace"] = torch.zeros(grid * tc_attention.TRACE_SLOTS * tc_attention.TRACE_EVENTS,
                                       dtype=torch.int64, device="cuda")
        ex = Executable(mod)
        for _ in range(3):
            ex(t)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            ex(t)
        e1.record()
        torch.cuda.synchronize()
        ex.check()
        ms = e0.elapsed_time(e1) / 10
        res["traced" if trace else "untraced"] = {"ms": ms, "tflops": flop / ms / 1e9}
        if trace:
            tr = t.pop("__trace").cpu().numpy().reshape(grid, tc_attention.TRACE_SLOTS, tc_attention.TRACE_EVENTS)
            nt = shp[2] // 256
            t_of_cta = nt - 1 - np.arange(grid) // (shp[0] * shp[1])
            res["timeline"] = summarise(tr, t_of_cta)
        ex.close()
    for k in ("untraced", "traced"):
        print(f"{k:9s}: {res[k]['ms']:.4f} ms, {res[k]['tflops']:.1f} TFLOP/s")
    for k, v in res["timeline"]["per_cta"].items():
        print(f"  CTA {k:16s}: {v['cta_kclk']:7.1f} kclk, {v['clk_per_block']:6.0f} clk per kv block")
    for k, v in res["timeline"]["intervals"].items():
        print(f"  {k:50s} median {v['median']:7.0f}  p10 {v['p10']:7.0f}  p90 {v['p90']:7.0f}")
    if args.out:
        with open(args.out, "w") as f:
            json.dump(res, f, indent=1)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
