"""Regenerate the golden fixtures under tests/golden (run where the reference checkout exists).

    python tests/golden/make_golden.py --reference PATH [--only small|full|all]
    EMMY_REFERENCE=PATH python tests/golden/make_golden.py

PATH is a checkout of fanjialin8-create/emmy-ptx (the directory holding its ``compile.py``).

For every small configuration in ``emmy_ptx_b200.irgen.SMALL`` and every coverage kernel in
``emmy_ptx_b200.corpus.CORPUS`` it writes

* ``ref_ptx/<key>.ptx`` — the PTX the *reference* emitter (``compile.py`` of
  fanjialin8-create/emmy-ptx, run unmodified through ``emmy_shim``'s ``Graph.from_dict``) writes
  for that IR.  On a GPU it is run on the same seeded inputs as this backend and the oracle, so
  it pins the oracle to the reference's own behaviour.  PTX that fails the static def-use check
  (``emmy_ptx_b200.codegen.ptxcheck``: a register read before any write on some path) is not
  kept, and neither is PTX for IR the reference rejects; the manifest records why
  (``ref_unsafe`` / ``ref_error``).
* ``vectors/<key>.npz`` — the float64 source-expression result (``oracle/torch_ref.py``) on the
  seeded inputs, stored as float64, and an input checksum.
* ``manifest.json`` — a hash of each IR, so a fixture made from a different IR is detected.

For every BASELINE configuration at full size (``irgen.FULL``) it writes ``ref_ptx_full/<key>.ptx``:
the reference emitter's PTX for the full-size IR, which ``bench.py`` launches with the same
geometry and buffers as this backend's kernel to time the reference's own kernels on the GPU
(``ref_ptx_full/manifest.json`` holds the IR hashes).
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))


def ir_hash(graph: dict, meta: dict) -> str:
    blob = json.dumps({"graph": graph, "meta": meta}, sort_keys=True).encode()
    return hashlib.sha256(blob).hexdigest()[:16]


def input_digest(tensors: dict) -> str:
    from emmy_ptx_b200.data import to_numpy_storage
    h = hashlib.sha256()
    for name in sorted(tensors):
        h.update(name.encode())
        h.update(to_numpy_storage(tensors[name]).tobytes())
    return h.hexdigest()[:16]


def _ptxas_error(ptx: str) -> str:
    """The first error line ptxas prints for ``ptx`` targeting sm_100a, or '' when it assembles."""
    import shutil
    ptxas = shutil.which("ptxas") or "/usr/local/cuda/bin/ptxas"
    with tempfile.TemporaryDirectory() as td:
        src = Path(td) / "k.ptx"
        src.write_text(ptx)
        r = subprocess.run([ptxas, "-arch=sm_100a", str(src), "-o", str(Path(td) / "k.cubin")],
                           capture_output=True, text=True)
    if r.returncode == 0:
        return ""
    lines = [ln.split("k.ptx", 1)[-1].strip(" ,") for ln in r.stderr.splitlines() if "error" in ln]
    return lines[0] if lines else f"exit status {r.returncode}"


def reference_ptx(compile_py: Path, env: dict, p) -> tuple[str | None, str]:
    """The reference emitter's PTX for problem ``p`` (its IR and meta.json in a scratch directory),
    or (None, why) when the reference rejects the IR or writes PTX that must not run."""
    from emmy_ptx_b200.codegen.ptxcheck import undefined_uses
    with tempfile.TemporaryDirectory() as td:
        ir = Path(td) / f"{p.entry}.ir.json"
        ir.write_text(json.dumps(p.graph))
        (Path(td) / "meta.json").write_text(json.dumps(p.meta()))
        r = subprocess.run([sys.executable, str(compile_py), str(ir)], capture_output=True, text=True, env=env)
    if r.returncode != 0:
        return None, (r.stderr.strip().splitlines() or ["exit status %d" % r.returncode])[-1]
    if _ptxas_error(r.stdout):
        return None, "ptxas: " + _ptxas_error(r.stdout)
    if undefined_uses(r.stdout):
        entry, _, reg, text = undefined_uses(r.stdout)[0]
        return None, f"unsafe: {entry}: {reg} read before any write on some path: {text.strip()}"
    return r.stdout, ""


def write_full(compile_py: Path, env: dict) -> int:
    """``ref_ptx_full/<key>.ptx`` for every full-size BASELINE configuration."""
    from emmy_ptx_b200 import irgen
    out = HERE / "ref_ptx_full"
    out.mkdir(exist_ok=True)
    manifest = {}
    for key, mk in irgen.FULL.items():
        p = mk()
        ptx, why = reference_ptx(compile_py, env, p)
        rec = {"ir": ir_hash(p.graph, p.meta()), "entry": p.entry}
        if ptx is None:
            rec["ref_error"] = why
            print(f"full {key}: no reference PTX: {why}")
        else:
            (out / f"{key}.ptx").write_text(ptx)
            rec["ref_ptx_lines"] = ptx.count("\n")
            print(f"full {key}: {p.name} ref PTX {rec['ref_ptx_lines']} lines")
        manifest[key] = rec
    (out / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    return 0


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("EMMY_REFERENCE"),
                    help="checkout of the reference (the directory holding compile.py); or set EMMY_REFERENCE")
    ap.add_argument("--only", default="all", choices=["all", "small", "full"])
    args = ap.parse_args()
    if not args.reference:
        print("give the reference checkout with --reference PATH or EMMY_REFERENCE", file=sys.stderr)
        return 2
    import numpy as np
    from emmy_ptx_b200 import irgen, corpus, data
    from emmy_ptx_b200.codegen.ptxcheck import undefined_uses
    from oracle import torch_ref

    compile_py = Path(args.reference) / "compile.py"
    if not compile_py.exists():
        print(f"reference compile.py not found at {compile_py}", file=sys.stderr)
        return 2
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(HERE / "emmy_shim"), str(ROOT)]))
    if args.only in ("all", "full"):
        write_full(compile_py, env)
    if args.only == "full":
        return 0
    (HERE / "ref_ptx").mkdir(exist_ok=True)
    (HERE / "vectors").mkdir(exist_ok=True)
    manifest = {}
    for key, mk in {**irgen.SMALL, **corpus.CORPUS}.items():
        p = mk()
        meta = p.meta()
        with tempfile.TemporaryDirectory() as td:
            ir = Path(td) / f"{p.entry}.ir.json"
            ir.write_text(json.dumps(p.graph))
            (Path(td) / "meta.json").write_text(json.dumps(meta))
            r = subprocess.run([sys.executable, str(compile_py), str(ir)], capture_output=True, text=True, env=env)
        rec = {"ir": ir_hash(p.graph, meta), "entry": p.entry}
        if r.returncode != 0:
            # the reference rejects (or crashes on) this IR: record its last error line, keep no PTX
            last = (r.stderr.strip().splitlines() or ["exit status %d" % r.returncode])[-1]
            rec["ref_error"] = last
            stale = HERE / "ref_ptx" / f"{key}.ptx"
            if stale.exists():
                stale.unlink()
            print(f"{key}: reference emitter failed: {last}")
        elif _ptxas_error(r.stdout):
            # the reference wrote PTX that does not assemble for the GPU (the JIT rejects it the same way)
            rec["ref_error"] = "ptxas: " + _ptxas_error(r.stdout)
            stale = HERE / "ref_ptx" / f"{key}.ptx"
            if stale.exists():
                stale.unlink()
            print(f"{key}: reference PTX does not assemble: {rec['ref_error']}")
        elif undefined_uses(r.stdout):
            # a register read before any write on some path: running it could fault the GPU, so the
            # PTX is not kept (nothing can launch it) and the finding is recorded instead
            entry, _, reg, text = undefined_uses(r.stdout)[0]
            rec["ref_unsafe"] = f"{entry}: {reg} read before any write on some path: {text.strip()}"
            stale = HERE / "ref_ptx" / f"{key}.ptx"
            if stale.exists():
                stale.unlink()
            print(f"{key}: reference PTX not kept: {rec['ref_unsafe']}")
        else:
            (HERE / "ref_ptx" / f"{key}.ptx").write_text(r.stdout)
            rec["ref_ptx_lines"] = r.stdout.count("\n")
            print(f"{key}: {p.name} ref PTX {r.stdout.count(chr(10))} lines")
        t = data.make_inputs(p)
        ref = torch_ref.reference(p, t)
        np.savez_compressed(HERE / "vectors" / f"{key}.npz",
                            **{k: v.double().numpy() for k, v in ref.items()})
        rec["inputs"] = input_digest(t)
        manifest[key] = rec
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
