"""Module writer: header, shared declarations, entries, and the launch record of each kernel.

The PTX text is the drop-in output (``python compile.py ir.json > out.ptx``, compile.py:1780-1789).
Each entry is preceded by one comment line ``// emmy-b200-kernel {json}`` carrying what the
launcher needs that PTX cannot express: grid/block, dynamic shared memory, parameter order,
the base alignment each pointer must have, outputs to zero before launch, and any TMA
descriptors to encode.  Comments are ignored by ptxas and the driver JIT.
"""
from __future__ import annotations

import json
import os

PTX_VERSION = "8.8"
TARGET = "sm_100a"
MARK = "// emmy-b200-kernel "


def shared_decls(built: list[dict]) -> list[str]:
    out = []
    for b in built:
        if b.get("raw_entry"):
            out.extend(b.get("raw_decls") or [])
            continue
        if b["dyn"]:
            out.append(f".extern .shared .align 1024 .b8 {b['pool_name']}[];")
        else:
            for sym, off, (ext, dt, align) in b["smem"]:
                n = 1
                for e in ext:
                    n *= e
                from ..ir import dt_bytes
                al = max(align or 0, 16)
                out.append(f".shared .align {al} .b8 {sym}[{n * dt_bytes(dt)}];")
    return out


def launch_record(b: dict) -> dict:
    rec = {
        "entry": b["name"],
        "params": b["params"],
        "grid": b.get("grid") or [],
        "block": b.get("block") or [],
        "dyn_smem": int(b.get("dyn_smem", 0)),
        "align": b.get("align", {}),
        "zero_outputs": b.get("zero_outputs", []),
        "kind": b.get("kind", "generic"),
    }
    for k in ("tmaps", "cluster", "extra", "pdl", "scratch", "stream", "after", "exchange", "self_zeroing"):
        if b.get(k):
            rec[k] = b[k]
    if b.get("carveout") is not None:
        rec["carveout"] = int(b["carveout"])
    return rec


def entry_text(b: dict) -> list[str]:
    if b.get("raw_entry"):
        return [MARK + json.dumps(launch_record(b), sort_keys=True)] + b["raw_entry"]
    params = [f"\t.param .u64 p_{n}" for n in b["params"]]
    # extension of the reference's ABI for promoted stripes: the TMA descriptors after arg_order, then
    # the status word the bounded waits write
    params += [f"\t.param .align 64 .b8 p_{spec['name']}[128]" for spec in b.get("tmaps") or []]
    params += [f"\t.param .u64 {'p_err' if spec.get('kind') == 'errword' else spec['param']}"
               for spec in b.get("extra") or []]
    out = [MARK + json.dumps(launch_record(b), sort_keys=True)]
    out.append(f".visible .entry {b['name']}(\n" + ",\n".join(params) + "\n)")
    if b.get("reqntid"):
        out.append(f".reqntid {int(b['reqntid'])}, 1, 1")
    elif b.get("block") and not os.environ.get("PTX_NO_MAXNTID"):
        dims = [str(int(d)) for d in b["block"]] + ["1"] * (3 - len(b["block"]))
        out.append(".maxntid " + ", ".join(dims[:3]))
    cap = os.environ.get("PTX_MAXNREG")
    if cap:
        out.append(f".maxnreg {int(cap)}")
    out.append("{")
    out.extend(b["decls"])
    out.extend(b["body"])
    out.append("\tret;")
    out.append("}")
    return out


def module_text(built: list[dict]) -> str:
    lines = [f".version {PTX_VERSION}", f".target {TARGET}", ".address_size 64", ""]
    decls = shared_decls(built)
    lines.extend(decls)
    if decls:
        lines.append("")
    for b in built:
        lines.extend(entry_text(b))
        lines.append("")
    return "\n".join(lines).rstrip("\n") + "\n"


def parse_records(ptx: str) -> list[dict]:
    """The launch records embedded in a module's text, in entry order."""
    recs = []
    for line in ptx.splitlines():
        if line.startswith(MARK):
            recs.append(json.loads(line[len(MARK):]))
    return recs
