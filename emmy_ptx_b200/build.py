"""Build the in-tree native library ``libemmy_launch.so`` (host C++ over libcuda/NCCL).

The kernels themselves are PTX emitted at run time by :mod:`emmy_ptx_b200.compiler` and
JIT-compiled by the driver (or assembled by ``ptxas -arch=sm_100a``); this library is the C-ABI
launcher.  It is compiled with nvcc (host code plus any device code in ``csrc``) for sm_100a
and written next to the package so it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libemmy_launch.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cpp")) + list(CSRC.glob("*.cu")))


def stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = sources() + [ROOT / "include" / "emmy_launch.h"] + list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > t for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile ``csrc/*`` into ``libemmy_launch.so`` (skipped when up to date)."""
    if not force and not stale():
        return LIB
    cmd = [nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-I", str(ROOT / "include"), "-I", "/usr/local/cuda/include",
           *[str(s) for s in sources()], "-o", str(LIB) + ".tmp", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("building libemmy_launch.so failed:\n" + r.stdout + r.stderr)
    if verbose:
        print(r.stdout + r.stderr)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose=True))
