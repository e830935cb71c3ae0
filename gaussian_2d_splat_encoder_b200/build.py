"""Build libgsplat_b200.so in-tree with nvcc for sm_100a (no JIT cache, no torch extension).

    python -m gaussian_2d_splat_encoder_b200.build
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
ROOT = PKG.parent
OUT = PKG / "libgsplat_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", str(ROOT / "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(CSRC.glob("*.cu"))


def build(verbose: bool = False, force: bool = False) -> Path:
    srcs = sources()
    deps = srcs + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "gsplat_b200.h", Path(__file__)]
    if OUT.exists() and not force and all(OUT.stat().st_mtime >= p.stat().st_mtime for p in deps):
        return OUT
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    for s in srcs:
        o = objdir / (s.stem + ".o")
        cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(s), "-o", str(o)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(o))
    tmp = OUT.with_suffix(".so.tmp")
    subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *objs], check=True)
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
