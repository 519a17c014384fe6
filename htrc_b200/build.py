"""Build libhtrc_flat.so in-tree with nvcc for sm_100a (no GPU needed: nvcc cross-compiles).

    python -m htrc_b200.build [--verbose]

The library is a plain C-ABI shared object (include/htrc_flat.h); Python loads it with ctypes.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libhtrc_flat.so"
SOURCES = ["api.cu", "prep.cu", "stats.cu", "rowmax.cu", "route.cu", "tile.cu", "kmeans.cu", "quant.cu", "static_ws.cu", "fp8.cu", "tree.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def build(verbose: bool = False, ptxas_verbose: bool = False, force: bool = False) -> Path:
    srcs = [CSRC / s for s in SOURCES]
    deps = srcs + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    if LIB.exists() and not force and all(LIB.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return LIB
    out_dir = ROOT / "_build"
    out_dir.mkdir(exist_ok=True)
    objs = []
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                    "-I", str(ROOT / "include")]
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]
    for s in srcs:
        o = out_dir / (s.stem + ".o")
        cmd = [nvcc_path(), "-c", str(s), "-o", str(o)] + flags
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(o))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc_path(), "-shared", "-o", str(tmp)] + objs + ARCH + ["-Xcompiler", "-fPIC"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print registers/spills/shared memory per kernel")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.verbose, a.ptxas, a.force or a.ptxas))


if __name__ == "__main__":
    sys.exit(main())
