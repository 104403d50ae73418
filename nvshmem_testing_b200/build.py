"""Build recipe for libmoe_ep.so (the C-ABI extension).

Compiles every CUDA source under ``csrc/`` for sm_100a with nvcc into one
in-tree shared library, ``nvshmem_testing_b200/_lib/libmoe_ep.so``.  The CUDA
runtime is linked statically and driver entry points are resolved at run
time, so the library loads on a host without a GPU driver.

Usage: ``python -m nvshmem_testing_b200.build [--force] [--verbose]``.
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
INCLUDE = ROOT / "include"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libmoe_ep.so"
SOURCES = ["route.cu", "fused.cu", "combine.cu", "router.cu", "mlp.cu", "driver.cu", "capi.cu", "noalloc.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libmoe_ep.so")
    return cand


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))
    return files


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(f.stat().st_mtime > t for f in _inputs())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile libmoe_ep.so if any input is newer than the library."""
    if not force and not needs_build():
        return LIB
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    nvcc = nvcc_path()
    objs = []
    common = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
                           "-I", str(INCLUDE), "-I", str(CSRC)]
    if ptxas_verbose:
        common += ["-Xptxas", "-v"]
    for s in SOURCES:
        obj = OUT_DIR / (Path(s).stem + ".o")
        cmd = [nvcc, "-c", str(CSRC / s), "-o", str(obj)] + common
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-o", str(tmp)] + [str(o) for o in objs] + ARCH_FLAGS + ["-cudart", "static"]
    if verbose:
        print(" ".join(cmd))
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    for o in objs:
        os.unlink(o)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args(argv)
    lib = build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas_verbose)
    print(lib)
    return 0


if __name__ == "__main__":
    sys.exit(main())
