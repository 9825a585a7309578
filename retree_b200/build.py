"""Build the C-ABI kernel library ``retree_b200/lib/libretree_b200.so`` for sm_100a.

    python -m retree_b200.build [--force] [--ptxas-verbose]

Each ``csrc/*.cu`` is compiled by nvcc (``-gencode arch=compute_100a,code=sm_100a``,
CUDA runtime linked statically) into ``_build/`` at the repository root and the
objects are linked into one shared library with a plain C ABI
(``include/retree_b200.h``).  nvcc cross-compiles, so no GPU is needed.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
OUT_DIR = PKG / "lib"
LIB = OUT_DIR / "libretree_b200.so"
BUILD_DIR = ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", "-I", str(INCLUDE),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or install the CUDA toolkit)")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    """Compile every kernel source and link the shared library; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    srcs = _sources()
    headers = _headers()
    todo = [s for s in srcs if force or ptxas_verbose or _stale(BUILD_DIR / (s.stem + ".o"), [s, *headers])]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(lambda s: _compile(s, ptxas_verbose), todo):
                logs.append((obj.name, log))
    objs = [BUILD_DIR / (s.stem + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if not quiet or ptxas_verbose:
        for name, log in logs:
            if log.strip():
                print(f"== {name}\n{log}", file=sys.stderr)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_verbose=a.ptxas_verbose, quiet=False))


if __name__ == "__main__":
    main()
