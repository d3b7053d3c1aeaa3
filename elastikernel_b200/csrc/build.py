"""Build recipe for the in-tree C-ABI library ``elastikernel_b200/_ek.so``.

Every ``.cu`` / ``.cpp`` file in this directory is compiled by nvcc for
sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) and linked into one
shared object with the CUDA runtime linked statically, so the library loads
without a CUDA toolkit or driver on the library path (the driver is resolved at
run time through ``cudaGetDriverEntryPointByVersion``).

Usage: ``python -m elastikernel_b200.csrc.build [--force] [-v]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
REPO = PKG.parent
LIB = PKG / "_ek.so"
OBJ_DIR = REPO / "_build" / "obj"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(INCLUDE), "-I", str(HERE)]
CU_FLAGS = ARCH + ["--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the elastikernel_b200 CUDA library cannot be built")


def sources() -> list[Path]:
    return sorted(p for p in HERE.iterdir() if p.suffix in (".cu", ".cpp"))


def headers() -> list[Path]:
    return sorted(p for p in HERE.iterdir() if p.suffix in (".cuh", ".h")) + [INCLUDE / "elastikernel.h"]


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJ_DIR / (src.name + ".o")
    cmd = [nvcc()] + COMMON + (CU_FLAGS if src.suffix == ".cu" else ARCH) + ["-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd[1:1] = ["-x", "cu"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout, res.stderr, flush=True)
    return obj


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in sources() + headers() + [Path(__file__)])


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link ``_ek.so`` if any source is newer than it."""
    if not force and not needs_build():
        return LIB
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", str(tmp)] + [str(o) for o in objs]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
