"""Build libflashborn_b200.so in-tree with nvcc for sm_100a (no GPU needed to build).

    python -m quantumdlblocks_b200.build [--debug] [-j N]

Each .cu in csrc/ compiles to an object under _build/ (parallel), then links into
quantumdlblocks_b200/libflashborn_b200.so with the CUDA runtime linked statically, so the
library depends only on the driver (libcuda) at run time.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libflashborn_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _newest_dep() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC)]
    paths.append(os.path.join(ROOT, "include", "flashborn_b200.h"))
    return max(os.path.getmtime(p) for p in paths)


def build(debug: bool = False, jobs: int = 8, force: bool = False, verbose: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= _newest_dep():
        return LIB
    os.makedirs(BUILD, exist_ok=True)
    flags = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
             "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")] + ARCH
    if debug:
        flags.append("-DFB_DEBUG=1")
    if verbose:
        flags.append("-Xptxas=-v")
    nv = nvcc()

    def compile_one(src: str) -> str:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        cmd = [nv, *flags, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
        if verbose and r.stderr:
            sys.stderr.write(r.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB + ".tmp"
    cmd = [nv, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs, "-ldl", "-lpthread", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    ap.add_argument("-j", type=int, default=8)
    a = ap.parse_args()
    print(build(debug=a.debug, jobs=a.j, force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
