"""Build ``libgemq_b200.so`` in-tree for sm_100a with nvcc.

The library has no libcuda link dependency (the TMA descriptor encoder is fetched
through ``cudaGetDriverEntryPoint``) and links the CUDA runtime statically, so it
loads on machines without a GPU driver (the CPU tests check its exported symbols).

    python -m robustgemq_b200.build [--force] [--verbose]
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
LIB = PKG / "libgemq_b200.so"
SOURCES = ["gemq_api.cu", "kernels_misc.cu", "kernels_route.cu", "kernels_decode.cu", "kernels_tc.cu",
           "kernels_tcd.cu", "kernels_simt.cu"]
HEADERS = ["gemq_common.cuh", "gemq_internal.h", "tc_work.cuh", "kperm.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES + HEADERS] + [ROOT / "include" / "gemq_b200.h"]
    return any(p.stat().st_mtime > t for p in deps)


def build(force: bool = False, verbose: bool = False, jobs: int = 4) -> Path:
    if not force and not _stale():
        return LIB
    nvcc = nvcc_path()
    objdir = ROOT / "_build"
    objdir.mkdir(exist_ok=True)
    common = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"),
              "--expt-relaxed-constexpr", "-rdc=true"]
    if verbose:
        common += ["-Xptxas", "-v"]
    procs = []
    objs = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = common + ["-c", str(CSRC / src), "-o", str(obj)]
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
        if len(procs) >= jobs:
            _wait(procs.pop(0), verbose)
    for p in procs:
        _wait(p, verbose)
    tmp = LIB.with_suffix(".so.tmp")
    link = [nvcc, *ARCH, "-shared", "-rdc=true", "-cudart", "static", "-o", str(tmp), *map(str, objs)]
    out = subprocess.run(link, capture_output=True, text=True)
    if out.returncode != 0:
        raise RuntimeError(f"link failed:\n{out.stdout}\n{out.stderr}")
    os.replace(tmp, LIB)
    return LIB


def _wait(item, verbose):
    src, proc = item
    out, _ = proc.communicate()
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{out}")
    if verbose and out:
        sys.stdout.write(f"--- {src}\n{out}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
