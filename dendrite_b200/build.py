"""Builds the in-tree shared library ``dendrite_b200/libdendrite_b200.so``.

Every CUDA source is compiled for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``); nvcc cross-compiles without a GPU. The
planner is plain C++ compiled by nvcc's host compiler into the same library.
Objects go to ``dendrite_b200/_build/``; the library is placed next to this
file so it travels with the package.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libdendrite_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-lineinfo", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build dendrite_b200")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _needs_build(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    jobs = []
    for src in sources():
        obj = BUILD / (src.name + ".o")
        if force or _needs_build(obj, src, headers):
            cmd = [nvcc, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
            if ptxas_verbose and src.suffix == ".cu":
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((src, cmd))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
            futs = {ex.submit(subprocess.run, cmd, capture_output=True, text=True): src
                    for src, cmd in jobs}
            errors = []
            for f in cf.as_completed(futs):
                r = f.result()
                if verbose or ptxas_verbose:
                    sys.stderr.write(r.stderr)
                if r.returncode != 0:
                    errors.append(f"{futs[f].name}:\n{r.stderr}")
            if errors:
                raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    objs = [BUILD / (s.name + ".o") for s in sources()]
    if force or jobs or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl",
               "-lpthread", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv, ptxas_verbose="--ptxas" in sys.argv)
    print(LIB)
