"""Builds libperegrine_cuda.so in-tree from peregrine_b200/csrc for sm_100a.

Plain nvcc (no torch extension machinery): the library is a torch-free C-ABI shared object
that any host (Zig @cImport, ctypes, C++) can load. Objects go to peregrine_b200/_build/,
the library to peregrine_b200/libperegrine_cuda.so; both are git-ignored but travel with the
repository snapshot to GPU machines.
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
LIB = PKG / "libperegrine_cuda.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"] + ARCH


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _deps() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _compile(nvcc: str, src: Path, verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (src.name + ".o")
    cmd = [nvcc, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [nvcc, "-O3", "-std=c++17", "-Xcompiler", "-fPIC", f"-I{INCLUDE}",
               "-x", "cu", *ARCH, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    newest_dep = max((p.stat().st_mtime for p in _deps()), default=0.0)
    todo = []
    for s in srcs:
        obj = BUILD / (s.name + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, newest_dep):
            todo.append(s)
    logs = {}
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(todo)))) as ex:
        for obj, log in ex.map(lambda s: _compile(nvcc, s, verbose), todo):
            logs[obj.name] = log
    objs = [BUILD / (s.name + ".o") for s in srcs]
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, "-shared", *ARCH, "-o", str(tmp), *map(str, objs), "-lrt", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    if verbose:
        for name, log in logs.items():
            print(f"== {name}\n{log}", file=sys.stderr)
    (BUILD / "ptxas.log").write_text("\n".join(f"== {k}\n{v}" for k, v in logs.items()))
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
