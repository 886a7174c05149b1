"""Build the sm_100a shared library `libtensorshrink_b200.so` in-tree.

    python -m tensorshrink_b200.build            # incremental
    python -m tensorshrink_b200.build --force    # rebuild everything

Each `csrc/*.cu` is compiled to an object with nvcc for
`-gencode arch=compute_100a,code=sm_100a` (cross-compiles without a GPU),
then linked into `tensorshrink_b200/_lib/libtensorshrink_b200.so` with the
CUDA runtime linked statically. The library exports only the C ABI declared
in `include/tensorshrink_b200.h`.
"""

from __future__ import annotations

import argparse
import os
import re
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "_lib"
OBJDIR = PKG / "_lib" / "obj"
LIBNAME = "libtensorshrink_b200.so"
TORCH_LIBNAME = "libtensorshrink_torch.so"
TORCH_SRC = PKG / "csrc_torch" / "ops.cpp"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def lib_path() -> Path:
    return LIBDIR / LIBNAME


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return max(f.stat().st_mtime for f in files)


def _included_cu(src: Path) -> list[Path]:
    """`.cu` files that `src` includes by name (a source compiled twice with
    different macros includes the other one)."""
    out = []
    for m in re.finditer(r'^#include "([^"]+\.cu)"', src.read_text(), re.M):
        f = CSRC / m.group(1)
        if f.exists():
            out.append(f)
    return out


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJDIR / (src.stem + ".o")
    newest = max([src.stat().st_mtime, _deps_mtime()] + [f.stat().st_mtime for f in _included_cu(src)])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr.strip():
        print(r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    LIBDIR.mkdir(parents=True, exist_ok=True)
    OBJDIR.mkdir(parents=True, exist_ok=True)
    if force:
        for o in OBJDIR.glob("*.o"):
            o.unlink()
    srcs = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    lib = lib_path()
    if force or not lib.exists() or lib.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(lib), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_torch_ops(lib, verbose)
    return lib


def build_torch_ops(lib: Path, verbose: bool = False) -> Path:
    """`libtensorshrink_torch.so`: the torch.ops.tensorshrink operators, a
    thin C++ layer (host code only) over the C ABI library."""
    import torch.utils.cpp_extension as ce
    out = LIBDIR / TORCH_LIBNAME
    deps = [TORCH_SRC, lib] + list(INCLUDE.glob("*.h"))
    if out.exists() and out.stat().st_mtime >= max(f.stat().st_mtime for f in deps):
        return out
    import torch
    cuda_inc = Path(nvcc()).resolve().parent.parent / "include"
    cmd = ["g++", "-O2", "-shared", "-fPIC", "-std=c++17", str(TORCH_SRC), "-o", str(out),
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in ce.include_paths()], f"-I{cuda_inc}", f"-I{INCLUDE}",
           *[f"-L{p}" for p in ce.library_paths()], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
           "-ltorch_cuda", f"-L{LIBDIR}", "-ltensorshrink_b200", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"torch ops build failed:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
