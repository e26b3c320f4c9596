"""Ahead-of-time build of the native libraries, in-tree.

* ``liblcpp_b200.so``  — every CUDA kernel and the C ABI (include/lcpp_b200.h),
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
* ``libpcg_datagen.so`` — host-side seeded input generator (PCG32).

There is no JIT: the reference compiles its kernels at first use
(src/lcpp/runtime/core.h:36-50); here everything is built before the first call.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"

LIB = PKG / "liblcpp_b200.so"
DATAGEN = PKG / "libpcg_datagen.so"

NVCC_ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.isabs(c) and os.path.exists(c) or not os.path.isabs(c)):
            return c
    return "nvcc"


def _stale(out: Path, deps) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), file=sys.stderr)
    subprocess.run([str(c) for c in cmd], check=True)


UNITS = ["unit_core", "unit_scan", "unit_sort", "unit_by_key"]
OBJDIR = PKG / "_build"


def _unit_deps(unit: str):
    """The unit file, the sources it includes, and every header."""
    src = CSRC / f"{unit}.cu"
    deps = [src] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    for line in src.read_text().splitlines():
        if line.startswith('#include "'):
            deps.append(CSRC / line.split('"')[1])
    return deps


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile the units in parallel (only those whose sources changed), then
    link them into liblcpp_b200.so.  Each unit is whole-program device code
    (no -rdc): the units share no device symbols."""
    from concurrent.futures import ThreadPoolExecutor

    all_deps = sorted({d for u in UNITS for d in _unit_deps(u)})
    if not force and not _stale(LIB, all_deps):
        return LIB  # up to date with every source (the objects may be absent, e.g. on a test box)
    OBJDIR.mkdir(exist_ok=True)
    objs = [OBJDIR / f"{u}.o" for u in UNITS]
    todo = [(u, o) for u, o in zip(UNITS, objs) if force or _stale(o, _unit_deps(u))]

    def compile_unit(uo):
        u, o = uo
        tmp = o.with_suffix(".o.tmp")
        _run([_nvcc(), *NVCC_ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
              f"-I{INCLUDE}", "-c", CSRC / f"{u}.cu", "-o", tmp], verbose)
        os.replace(tmp, o)

    with ThreadPoolExecutor(max_workers=len(UNITS)) as ex:
        list(ex.map(compile_unit, todo))
    if force or todo or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        _run([_nvcc(), *NVCC_ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp, "-ldl"],
             verbose)
        os.replace(tmp, LIB)
    return LIB


def build_datagen(force: bool = False, verbose: bool = False) -> Path:
    src = CSRC / "datagen.c"
    if force or _stale(DATAGEN, [src]):
        tmp = DATAGEN.with_suffix(".so.tmp")
        _run(["gcc", "-O3", "-std=c11", "-D_GNU_SOURCE", "-fPIC", "-shared", src, "-o", tmp,
              "-lm", "-lpthread"], verbose)
        os.replace(tmp, DATAGEN)
    return DATAGEN


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_library(force, verbose)
    build_datagen(force, verbose)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose=True)
