"""Builds the CPU oracle (test infrastructure only) in-tree:
``oracle/liblcpp_oracle.so`` from ``oracle/lcpp_oracle.c`` and
``tests/golden/_build/refgen`` from ``tests/golden/refgen.cpp``.

The reference itself (LuisaCompute DSL kernels) cannot be compiled here, so
there is no ``oracle/_ref`` build.
"""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
ORACLE_SO = HERE / "liblcpp_oracle.so"
REFGEN_SRC = ROOT / "tests" / "golden" / "refgen.cpp"
REFGEN_BIN = ROOT / "tests" / "golden" / "_build" / "refgen"


def _stale(out: Path, src: Path) -> bool:
    return not out.exists() or src.stat().st_mtime > out.stat().st_mtime


def build_oracle(force: bool = False) -> Path:
    src = HERE / "lcpp_oracle.c"
    if force or _stale(ORACLE_SO, src):
        tmp = ORACLE_SO.with_suffix(".so.tmp")
        subprocess.run(["gcc", "-O3", "-std=c11", "-D_GNU_SOURCE", "-fPIC", "-shared", str(src),
                        "-o", str(tmp), "-lm", "-lpthread"], check=True)
        os.replace(tmp, ORACLE_SO)
    return ORACLE_SO


def build_refgen(force: bool = False) -> Path:
    if force or _stale(REFGEN_BIN, REFGEN_SRC):
        REFGEN_BIN.parent.mkdir(parents=True, exist_ok=True)
        tmp = REFGEN_BIN.with_name("refgen.tmp")
        subprocess.run(["g++", "-O2", "-std=c++17", str(REFGEN_SRC), "-o", str(tmp)], check=True)
        os.replace(tmp, REFGEN_BIN)
    return REFGEN_BIN


def build_all(force: bool = False) -> None:
    build_oracle(force)
    build_refgen(force)


if __name__ == "__main__":
    build_all(force=True)
