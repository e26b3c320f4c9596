"""Builds tests/cpp/device_test.cpp against the public C++ headers
(include/lcpp/) and liblcpp_b200.so.  Output: tests/cpp/_build/device_test."""
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
OUT = HERE / "_build" / "device_test"


def build() -> Path:
    OUT.parent.mkdir(parents=True, exist_ok=True)
    lib_dir = ROOT / "lc_parallel_primitive_b200"
    cmd = ["g++", "-std=c++20", "-O2", f"-I{ROOT / 'include'}", "-I/usr/local/cuda/include",
           str(HERE / "device_test.cpp"), "-o", str(OUT), f"-L{lib_dir}", "-llcpp_b200",
           f"-Wl,-rpath,{lib_dir}", "-L/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64"]
    subprocess.run(cmd, check=True)
    return OUT
