"""The reference's own device tests, restated in C++ against the B200 build's
public headers (include/lcpp/, same class and method names as the
reference's src/lcpp/device/*.h) — tests/cpp/device_test.cpp."""
import subprocess

import pytest

from tests.cpp.build_cpp_test import build


def test_cpp_dropin_compiles():
    # No GPU needed: the public C++20 surface compiles and links against the C ABI.
    assert build().exists()


@pytest.mark.gpu
def test_cpp_dropin_runs(cuda):
    exe = build()
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert "OK: 0 failure(s)" in r.stdout
