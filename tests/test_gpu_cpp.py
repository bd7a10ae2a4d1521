"""Builds and runs the C++ CudaBackend tests (tests/cpp/test_cuda_backend.cpp) against libnibble_cuda.so and the
C oracle. The compile step runs anywhere (CPU test); running needs a GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "test_cuda_backend")


def _build():
    import oracle
    from nibble_b200 import _abi  # noqa: F401  (the library must exist)
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build(with_ref=False)
    cmd = ["g++", "-std=c++20", "-O2", "-Wall", "-Wextra", "-o", BIN,
           os.path.join(ROOT, "tests", "cpp", "test_cuda_backend.cpp"),
           os.path.join(ROOT, "nibble_b200", "csrc", "host", "cuda_backend.cpp"),
           "-L" + os.path.join(ROOT, "nibble_b200"), "-lnibble_cuda",
           "-L" + os.path.join(ROOT, "oracle"), "-loracle",
           "-Wl,-rpath," + os.path.join(ROOT, "nibble_b200") + ":" + os.path.join(ROOT, "oracle"), "-lm"]
    # the library names on disk are lib<name>.so: link against them by path-independent -l
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_cpp_backend_compiles():
    _build()
    assert os.path.exists(BIN)


@pytest.mark.gpu
def test_cpp_backend_runs():
    _build()
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all passed" in r.stdout
