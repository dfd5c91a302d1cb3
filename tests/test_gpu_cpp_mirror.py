"""Builds tests/cpp/mirror_test.cpp against include/levo_ops.hpp and
liblevo_b200.so with nvcc, and runs it on the GPU: the C++ face of the library
keeps the reference's operator names, known answers and exception types."""
from __future__ import annotations

import shutil
import subprocess

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def test_cpp_mirror_program(tmp_path, ops):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    exe = tmp_path / "mirror_test"
    lib_dir = ops.LIB_PATH.parent
    build = subprocess.run(
        [nvcc, "-std=c++17", "-O2", "-I", str(ROOT / "include"), str(ROOT / "tests" / "cpp" / "mirror_test.cpp"),
         "-L", str(lib_dir), "-llevo_b200", f"-Xlinker=-rpath={lib_dir}", "-o", str(exe)],
        capture_output=True, text=True)
    assert build.returncode == 0, build.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "mirror ok" in run.stdout
