"""The C++ cuda_backend shim (include/cuda_backend.hpp) driving the
reference's fused forward loop, compiled with g++ against the C ABI and run
as a standalone program that prints PASS / FAIL."""
from __future__ import annotations

import os
import subprocess
import tempfile

import pytest

from conftest import PKG_DIR, ROOT

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def shim_exe(tg, O):
    exe = os.path.join(tempfile.mkdtemp(), "forward_loop_shim")
    subprocess.run(
        ["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
         "-I", os.path.join(ROOT, "oracle"),
         os.path.join(ROOT, "tests", "cpp", "forward_loop_shim.cpp"),
         "-L", PKG_DIR, "-ltg_cuda_backend", "-L", os.path.join(ROOT, "oracle"),
         "-loracle", f"-Wl,-rpath,{PKG_DIR}",
         f"-Wl,-rpath,{os.path.join(ROOT, 'oracle')}", "-o", exe], check=True)
    return exe


@pytest.mark.parametrize("owned", [0, 1])
def test_forward_loop_through_cpp_shim(shim_exe, owned):
    r = subprocess.run([shim_exe, "40", str(owned)], capture_output=True, text=True,
                       timeout=300)
    print(r.stdout, r.stderr)
    assert r.returncode == 0
    assert "PASS" in r.stdout
