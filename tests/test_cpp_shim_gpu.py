"""The C++ cuda_backend shim (include/cuda_backend.hpp) driving the
reference's fused forward loop, compiled with g++ against the C ABI and run
as standalone programs that print PASS / FAIL: the attention ops of the loop
on synthetic per-layer inputs (forward_loop_shim.cpp), and the whole decode
step with host-side weight stubs, each layer's q depending on the previous
layer's attention output (forward_model_shim.cpp)."""
from __future__ import annotations

import os
import subprocess
import tempfile

import pytest

from conftest import PKG_DIR, ROOT

pytestmark = pytest.mark.gpu


def _build(name):
    exe = os.path.join(tempfile.mkdtemp(), name)
    subprocess.run(
        ["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"),
         "-I", os.path.join(ROOT, "oracle"),
         os.path.join(ROOT, "tests", "cpp", name + ".cpp"),
         "-L", PKG_DIR, "-ltg_cuda_backend", "-L", os.path.join(ROOT, "oracle"),
         "-loracle", f"-Wl,-rpath,{PKG_DIR}",
         f"-Wl,-rpath,{os.path.join(ROOT, 'oracle')}", "-o", exe], check=True)
    return exe


@pytest.fixture(scope="module")
def shim_exe(tg, O):
    return _build("forward_loop_shim")


@pytest.fixture(scope="module")
def model_exe(tg, O):
    return _build("forward_model_shim")


@pytest.mark.parametrize("owned", [0, 1])
def test_forward_loop_through_cpp_shim(shim_exe, owned):
    r = subprocess.run([shim_exe, "40", str(owned)], capture_output=True, text=True,
                       timeout=300)
    print(r.stdout, r.stderr)
    assert r.returncode == 0
    assert "PASS" in r.stdout


@pytest.mark.parametrize("owned", [0, 1])
def test_decode_step_with_host_layers_through_cpp_shim(model_exe, owned):
    r = subprocess.run([model_exe, "6", str(owned)], capture_output=True, text=True,
                       timeout=600)
    print(r.stdout, r.stderr)
    assert r.returncode == 0
    assert "PASS" in r.stdout
