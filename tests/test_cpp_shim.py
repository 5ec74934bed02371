"""The C++17 host layer (sana.cpp_b200/host: the reference's transformer.h / transformer_ops.h
/ scheduler.h entry points over the C ABI), exercised by tests/cpp/test_shim.cpp compiled and
linked the way a sana.cpp build links it (against lib/libsana_shim.so and lib/libsana_cuda.so).

* without a GPU: the program builds, and calls report the missing device and shape errors as
  the reference's exception types;
* on the GPU: the reference's known-answer tests through the reference API in the fp32 check
  mode, its std::invalid_argument contracts, and bf16-mode consistency of block_forward /
  run_model_blocks and of the device loop against the step-by-step loop.
"""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

PKG = os.path.join(ROOT, "sana.cpp_b200")
LIB = os.path.join(PKG, "lib")


@pytest.fixture(scope="module")
def shim_binary(tmp_path_factory):
    if shutil.which("g++") is None:
        pytest.skip("g++ not available")
    import sys
    sys.path.insert(0, PKG)
    import build as pkg_build  # sana.cpp_b200/build.py
    if not (os.path.exists(pkg_build.SHIM_SO) and os.path.exists(pkg_build.FRONTEND_SO)):
        pkg_build.build_shim()
        pkg_build.build_frontend()
    out = str(tmp_path_factory.mktemp("shim") / "test_shim")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(PKG, "host", "include"), "-I", os.path.join(PKG, "host"),
           "-I", os.path.join(ROOT, "tests", "cpp"), os.path.join(ROOT, "tests", "cpp", "test_shim.cpp"), os.path.join(PKG, "host", "tensor.cpp"),
           "-L", LIB, "-lsana_shim", "-lsana_frontend", "-lsana_cuda", f"-Wl,-rpath,{LIB}", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "warning" not in r.stderr, r.stderr
    return out


def test_shim_builds_and_maps_errors_without_gpu(shim_binary):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([shim_binary, "--no-gpu"], capture_output=True, text=True, timeout=120, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failed" in r.stdout


@pytest.mark.gpu
def test_shim_reference_api_on_gpu(shim_binary):
    r = subprocess.run([shim_binary], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failed" in r.stdout
