"""The C++ host mirror (forge-gpu_b200/host/forge.hpp) through its own test
program tests/cpp/test_host.cpp, written like the reference's Rust tests:
compiled with g++ against include/forge_sph.h and libforge_sph.so."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "forge-gpu_b200")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(tmp_path):
    lib = os.path.join(PKG, "libforge_sph.so")
    assert os.path.exists(lib), "build the library first (make -C forge-gpu_b200)"
    exe = str(tmp_path / "test_host")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(PKG, "host"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "cpp", "test_host.cpp"), "-L", PKG, "-lforge_sph",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{PKG}:{os.path.join(CUDA, 'lib64')}",
           "-o", exe]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def _run(exe, mode):
    r = subprocess.run([exe, mode], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "FAIL" not in r.stdout and "PASS" in r.stdout, r.stdout
    return r.stdout


def test_cpp_host_logic(tmp_path):
    out = _run(_build(tmp_path), "cpu")
    assert out.count("PASS") == 3


@pytest.mark.gpu
def test_cpp_host_reference_tests_on_gpu(cuda, tmp_path):
    out = _run(_build(tmp_path), "gpu")
    assert out.count("PASS") == 8
