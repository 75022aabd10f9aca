"""Build and run the C++ mirror test (include/rsort_b200.hpp over the C ABI)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "test_cub_api.cpp")
LIBDIR = os.path.join(ROOT, "rccl_b200", "_lib")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def binary(tmp_path_factory):
    from rccl_b200 import build_ext
    build_ext.build()
    out = str(tmp_path_factory.mktemp("cpp") / "test_cub_api")
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(CUDA, "include"), SRC, "-o", out, "-L", LIBDIR,
                    "-lrsort_b200", f"-Wl,-rpath,{LIBDIR}", "-L", os.path.join(CUDA, "lib64"),
                    "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"], check=True)
    return out


def test_cpp_mirror_host_checks(binary):
    r = subprocess.run([binary], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stderr
    assert "host checks: PASS" in r.stdout


@pytest.mark.gpu
def test_cpp_mirror_gpu_checks(binary):
    r = subprocess.run([binary, "--gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "gpu checks: PASS" in r.stdout
