"""loom.cpp's C++ selection API (include/loom_select.hpp) compiled against the library.

The program tests/cpp/test_select_api.cpp follows loom.cpp's own test harness style; its argument
errors need no GPU, its known answers do.
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
EXE = os.path.join(ROOT, "_build", "tests", "test_select_api")


@pytest.fixture(scope="module")
def exe():
    os.makedirs(os.path.dirname(EXE), exist_ok=True)
    pkg = os.path.join(ROOT, "loom.cpp_b200")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "cpp", "test_select_api.cpp"), "-o", EXE, "-L", pkg, "-lloom_select",
           f"-Wl,-rpath,{pkg}", "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return EXE


def test_argument_errors_without_gpu(exe):
    r = subprocess.run([exe, "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr


@pytest.mark.gpu
def test_known_answers_on_gpu(exe):
    r = subprocess.run([exe, "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
