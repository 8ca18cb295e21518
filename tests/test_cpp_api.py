"""Builds and runs the C++ drop-in API test (tests/cpp/test_template_api.cpp)
against the in-tree libponni_b200.so."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "test_template_api.cpp")


@pytest.fixture(scope="module")
def binary(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("cpp") / "test_template_api")
    libdir = os.path.join(ROOT, "ponni_b200")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-I", os.path.join(ROOT, "include"), SRC, "-o", out,
                    "-L", libdir, "-lponni_b200", f"-Wl,-rpath,{libdir}"], check=True)
    return out


def test_cpp_host_api(binary, tmp_path):
    r = subprocess.run([binary, "host"], cwd=tmp_path, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr + r.stdout


@pytest.mark.gpu
def test_cpp_gpu_api(binary, tmp_path):
    r = subprocess.run([binary, "gpu"], cwd=tmp_path, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr + r.stdout
