"""Builds and runs the C++ port of the crate's integration tests
(tests/cpp/correctness_port.cpp) against the C++ API mirror.  The CPU test runs
the cases that need no GPU (shape panics, zero-sized dimensions); the GPU test
runs the whole port."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(ROOT, "flash-attention-cpu_b200", "lib")
ORACLE = os.path.join(ROOT, "oracle", "fa_oracle.c")


@pytest.fixture(scope="module")
def binary(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("cpp") / "correctness_port")
    subprocess.run(["g++", "-std=c++20", "-O2", "-o", out,
                    os.path.join(ROOT, "tests", "cpp", "correctness_port.cpp"), "-x", "c",
                    ORACLE, "-x", "none", f"-L{LIB}", "-lfa_b200", f"-Wl,-rpath,{LIB}",
                    "-lm", "-lpthread"], check=True)
    return out


def test_cpp_port_cpu_cases(binary):
    r = subprocess.run([binary, "cpu"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.mark.gpu
def test_cpp_port_all_cases(binary, gpu_lib):
    r = subprocess.run([binary], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr


@pytest.fixture(scope="module")
def basic_example(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("cpp") / "basic")
    subprocess.run(["g++", "-std=c++20", "-O2", "-o", out,
                    os.path.join(ROOT, "flash-attention-cpu_b200", "cpp", "examples", "basic.cpp"),
                    f"-L{LIB}", "-lfa_b200", f"-Wl,-rpath,{LIB}"], check=True)
    return out


def test_basic_example_builds(basic_example):
    assert os.path.exists(basic_example)


@pytest.mark.gpu
def test_basic_example_runs(basic_example, gpu_lib):
    # the crate's examples/basic.rs flow through the C++ mirror on the GPU
    r = subprocess.run([basic_example], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.strip().endswith("ok")
