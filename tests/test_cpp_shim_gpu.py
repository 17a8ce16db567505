"""Runs tests/cpp/test_ops_gpu: the reference suite's attention and rope
groups (src/test_ops.cpp:295-546) and its matmul / rmsnorm / vec_add /
ffn_swiglu / argmax groups (test_ops.cpp:42-127, 202-268, 583-596,
638-918) through the C++20 ops_gpu.h layer."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "tests", "cpp", "test_ops_gpu")


@pytest.mark.gpu
def test_reference_style_cpp_suite(cuda):
    if not os.path.exists(BIN):
        subprocess.run(["make", "-C", ROOT, "cpptest"], check=True)
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert " 0 failed" in r.stdout, r.stdout
