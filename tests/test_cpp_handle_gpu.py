"""The C++ Handle mirror (cublas-rs_b200/cpp/cublas_rs.hpp) running the
reference's example known-answer checks on the GPU
(cublas-rs_b200/examples/sgemm_example.cpp, built by build())."""
import os
import subprocess

import pytest

from conftest import PKG

pytestmark = pytest.mark.gpu


def test_cpp_example_known_answers():
    exe = os.path.join(PKG, "examples", "sgemm_example")
    if not os.path.exists(exe):
        subprocess.run(["make", "-C", PKG, "examples/sgemm_example"], check=True)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all OK" in r.stdout
