"""Runs the C++ drop-in API test (tests/cpp/test_api.cpp, built by
__graft_entry__.build()) on the GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "cpp", "bin", "test_api")


@pytest.mark.gpu
def test_cpp_api(cuda):
    if not os.path.exists(EXE):
        pytest.fail("tests/cpp/bin/test_api is not built: run __graft_entry__.build()")
    r = subprocess.run([EXE], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout
