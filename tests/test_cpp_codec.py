"""The drop-in FP8E4M3 / FP8E5M2 classes on the host (include/cuda/quantize/
fp8_types.hpp, through tests/cpp/test_codec.cpp) against the reference's own
codes (golden vectors of fp8_types.hpp:64-207).  CPU only."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "cpp", "bin", "test_codec")


def test_host_codec_matches_reference_golden():
    if not os.path.exists(EXE):
        pytest.fail("tests/cpp/bin/test_codec is not built: run __graft_entry__.build()")
    g = np.load(os.path.join(ROOT, "tests", "golden", "fp8_codec.npz"))
    x = np.ascontiguousarray(g["x"], np.float32)
    out = subprocess.run([EXE], input=x.tobytes(), capture_output=True, check=True, timeout=120).stdout
    codes = np.frombuffer(out[: 2 * x.size], np.uint8).reshape(-1, 2)
    np.testing.assert_array_equal(codes[:, 0], g["e4m3"])
    np.testing.assert_array_equal(codes[:, 1], g["e5m2"])
    dec = np.frombuffer(out[2 * x.size:], np.float32)
    np.testing.assert_array_equal(dec[:256].view(np.uint32), g["dec_e4m3"].view(np.uint32))
    np.testing.assert_array_equal(dec[256:].view(np.uint32), g["dec_e5m2"].view(np.uint32))
