"""The QAT drop-in header (include/cuda/quantize/qat.hpp) on the CPU: its own
checks (tests/cpp/test_qat.cpp) and AMPManager's config file read and written
by the reference's own code (qat.cpp, built into oracle/_ref) when present."""
import ctypes as C
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "cpp", "bin", "test_qat")


@pytest.fixture(scope="module")
def exe():
    if not os.path.exists(EXE):
        pytest.fail("tests/cpp/bin/test_qat is not built: run __graft_entry__.build()")
    return EXE


def test_qat_header_checks(exe):
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "0 failures" in r.stdout, r.stdout + r.stderr


def test_amp_config_file_is_the_reference_format(exe, tmp_path):
    import oracle_lib as O
    ref = O.ref_host()
    if ref is None:
        pytest.skip("reference host build (oracle/_ref) not present")
    ours = str(tmp_path / "ours.bin")
    subprocess.run([exe, "write", ours], check=True, timeout=60)
    prec, scale, zp, tr = C.c_int(), C.c_float(), C.c_float(), C.c_int()
    n = ref.ref_amp_load(ours.encode(), b"gate", C.byref(prec), C.byref(scale), C.byref(zp), C.byref(tr))
    assert (n, prec.value, scale.value, zp.value, tr.value) == (3, 3, 1.5, 0.0, 1)
    n = ref.ref_amp_load(ours.encode(), b"k_proj", C.byref(prec), C.byref(scale), C.byref(zp), C.byref(tr))
    assert (n, prec.value, scale.value) == (3, 4, 1.0)
    theirs = str(tmp_path / "theirs.bin")
    ref.ref_amp_save_two(theirs.encode())
    out = subprocess.run([exe, "read", theirs], capture_output=True, text=True, check=True, timeout=60).stdout.split("\n")
    assert out[0] == "2"
    assert out[1].split() == ["attn.qkv", "3", "0.125", "0", "1"]
    assert out[2].split() == ["mlp.down", "2", "0.03125", "0", "1"]
