"""Calibrator cache files (calibrator.cpp:42-56, 131-152, 192-206, 255-278 of
pplmx/nova): the drop-in header and the reference's own calibrator.cpp (built
into oracle/_ref) read and write the same bytes.  CPU only."""
import ctypes as C
import os
import struct
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "cpp", "bin", "test_calib")
REF = os.path.join(ROOT, "oracle", "_ref", "libnova_ref_calib.so")


def caches():
    """One cache per calibrator kind, laid out as the reference writes them."""
    rng = np.random.default_rng(5)
    hist = rng.integers(0, 1 << 20, 300, dtype=np.uint32)
    chans = rng.random(6).astype(np.float32)
    return {
        0: struct.pack("<ff", -3.25, 7.5),                                        # min, max
        1: struct.pack("<iff", 300, -1.5, 2.25) + hist.tobytes(),                 # bins, min, max, counts
        2: struct.pack("<ff", 0.0078125, 0.0),                                    # scale, zero point
        3: struct.pack("<i", 3) + chans.tobytes(),                                # channels, (scale, zp) pairs
    }


@pytest.mark.parametrize("kind", [0, 1, 2, 3])
def test_cache_round_trip_matches_reference(kind, tmp_path):
    if not os.path.exists(EXE):
        pytest.fail("tests/cpp/bin/test_calib is not built: run __graft_entry__.build()")
    blob = caches()[kind]
    src = tmp_path / "in.bin"
    src.write_bytes(blob)
    ours = tmp_path / "ours.bin"
    subprocess.run([EXE, str(kind), str(src), str(ours)], check=True, timeout=60)
    assert ours.read_bytes() == blob          # ours reads and writes the layout unchanged
    if not os.path.exists(REF):
        pytest.skip("reference calibrator build (oracle/_ref) not present")
    ref = C.CDLL(REF)
    ref.ref_calib_cache_roundtrip.argtypes = [C.c_int, C.c_char_p, C.c_char_p]
    theirs = tmp_path / "theirs.bin"
    assert ref.ref_calib_cache_roundtrip(kind, str(ours).encode(), str(theirs).encode()) == 0
    assert theirs.read_bytes() == blob        # the reference reads our file and writes the same bytes
