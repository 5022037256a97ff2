"""FP8 activations on the CPU: the drop-in header's host functions
(include/cuda/quantize/fp8_activation.hpp through tests/cpp/test_act.cpp) and
the oracle agree on every code, for both reference formats."""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "cpp", "bin", "test_act")


def test_activation_header_matches_oracle_on_every_code():
    import oracle_lib as O
    if not os.path.exists(EXE):
        pytest.fail("tests/cpp/bin/test_act is not built: run __graft_entry__.build()")
    out = subprocess.run([EXE], capture_output=True, text=True, check=True, timeout=60).stdout.strip().split("\n")
    assert len(out) == 8
    codes = np.arange(256, dtype=np.uint8)
    for fmt in (0, 1):
        for op in range(4):
            got = np.array(out[fmt * 4 + op].split(), np.uint8)
            np.testing.assert_array_equal(got, O.fp8_activation(codes, fmt, op, 0.01), err_msg=f"fmt {fmt} op {op}")


def test_relu_semantics():
    """relu keeps every non-negative code (NaN and Inf codes included) and maps
    negative ones to the +0 code (fp8_activation.hpp:31-36)."""
    import oracle_lib as O
    codes = np.arange(256, dtype=np.uint8)
    for fmt in (0, 1):
        dec = np.array([(O.lib.orc_e4m3_compat_decode if fmt == 0 else O.lib.orc_e5m2_compat_decode)(int(c))
                        for c in codes], np.float32)
        r = O.fp8_activation(codes, fmt, 0)
        neg = dec < 0
        assert (r[neg] == 0).all() and (r[~neg] == codes[~neg]).all()
