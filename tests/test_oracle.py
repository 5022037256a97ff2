"""The CPU oracle pinned to the reference (CPU only).

Golden vectors in tests/golden/ were produced by the reference's own host
code (tests/golden/make_golden.py); where oracle/_ref is built, the oracle is
also compared live with that code.  Literal expectations are the values the
reference's own tests pin, cited by file:line."""
import os

import numpy as np
import pytest

import oracle_lib as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_compat_codec_matches_reference_golden():
    g = np.load(os.path.join(GOLD, "fp8_codec.npz"))
    np.testing.assert_array_equal(O.quantize_compat(g["x"], 0), g["e4m3"])
    np.testing.assert_array_equal(O.quantize_compat(g["x"], 1), g["e5m2"])
    for fmt, key in ((0, "dec_e4m3"), (1, "dec_e5m2")):
        dec = np.array([(O.lib.orc_e4m3_compat_decode if fmt == 0 else O.lib.orc_e5m2_compat_decode)(c)
                        for c in range(256)], np.float32)
        ref = g[key]
        assert np.array_equal(np.isnan(dec), np.isnan(ref))
        ok = ~np.isnan(ref)
        np.testing.assert_array_equal(dec[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_compat_codec_live_against_reference_build():
    r = O.ref_host()
    if r is None:
        pytest.skip("oracle/_ref not built")
    rng = np.random.default_rng(5)
    # every exponent x a mantissa grid fine enough for every rounding tie
    E = np.arange(256, dtype=np.uint32)
    M = np.arange(0, 1 << 23, 1 << 11, dtype=np.uint32)
    bits = ((E[:, None] << 23) | M[None, :]).ravel()
    bits = np.concatenate([bits, bits | np.uint32(1 << 31), rng.integers(0, 1 << 32, 100000, dtype=np.uint64).astype(np.uint32)])
    x = bits.view(np.float32)
    ref = np.empty(x.size, np.uint8)
    r.ref_e4m3_encode_array(x.ctypes.data, ref.ctypes.data, x.size)
    np.testing.assert_array_equal(O.quantize_compat(x, 0), ref)
    sub = x[::53]
    np.testing.assert_array_equal(O.quantize_compat(sub, 1), np.array([r.ref_e5m2_encode(float(v)) for v in sub], np.uint8))


def test_reference_pinned_special_codes():
    """fp8_types_test.cpp:30-34,59-83,132-154"""
    e = O.lib.orc_e4m3_compat_encode
    assert e(0.0) == 0 and e(float("inf")) == 0x7C and e(float("-inf")) == 0xFC
    assert e(float("nan")) == 0x7D and e(-0.0) == 0x80
    e5 = O.lib.orc_e5m2_compat_encode
    assert e5(0.0) == 0 and e5(float("inf")) == 0x7C and e5(float("-inf")) == 0xFC and e5(float("nan")) == 0x7D
    assert e5(-0.0) == 0x80
    d = O.lib.orc_e4m3_compat_decode
    assert np.isinf(d(0x7C)) and d(0x7C) > 0 and np.isinf(d(0xFC)) and d(0xFC) < 0 and np.isnan(d(0x7D))
    # round trips within 15% for normal values (fp8_types_test.cpp:48-57)
    for v in (0.1, 0.5, 1.0, 2.0, 10.0, 50.0, 100.0, 200.0):
        assert abs(d(e(v)) - v) / v <= 0.15


def test_reference_codec_defects_are_reproduced():
    """The restatement keeps the reference's encoder defects (dropped E4M3
    mantissa carry fp8_types.hpp:94; subnormal bits overflowing into the
    exponent :78-84; overflow to Inf :86-88) -- they are part of parity."""
    e, d = O.lib.orc_e4m3_compat_encode, O.lib.orc_e4m3_compat_decode
    assert d(e(15.9)) == 8.0 and d(e(250.0)) == 128.0 and d(e(7.99)) == 4.0
    assert e(0.0019) == 0x79 and d(0x79) == 288.0
    assert e(241.0) == 0x77 and e(248.0) == 0x70  # 248 rounds up into the dropped carry: 128
    assert e(256.0) == 0x7C and e(1e6) == 0x7C


def test_ocp_codec_against_torch():
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(0)
    for fmt, dt, mx in ((0, torch.float8_e4m3fn, 448.0), (1, torch.float8_e5m2, 57344.0)):
        x = (np.exp2(rng.uniform(-30, np.log2(mx), 200000)) * np.where(rng.random(200000) < 0.5, -1, 1)).astype(np.float32)
        x = np.concatenate([x, np.array([0.0, -0.0, mx, -mx], np.float32)])
        t = torch.from_numpy(x).to(dt).view(torch.uint8).numpy()
        np.testing.assert_array_equal(O.quantize_ocp(x, 1.0, fmt), t)


def test_ocp_codec_saturation_and_nan():
    e4, e5 = O.lib.orc_e4m3_ocp_encode, O.lib.orc_e5m2_ocp_encode
    assert e4(1e9) == 0x7E and e4(-1e9) == 0xFE and e4(float("inf")) == 0x7E and e4(470.0) == 0x7E
    assert e4(float("nan")) == 0x7F and e5(float("nan")) == 0x7F
    assert e5(1e9) == 0x7B and e5(float("-inf")) == 0xFB
    assert e4(2.0 ** -9) == 0x01 and e4(2.0 ** -10) == 0x00 and e4(1.5 * 2.0 ** -9) == 0x02  # ties to even
    assert e4(1.5 * 2.0 ** -10) == 0x01 and e5(2.0 ** -16) == 0x01 and e5(2.0 ** -17) == 0x00


def test_int8_host_reference_semantics():
    """int8_kernels_test.cpp:29-37 restated: rn(x/s) clamped to +-127."""
    x = np.array([0.05, 0.15, -0.05, -0.15, 12.7, 12.75, 1000.0, -1000.0, np.nan], np.float32)
    q = O.quantize_int8(x, 0.1)
    assert list(q) == [0, 2, 0, -2, 127, 127, 127, -127, 0]


def test_from_float_and_quantized_matmul_golden():
    g = np.load(os.path.join(GOLD, "from_float.npz"))
    for i in range(4):
        x = g[f"x{i}"]
        q = np.empty(x.size, np.int8)
        s = np.zeros(1, np.float32)
        assert O.lib.orc_quantized_tensor_from_float(O.ptr(x), x.size, float(g[f"scale_in{i}"]), O.ptr(q), O.ptr(s)) == 1
        np.testing.assert_array_equal(q, g[f"q{i}"])
        assert s[0] == g[f"scale{i}"]
    mm = np.load(os.path.join(GOLD, "quantized_matmul.npz"))
    for i in range(3):
        a, b, s = mm[f"a{i}"], mm[f"b{i}"], mm[f"s{i}"]
        m, k = a.shape
        n = b.shape[1]
        out = np.empty((m, n), np.int8)
        O.lib.orc_quantized_matmul(O.ptr(a), O.ptr(b), O.ptr(out), m, k, n, float(s[0]), float(s[1]))
        np.testing.assert_array_equal(out, mm[f"out{i}"])


def ramp(lo, hi, n):
    """calibrator_test.cpp:22-29"""
    t = (np.arange(n, dtype=np.float32) / np.float32(n)).astype(np.float32)
    return (np.float32(lo) + t * np.float32(hi - lo)).astype(np.float32)


def test_calibrators_reference_expectations():
    """calibrator_test.cpp:32-53 (MinMax 10/127, 20/254), :131-149 (1e-6
    floors), :86-103 (higher percentile -> larger scale)."""
    r = O.minmax_calibrate(ramp(-10, 10, 1024), True)
    assert abs(r[0] - 10 / 127) <= 0.01 and r[1] == 0 and r[2] == 1
    r = O.minmax_calibrate(ramp(-5, 15, 1024), False)
    assert abs(r[0] - 20 / 254) <= 0.01 and r[2] == 0
    assert O.minmax_calibrate(np.full(100, 0.001, np.float32))[0] >= 1e-6
    assert O.minmax_calibrate(np.full(100, 5.0, np.float32))[0] >= 1e-6
    rng = np.random.default_rng(0)
    d = np.where(rng.random(10000) < 0.95, rng.random(10000) * 10, rng.random(10000) * 100).astype(np.float32)
    outs = []
    for p in (99.0, 99.9):
        h = np.empty(256, np.uint32)
        o = np.empty(5, np.float32)
        O.lib.orc_histogram_calibrate(O.ptr(d), d.size, 256, p, 1, O.ptr(h), O.ptr(o))
        outs.append(o[0])
        assert h.sum() == d.size
    assert outs[1] >= outs[0]
    o = np.empty(5, np.float32)
    x = ramp(-5, 5, 1024)
    O.lib.orc_mse_calibrate(O.ptr(x), x.size, 1, O.ptr(o))
    assert o[0] > 0 and o[2] == 1


def test_histogram_counts_and_edges():
    rng = np.random.default_rng(1)
    x = (rng.random(1024) * 100).astype(np.float32)
    for bins in (1, 256, 2048):
        assert O.histogram(x, 0.0, 100.0, bins).sum() == 1024
    h = O.histogram(np.array([np.nan, np.inf, -np.inf, -5.0, 200.0], np.float32), 0.0, 100.0, 10)
    assert list(h) == [3, 0, 0, 0, 0, 0, 0, 0, 0, 2]
    assert O.histogram(x, 1.0, 1.0, 16).sum() == 0  # range <= 1e-6: nothing counted


def test_fp8_gemm_oracle_identity():
    """fp8_gemm_test.cpp:58-162 on the oracle's restatement of the naive kernel"""
    a = np.arange(1, 17, dtype=np.float32).reshape(4, 4)
    c = O.fp8_gemm_reference(O.quantize_compat(a), O.quantize_compat(np.eye(4, dtype=np.float32)), 1, 1, 1)
    np.testing.assert_allclose(c, a, rtol=0.05)


def test_rows_cols_quantize_oracle_consistency():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((9, 40)).astype(np.float32)
    q, s = O.quantize_rows(x, 0)
    for r in range(9):
        amax = np.float32(np.abs(x[r]).max())
        assert s[r] == amax / np.float32(448.0)
        inv = np.float32(448.0) / amax
        np.testing.assert_array_equal(q[r], O.quantize_ocp((x[r] * inv).astype(np.float32), 1.0, 0))
    # a row of tiny values: qmax / amax overflows, the row is divided by its scale
    tiny = np.array([[1e-39, -5e-40, 0.0, 2.5e-40]], np.float32)
    qt, st = O.quantize_rows(tiny, 0)
    with np.errstate(over="ignore"):
        assert np.isinf(np.float32(448.0) / np.float32(1e-39))
    np.testing.assert_array_equal(qt[0], O.quantize_ocp(tiny[0], float(st[0]), 0))
    z, sz = O.quantize_rows(np.zeros((1, 8), np.float32), 0)
    assert sz[0] == 1.0 and not z.any()
    qc, sc = O.quantize_cols(x, 2)
    np.testing.assert_array_equal(qc.T, O.quantize_rows(np.ascontiguousarray(x.T), 2)[0])


def test_fake_quantize_oracle_matches_reference_golden():
    """QAT FakeQuantize::forward (qat.hpp:64-72): the oracle restatement is
    bit-identical to the reference's own host code (golden vectors, and live
    against the reference build when it is present)."""
    g = np.load(os.path.join(GOLD, "qat_fake_quant.npz"))
    r = O.ref_host()
    for i in range(5):
        x, y, (scale, zp) = g[f"x{i}"], g[f"y{i}"], g[f"p{i}"]
        got = O.fake_quantize(x, float(scale), float(zp))
        np.testing.assert_array_equal(got.view(np.uint32), y.view(np.uint32))
        if r is not None:
            live = np.empty_like(x)
            r.ref_fake_quantize(O.ptr(x), O.ptr(live), x.size, float(scale), float(zp))
            np.testing.assert_array_equal(live.view(np.uint32), y.view(np.uint32))
