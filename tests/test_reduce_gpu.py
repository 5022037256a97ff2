"""Reductions, histograms, calibration and per-row / per-column quantize
against the CPU oracle (int8_kernels.cu:97-169,275-410; calibrator.cpp)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nq(cuda):
    import nova_b200.capi as capi
    return capi


def rand(n, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


@pytest.mark.parametrize("n", [1, 3, 255, 1024, 100003, 1 << 22])
def test_minmax_device_and_host(nq, n):
    import ctypes as C
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = rand(n, n, 10.0)
    if n > 8:
        x[5] = np.nan
    exp = O.minmax(x)
    d_x, d_out = dev(x), empty(8)
    nq.minmax_async(ptr(d_x), n, ptr(d_out), stream())
    got = host(d_out, np.float32)
    assert (got[0], got[1]) == exp
    # reference API: device input, device outputs (int8_kernels_test.cpp:207-236)
    d_lo, d_hi = empty(4), empty(4)
    nq.compute_minmax(ptr(d_x), n, ptr(d_lo), ptr(d_hi), stream())
    assert (host(d_lo, np.float32)[0], host(d_hi, np.float32)[0]) == exp
    # host input, host outputs (MinMaxCalibrator passes host pointers)
    lo, hi = C.c_float(), C.c_float()
    nq.compute_minmax(x.ctypes.data, n, C.addressof(lo), C.addressof(hi), stream())
    assert (lo.value, hi.value) == exp


def test_minmax_empty_and_all_nan(nq):
    import ctypes as C
    from gpu_util import dev, ptr, stream
    lo, hi = C.c_float(5), C.c_float(5)
    nq.compute_minmax(0, 0, C.addressof(lo), C.addressof(hi), stream())
    assert (lo.value, hi.value) == (0.0, 0.0)
    x = np.full(1000, np.nan, np.float32)
    d_x = dev(x)
    nq.compute_minmax(ptr(d_x), 1000, C.addressof(lo), C.addressof(hi), stream())
    assert lo.value == np.finfo(np.float32).max and hi.value == -np.finfo(np.float32).max


def test_minmax_reference_ramp(nq):
    """int8_kernels_test.cpp:207-236: ramp i/n*100-50 -> min -50, max ~49.9"""
    import ctypes as C
    n = 1024
    x = (np.arange(n, dtype=np.float32) / n * 100.0 - 50.0).astype(np.float32)
    lo, hi = C.c_float(), C.c_float()
    nq.compute_minmax(x.ctypes.data, n, C.addressof(lo), C.addressof(hi), 0)
    assert abs(lo.value + 50.0) <= 0.5 and abs(hi.value - 49.9) <= 0.5


@pytest.mark.parametrize("bins", [1, 2, 256, 2048, 20000, 65536])
@pytest.mark.parametrize("n", [1000, 1 << 20])
def test_histogram(nq, bins, n):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = rand(n, bins + n, 1.0)
    x[:4] = [np.nan, np.inf, -np.inf, 100.0]
    lo, hi = -2.5, 3.0
    d_x, d_h = dev(x), empty(4 * bins)
    nq.build_histogram(ptr(d_x), ptr(d_h), n, lo, hi, bins, stream())
    np.testing.assert_array_equal(host(d_h, np.uint32), O.histogram(x, lo, hi, bins))


def test_histogram_host_input_counts_all(nq):
    """int8_kernels_test.cpp:238-268: every element lands in a bin."""
    from gpu_util import empty, host, ptr, stream
    rng = np.random.default_rng(3)
    x = (rng.random(1024, dtype=np.float32) * 100.0).astype(np.float32)
    d_h = empty(4 * 256)
    nq.build_histogram(x.ctypes.data, ptr(d_h), 1024, 0.0, 100.0, 256, stream())
    assert int(host(d_h, np.uint32).sum()) == 1024


@pytest.mark.parametrize("fmt", [0, 1, 2])
@pytest.mark.parametrize("bf16", [False, True])
def test_amax_scale_and_calibrate_quantize(nq, fmt, bf16):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    n = (1 << 20) + 5
    x = rand(n, 77, 0.02)
    x[1000] = -3.5
    if bf16:
        xb = O.f32_to_bf16_bits(x)
        x = O.bf16_bits_to_f32(xb)
        d_x = dev(xb)
    else:
        d_x = dev(x)
    d_as, d_q = empty(8), empty(n)
    nq.calibrate_quantize(ptr(d_x), 1 if bf16 else 0, ptr(d_q), n, fmt, ptr(d_as), stream())
    amax_scale = host(d_as, np.float32)
    amax = O.lib.orc_amax(O.ptr(x), n)
    qmax = [448.0, 57344.0, 127.0][fmt]
    assert amax_scale[0] == amax
    assert amax_scale[1] == np.float32(amax) / np.float32(qmax)
    np.testing.assert_array_equal(host(d_q, np.uint8), O.quantize_ocp(x, float(amax_scale[1]), fmt))


@pytest.mark.parametrize("fmt", [0, 2])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("shape", [(7, 33), (64, 4096), (3, 16), (300, 8192), (50, 28672), (20, 28672),
                                   (1000, 2048), (5, 1024)])
def test_quantize_rows(nq, fmt, bf16, shape):
    """All row-width regimes: unaligned/odd widths (two-pass kernel), rows
    under 4 KB (register-resident), 4 KB .. 100 KB (bulk-staged ring; 28672
    bf16 = 56 KB takes 3 stages) and fp32 rows over 100 KB (two-pass).  Row 1
    holds tiny values whose qmax / amax overflows (the division path)."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    r, c = shape
    x = rand(r * c, r * 31 + c, 1.0).reshape(r, c)
    x[0, : min(c, 5)] *= 20.0
    if r > 1:
        x[1] *= np.float32(1e-39)
    if r > 2:
        x[2] = 0.0
    if bf16:
        x = O.f32_to_bf16_bits(x)
    d_x, d_q, d_s = dev(x), empty(r * c), empty(4 * r)
    nq.quantize_rows(ptr(d_x), 1 if bf16 else 0, ptr(d_q), ptr(d_s), r, c, fmt, stream())
    q_exp, s_exp = O.quantize_rows(x, fmt, bf16)
    np.testing.assert_array_equal(host(d_s, np.float32), s_exp)
    np.testing.assert_array_equal(host(d_q, np.uint8, (r, c)), q_exp)


@pytest.mark.parametrize("fmt", [0, 2])
@pytest.mark.parametrize("shape", [(5, 13), (1024, 3000), (4096, 64)])
def test_quantize_cols(nq, fmt, shape):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    r, c = shape
    x = rand(r * c, r + c, 0.02).reshape(r, c)
    d_x, d_q, d_s = dev(x), empty(r * c), empty(4 * c)
    nq.quantize_cols(ptr(d_x), ptr(d_q), ptr(d_s), r, c, fmt, stream())
    q_exp, s_exp = O.quantize_cols(x, fmt)
    np.testing.assert_array_equal(host(d_s, np.float32), s_exp)
    np.testing.assert_array_equal(host(d_q, np.uint8, (r, c)), q_exp)


def test_minmax_rows(nq):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    r, c = 37, 1001
    x = rand(r * c, 4, 3.0).reshape(r, c)
    d_x, d_lo, d_hi = dev(x), empty(4 * r), empty(4 * r)
    nq.minmax_rows(ptr(d_x), r, c, ptr(d_lo), ptr(d_hi), stream())
    lo, hi = host(d_lo, np.float32), host(d_hi, np.float32)
    for i in range(r):
        assert (lo[i], hi[i]) == O.minmax(x[i])
