"""The reference's own GPU kernels (pplmx/nova src/cuda/quantize/*.cu, built
for sm_100a into oracle/_ref/ by oracle/Makefile) run on the same inputs as
the oracle and as libnova_q: this pins the oracle to the reference itself.
Skipped when oracle/_ref was not built."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env(cuda):
    import oracle_lib as O
    import nova_b200.capi as capi
    r = O.ref_gpu()
    if r is None:
        pytest.skip("oracle/_ref/libnova_ref_gpu.so not built")
    return O, r, capi


def rand(n, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


@pytest.mark.parametrize("sym", [1, 0])
def test_int8_quantize_reference_kernel(env, sym):
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    n = 100003
    x = rand(n, 1, 4.0)
    d_x, d_ref, d_new = dev(x), empty(n), empty(n)
    assert r.ref_gpu_quantize_f32_to_int8(ptr(d_x), ptr(d_ref), n, 0.0371, 0.25, sym) == 0
    nq.quantize_f32_to_int8(ptr(d_x), ptr(d_new), n, 0.0371, 0.25, sym, stream())
    ref = host(d_ref, np.int8)
    np.testing.assert_array_equal(ref, O.quantize_int8(x, 0.0371, 0.25, bool(sym)))
    np.testing.assert_array_equal(host(d_new, np.int8), ref)
    d_y_ref, d_y_new = empty(4 * n), empty(4 * n)
    assert r.ref_gpu_dequantize_int8_to_f32(ptr(d_ref), ptr(d_y_ref), n, 0.0371, 0.25, sym) == 0
    nq.dequantize_int8_to_f32(ptr(d_ref), ptr(d_y_new), n, 0.0371, 0.25, sym, stream())
    np.testing.assert_array_equal(host(d_y_new, np.float32), host(d_y_ref, np.float32))


def test_int8_with_calibration_reference_kernel(env):
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    n = 65537
    x = rand(n, 2, 3.0)
    lo, hi = O.minmax(x)
    d_x, d_ref, d_new = dev(x), empty(n), empty(n)
    assert r.ref_gpu_quantize_with_calibration(ptr(d_x), ptr(d_ref), n, lo, hi) == 0
    nq.quantize_f32_to_int8_with_calibration(ptr(d_x), ptr(d_new), n, lo, hi, stream())
    np.testing.assert_array_equal(host(d_new, np.int8), host(d_ref, np.int8))


@pytest.mark.parametrize("e5m2", [0, 1])
def test_fp8_quantize_reference_kernel(env, e5m2):
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    x = np.concatenate([O.special_floats(), rand(50000, 3, 50.0)]).astype(np.float32)
    n = x.size
    d_x, d_ref, d_new = dev(x), empty(n), empty(n)
    assert r.ref_gpu_quantize_fp8(ptr(d_x), ptr(d_ref), n, e5m2) == 0
    (nq.quantize_f32_to_fp8e5m2 if e5m2 else nq.quantize_f32_to_fp8e4m3)(ptr(d_x), ptr(d_new), n, stream())
    ref = host(d_ref, np.uint8)
    np.testing.assert_array_equal(ref, O.quantize_compat(x, e5m2))
    np.testing.assert_array_equal(host(d_new, np.uint8), ref)


def test_minmax_and_calibrator_reference(env):
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    n = 1 << 20
    x = rand(n, 0, 0.02)   # BASELINE configs[0] weight distribution
    lo, hi = C.c_float(), C.c_float()
    assert r.ref_gpu_compute_minmax(x.ctypes.data, n, C.addressof(lo), C.addressof(hi)) == 0
    assert (lo.value, hi.value) == O.minmax(x)
    l2, h2 = C.c_float(), C.c_float()
    nq.compute_minmax(x.ctypes.data, n, C.addressof(l2), C.addressof(h2), stream())
    assert (l2.value, h2.value) == (lo.value, hi.value)
    for sym in (1, 0):
        out = np.empty(5, np.float32)
        assert r.ref_gpu_minmax_calibrate(x.ctypes.data, n, sym, out.ctypes.data) == 0
        np.testing.assert_array_equal(out, O.minmax_calibrate(x, bool(sym)))


def test_histogram_reference_kernel(env):
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    n = 200000
    x = rand(n, 9, 1.0)
    lo, hi = O.minmax(x)
    d_x, d_ref, d_new = dev(x), empty(4 * 256), empty(4 * 256)
    assert r.ref_gpu_build_histogram(ptr(d_x), ptr(d_ref), n, lo, hi, 256) == 0
    nq.build_histogram(ptr(d_x), ptr(d_new), n, lo, hi, 256, stream())
    ref = host(d_ref, np.uint32)
    np.testing.assert_array_equal(ref, O.histogram(x, lo, hi, 256))
    np.testing.assert_array_equal(host(d_new, np.uint32), ref)


def test_fp8_gemm_reference_kernel(env):
    """FP8GEMM::forward of the reference (naive kernel, fp8_gemm.cu:64-86) is
    bit-identical to the oracle restatement; the tcgen05 GEMM agrees with it
    within the FP8 tolerance on codes both decoders read the same way."""
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    m, k, n = 128, 1024, 1024   # BASELINE configs[0] GEMM
    rng = np.random.default_rng(11)
    xa = rng.standard_normal((m, k)).astype(np.float32)
    xb = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
    sa = float(np.abs(xa).max() / 127.0)
    sb = float(np.abs(xb).max() / 127.0)
    qa = O.quantize_compat(xa / np.float32(sa))
    qb = O.quantize_compat(xb / np.float32(sb))
    # codes whose compat and OCP readings differ (exponent field 0, 0x7C,
    # 0x7D, 0x7F, ...; the compat encoder emits some for tiny inputs) are
    # zeroed so that both GEMMs see the same values
    agree = np.array([O.lib.orc_e4m3_compat_decode(c) == O.lib.orc_e4m3_ocp_decode(c) for c in range(256)])
    qa[~agree[qa]] = 0
    qb[~agree[qb]] = 0
    d_a, d_b, d_ref, d_new = dev(qa), dev(qb), empty(4 * m * n), empty(4 * m * n)
    assert r.ref_gpu_fp8_gemm(ptr(d_a), ptr(d_b), ptr(d_ref), m, k, n, sa, sb, 1.0) == 0
    ref = host(d_ref, np.float32, (m, n))
    np.testing.assert_array_equal(ref, O.fp8_gemm_reference(qa, qb, sa, sb, 1.0))
    nq.fp8_gemm_forward(ptr(d_a), ptr(d_b), ptr(d_new), m, k, n, sa, sb, 1.0, stream())
    got = host(d_new, np.float32, (m, n))
    floor = 1e-2 * np.sqrt(np.mean(ref.astype(np.float64) ** 2))
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), floor)) <= 1e-2
