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


def _e4m3_disagreeing_codes(O):
    """The 19 E4M3 codes whose reference (compat) and OCP readings differ."""
    out = []
    for c in range(256):
        a, b = O.lib.orc_e4m3_compat_decode(c), O.lib.orc_e4m3_ocp_decode(c)
        if not (a == b or (np.isnan(a) and np.isnan(b))):
            out.append(c)
    return out


def test_fp8_gemm_with_codes_read_differently(env):
    """FP8GEMM::forward on codes the reference encoder emits for tiny inputs:
    exponent field 0 (0x01-0x07, 0x81-0x87), which the reference decoder
    reads as normal numbers ((1 + m/8) * 2^-7) and the tensor cores as OCP
    subnormals (m * 2^-9).  The readings of such a code differ by at most
    0.0127 (code units), so each output of the drop-in GEMM differs from the
    reference kernel's (fp8_gemm.cu:64-86) by at most
        scale_a * scale_b * sum_k (|da_k| |b_k| + |a_k| |db_k| + |da_k| |db_k|)
    (da, db: the per-code reading differences) plus fp32 summation error.
    Asserted element-wise with 5% of all codes planted in that range (where
    the floored max relative error reaches ~2e-2: the codes mean different
    numbers), and the FP8 bar (1e-2) at the frequency the reference encoder
    produces them from N(0,1) data (about 3 in 10^6 codes)."""
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    codes = _e4m3_disagreeing_codes(O)
    assert len(codes) == 19
    tiny = [c for c in codes if (c & 0x78) == 0]
    specials = [c for c in codes if (c & 0x78) != 0]
    comp = np.array([O.lib.orc_e4m3_compat_decode(c) for c in range(256)], np.float64)
    ocp = np.array([O.lib.orc_e4m3_ocp_decode(c) for c in range(256)], np.float64)
    m, k, n = 128, 1024, 1024
    for planted in (0.05, 0.0):
        rng = np.random.default_rng(23)
        xa = rng.standard_normal((m, k)).astype(np.float32)
        xb = (rng.standard_normal((k, n)) * 0.02).astype(np.float32)
        sa = float(np.abs(xa).max() / 127.0)
        sb = float(np.abs(xb).max() / 127.0)
        qa = O.quantize_compat(xa / np.float32(sa))
        qb = O.quantize_compat(xb / np.float32(sb))
        for q in (qa, qb):
            # the reference encoder drops the mantissa carry, so inputs next to
            # +-127 come out as its infinity code 0xFC / 0x7C: those specials are
            # the next test's subject, here they are zeroed
            q[np.isin(q, specials)] = 0
            if planted:
                mask = rng.random(q.shape) < planted
                q[mask] = rng.choice(np.array(tiny, np.uint8), int(mask.sum()))
        if planted:
            assert np.isin(qa, tiny).mean() > 0.04 and np.isin(qb, tiny).mean() > 0.04
        d_a, d_b, d_ref, d_new = dev(qa), dev(qb), empty(4 * m * n), empty(4 * m * n)
        assert r.ref_gpu_fp8_gemm(ptr(d_a), ptr(d_b), ptr(d_ref), m, k, n, sa, sb, 1.0) == 0
        nq.fp8_gemm_forward(ptr(d_a), ptr(d_b), ptr(d_new), m, k, n, sa, sb, 1.0, stream())
        ref = host(d_ref, np.float32, (m, n)).astype(np.float64)
        got = host(d_new, np.float32, (m, n)).astype(np.float64)
        ab, bb = np.abs(comp[qa]), np.abs(comp[qb])
        da, db = np.abs(comp[qa] - ocp[qa]), np.abs(comp[qb] - ocp[qb])
        s2 = np.float64(np.float32(sa) * np.float32(sb))
        bound = s2 * (da @ bb + ab @ db + da @ db) + 1e-5 * s2 * (ab @ bb)
        assert np.all(np.abs(got - ref) <= bound), float(np.max(np.abs(got - ref) - bound))
        assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-3
        if not planted:
            floor = 1e-2 * np.sqrt(np.mean(ref ** 2))
            assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), floor)) <= 1e-2
        # the same codes read the OCP way by the oracle: only the sum order differs
        o = O.gemm_fp8_acc(qa, qb, 0, 0, True).astype(np.float64) * s2
        floor = 1e-2 * np.sqrt(np.mean(o ** 2))
        assert np.max(np.abs(got - o) / np.maximum(np.abs(o), floor)) <= 1e-4


def test_fp8_gemm_with_special_codes(env):
    """The specials of the two readings: the reference decodes 0x7C / 0xFC
    as +-Inf and 0x7D as NaN, where OCP E4M3FN has +-384 and 416; 0x7F / 0xFF
    are +-480 to the reference and NaN in OCP.  Neither encoder produces them
    from finite in-range inputs.  A row of A holding one makes every output
    of that row non-finite in the reference (0x7C, 0x7D, 0xFC) or in the
    drop-in GEMM (0x7F, 0xFF); the other rows keep the FP8 bar."""
    O, r, nq = env
    from gpu_util import dev, empty, host, ptr, stream
    m, k, n = 128, 512, 256
    rng = np.random.default_rng(29)
    qa = O.quantize_compat((rng.standard_normal((m, k)) * 20).astype(np.float32))
    qb = O.quantize_compat((rng.standard_normal((k, n)) * 20).astype(np.float32))
    agree = np.array([c not in _e4m3_disagreeing_codes(O) for c in range(256)])
    qa[~agree[qa]] = 0
    qb[~agree[qb]] = 0
    planted = {3: 0x7C, 7: 0x7D, 11: 0x7F, 13: 0xFC, 17: 0xFF}
    for row, code in planted.items():
        qa[row, 5 + row] = code
    d_a, d_b, d_ref, d_new = dev(qa), dev(qb), empty(4 * m * n), empty(4 * m * n)
    assert r.ref_gpu_fp8_gemm(ptr(d_a), ptr(d_b), ptr(d_ref), m, k, n, 1.0, 1.0, 1.0) == 0
    nq.fp8_gemm_forward(ptr(d_a), ptr(d_b), ptr(d_new), m, k, n, 1.0, 1.0, 1.0, stream())
    ref = host(d_ref, np.float32, (m, n))
    got = host(d_new, np.float32, (m, n))
    for row, code in planted.items():
        if np.isfinite(O.lib.orc_e4m3_compat_decode(code)):
            assert np.isfinite(ref[row]).all() and np.isnan(got[row]).all(), hex(code)
        else:
            assert (~np.isfinite(ref[row])).all() and np.isfinite(got[row]).all(), hex(code)
    clean = np.array([i not in planted for i in range(m)])
    rc, gc = ref[clean].astype(np.float64), got[clean].astype(np.float64)
    floor = 1e-2 * np.sqrt(np.mean(rc ** 2))
    assert np.max(np.abs(gc - rc) / np.maximum(np.abs(rc), floor)) <= 1e-2


def _mse_cases():
    rng = np.random.default_rng(31)
    return [
        ("ramp", np.linspace(-10.0, 10.0, 1000, dtype=np.float32), 1),
        ("normal_50k", rng.standard_normal(50000).astype(np.float32), 1),
        ("normal_3001_asym", (rng.standard_normal(3001) * 0.02 + 0.01).astype(np.float32), 0),
        ("weights_1m", (rng.standard_normal(1 << 20) * 0.02).astype(np.float32), 1),
        ("wide", (rng.standard_normal(20000) * 300.0).astype(np.float32), 1),
        ("constant", np.full(777, 0.5, np.float32), 1),
    ]


@pytest.mark.parametrize("case", range(6))
def test_mse_calibrator_pinned(env, tmp_path, case):
    """MSECalibrator::calibrate (calibrator.cpp:158-190): the drop-in header
    (from host and from device memory), the oracle restatement and the
    reference's own calibrator (on host memory, the only kind its scale
    search can read) give bit-identical scale, zero point, min and max."""
    import ctypes as Cc
    import os
    import subprocess
    O, r, nq = env
    name, x, sym = _mse_cases()[case]
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "tests", "cpp", "bin", "test_mse")
    if not os.path.exists(exe):
        pytest.fail("tests/cpp/bin/test_mse is not built: run __graft_entry__.build()")
    orc = np.zeros(5, np.float32)
    O.lib.orc_mse_calibrate(O.ptr(x), x.size, sym, O.ptr(orc))
    ref = np.zeros(5, np.float32)
    assert r.ref_gpu_mse_calibrate(x.ctypes.data_as(Cc.c_void_p), x.size, sym, ref.ctypes.data_as(Cc.c_void_p)) == 0
    np.testing.assert_array_equal(orc.view(np.uint32), ref.view(np.uint32), err_msg=name)
    path = tmp_path / "x.bin"
    path.write_bytes(x.tobytes())
    for where in ("host", "device"):
        out = subprocess.run([exe, str(path), str(sym), where], capture_output=True, text=True, timeout=120)
        assert out.returncode == 0, out.stderr
        got = np.array([int(v, 16) for v in out.stdout.split()], np.uint32)
        np.testing.assert_array_equal(got, ref.view(np.uint32), err_msg=f"{name} {where}")
