"""Element-wise quantize / dequantize kernels against the CPU oracle.

Bit-exact for every code (the oracle restates int8_kernels.cu:15-60,
fp8_kernels.cu:12-122, fp8_types.hpp:64-207 and the OCP spec).  Sizes cover
the vector body, the scalar tail and unaligned pointers."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SIZES = [1, 15, 16, 17, 1000, 4096 + 7, 1 << 20]


@pytest.fixture(scope="module")
def nq(cuda):
    import nova_b200.capi as capi
    return capi


def rand(n, seed, scale=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * scale).astype(np.float32)


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("off", [0, 4])
def test_compat_fp8_quantize_bit_exact(nq, n, fmt, off):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = rand(n, 1 + n, 100.0)
    x[: min(n, 8)] = [0.0, -0.0, np.inf, -np.inf, np.nan, 250.0, 0.0019, 15.9][: min(n, 8)]
    d_x, d_q = dev(x, off), empty(n, off // 4)
    fn = nq.quantize_f32_to_fp8e4m3 if fmt == 0 else nq.quantize_f32_to_fp8e5m2
    fn(ptr(d_x), ptr(d_q), n, stream())
    np.testing.assert_array_equal(host(d_q, np.uint8), O.quantize_compat(x, fmt))


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("off", [0, 4])
def test_compat_fp8_quantize_table_path_every_pattern(nq, fmt, off):
    """From 4 Mi elements on the reference-codec encode reads a table indexed by
    the float's clamped exponent and top 7 mantissa bits (plus the sign and a
    NaN test).  Every 16-bit top
    pattern -- each sign, exponent and top-7 mantissa bits -- with low mantissa
    bits 0, 1, 0x8000 and 0xFFFF (every NaN form included), repeated past 4 Mi
    with a ragged tail, must match the oracle bit for bit."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    top = np.arange(1 << 16, dtype=np.uint32) << 16
    low = np.array([0, 1, 0x8000, 0xFFFF], dtype=np.uint32)
    u = (top[:, None] | low[None, :]).reshape(-1)
    n = (1 << 22) + 3
    x = np.tile(u, n // u.size + 1)[:n].view(np.float32)
    d_x, d_q = dev(x, off), empty(n, off // 4)
    fn = nq.quantize_f32_to_fp8e4m3 if fmt == 0 else nq.quantize_f32_to_fp8e5m2
    fn(ptr(d_x), ptr(d_q), n, stream())
    np.testing.assert_array_equal(host(d_q, np.uint8), O.quantize_compat(x, fmt))


@pytest.mark.parametrize("fmt", [0, 1])
def test_compat_fp8_special_values(nq, fmt):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = O.special_floats()
    d_x, d_q = dev(x), empty(x.size)
    fn = nq.quantize_f32_to_fp8e4m3 if fmt == 0 else nq.quantize_f32_to_fp8e5m2
    fn(ptr(d_x), ptr(d_q), x.size, stream())
    q = host(d_q, np.uint8)
    np.testing.assert_array_equal(q, O.quantize_compat(x, fmt))
    # codes pinned by the reference tests (fp8_types_test.cpp:59-83,
    # fp8_kernels_test.cpp:266-363): +Inf 0x7C, -Inf 0xFC, NaN 0x7D, -0 0x80
    assert q[2] == 0x7C and q[3] == 0xFC and q[4] == 0x7D and q[1] == 0x80 and q[0] == 0x00


@pytest.mark.parametrize("fmt", [0, 1])
def test_compat_fp8_dequantize_all_codes(nq, fmt):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    codes = np.tile(np.arange(256, dtype=np.uint8), 65)  # 16640, not a multiple of 16 * 256
    d_q, d_y = dev(codes), empty(codes.size * 4)
    fn = nq.dequantize_fp8e4m3_to_f32 if fmt == 0 else nq.dequantize_fp8e5m2_to_f32
    fn(ptr(d_q), ptr(d_y), codes.size, 0.37, stream())
    got = host(d_y, np.float32)
    exp = O.dequantize_compat(codes, 0.37, fmt)
    np.testing.assert_array_equal(got.view(np.uint32)[~np.isnan(exp)], exp.view(np.uint32)[~np.isnan(exp)])
    assert np.isnan(got[np.isnan(exp)]).all()


def test_batched_fp8(nq):
    import torch
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    sizes = [1, 33, 4096, 100003]
    xs = [rand(n, 50 + n, 3.0) for n in sizes]
    scales = np.array([0.5, 2.0, 10.0, 0.01], np.float32)
    d_x = [dev(x) for x in xs]
    d_q = [empty(n) for n in sizes]
    src_arr = dev(np.array([ptr(t) for t in d_x], np.uint64))
    dst_arr = dev(np.array([ptr(t) for t in d_q], np.uint64))
    d_sizes = dev(np.array(sizes, np.uint64))
    d_scales = dev(scales)
    nq.quantize_batched_f32_to_fp8e4m3(ptr(src_arr), ptr(dst_arr), len(sizes), ptr(d_sizes), ptr(d_scales), stream())
    for x, q, s in zip(xs, d_q, scales):
        exp = np.empty(x.size, np.uint8)
        O.lib.orc_quantize_scaled_fp8_compat(O.ptr(x), O.ptr(exp), x.size, float(s))
        np.testing.assert_array_equal(host(q, np.uint8), exp)
    d_y = [empty(n * 4) for n in sizes]
    y_arr = dev(np.array([ptr(t) for t in d_y], np.uint64))
    nq.dequantize_batched_fp8e4m3_to_f32(ptr(dst_arr), ptr(y_arr), len(sizes), ptr(d_sizes), ptr(d_scales), stream())
    for q, y, s in zip(d_q, d_y, scales):
        exp = O.dequantize_compat(host(q, np.uint8), float(s), 0)
        np.testing.assert_array_equal(host(y, np.float32), exp)
    torch.cuda.synchronize()


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("sym", [True, False])
def test_int8_quantize_bit_exact(nq, n, sym):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = rand(n, 7 + n, 5.0)
    scale, zp = 0.0371, 0.25
    d_x, d_q = dev(x), empty(n)
    nq.quantize_f32_to_int8(ptr(d_x), ptr(d_q), n, scale, zp, int(sym), stream())
    np.testing.assert_array_equal(host(d_q, np.int8), O.quantize_int8(x, scale, zp, sym))
    d_y = empty(4 * n)
    nq.dequantize_int8_to_f32(ptr(d_q), ptr(d_y), n, scale, zp, int(sym), stream())
    np.testing.assert_array_equal(host(d_y, np.float32), O.dequantize_int8(host(d_q, np.int8), scale, zp, sym))


def test_int8_reference_test_cases(nq):
    """int8_kernels_test.cpp: exact vs host rounding (:47-77), zeros
    (:152-175), clamping (:177-205), round trip <= 20% (:111-150)."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    rng = np.random.default_rng(1234)
    x = ((rng.random(1024, dtype=np.float32) - 0.5) * 20.0).astype(np.float32)
    d_x, d_q = dev(x), empty(1024)
    nq.quantize_f32_to_int8(ptr(d_x), ptr(d_q), 1024, 0.1, 0.0, 1, stream())
    q = host(d_q, np.int8)
    np.testing.assert_array_equal(q, O.quantize_int8(x, 0.1))
    z = np.zeros(100, np.float32)
    d_z, d_zq = dev(z), empty(100)
    nq.quantize_f32_to_int8(ptr(d_z), ptr(d_zq), 100, 0.1, 0.0, 1, stream())
    assert (host(d_zq, np.int8) == 0).all()
    c = np.where(np.arange(100) % 2 == 0, 1000.0, -1000.0).astype(np.float32)
    d_c, d_cq = dev(c), empty(100)
    nq.quantize_f32_to_int8(ptr(d_c), ptr(d_cq), 100, 0.1, 0.0, 1, stream())
    cq = host(d_cq, np.int8)
    assert cq.min() == -127 and cq.max() == 127
    x2 = ((rng.random(1024, dtype=np.float32) - 0.5) * 10.0).astype(np.float32)
    d_x2, d_q2, d_y2 = dev(x2), empty(1024), empty(4096)
    nq.quantize_f32_to_int8(ptr(d_x2), ptr(d_q2), 1024, 0.05, 0.0, 1, stream())
    nq.dequantize_int8_to_f32(ptr(d_q2), ptr(d_y2), 1024, 0.05, 0.0, 1, stream())
    y2 = host(d_y2, np.float32)
    keep = np.abs(x2) >= 0.1
    assert (np.abs(x2[keep] - y2[keep]) / np.abs(x2[keep])).max() <= 0.2


@pytest.mark.parametrize("n", [17, 1 << 16])
def test_int8_with_calibration_and_round_away(nq, n):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = rand(n, 99, 2.0)
    lo, hi = O.minmax(x)
    d_x, d_q = dev(x), empty(n)
    nq.quantize_f32_to_int8_with_calibration(ptr(d_x), ptr(d_q), n, lo, hi, stream())
    exp = np.empty(n, np.int8)
    O.lib.orc_quantize_int8_with_calibration(O.ptr(x), O.ptr(exp), n, lo, hi)
    np.testing.assert_array_equal(host(d_q, np.int8), exp)
    # ties: x/scale exactly k + 0.5 rounds away from zero (std::round)
    s = 0.5
    t = (np.arange(n, dtype=np.float32) % 300 - 150) * 0.25
    d_t, d_tq = dev(t), empty(n)
    nq.quantize_f32_to_int8_round_away(ptr(d_t), ptr(d_tq), n, s, stream())
    exp2 = np.empty(n, np.int8)
    O.lib.orc_quantize_int8_half_away(O.ptr(t), O.ptr(exp2), n, s)
    np.testing.assert_array_equal(host(d_tq, np.int8), exp2)


@pytest.mark.parametrize("fmt", [0, 1, 2])
@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("n", [31, 1 << 20])
def test_scaled_quantize_bit_exact(nq, fmt, bf16, n):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = rand(n, 5 + fmt, 30.0)
    x[:6] = [0.0, -0.0, np.inf, -np.inf, 1e30, -1e30]
    if bf16:
        xb = O.f32_to_bf16_bits(x)
        x_eff = O.bf16_bits_to_f32(xb)
        d_x = dev(xb)
    else:
        x_eff = x
        d_x = dev(x)
    scale = np.array([0.0917], np.float32)
    d_s, d_q = dev(scale), empty(n)
    nq.quantize_scaled(ptr(d_x), 1 if bf16 else 0, ptr(d_q), n, fmt, ptr(d_s), stream())
    np.testing.assert_array_equal(host(d_q, np.uint8), O.quantize_ocp(x_eff, float(scale[0]), fmt))
    d_y = empty(4 * n)
    nq.dequantize_scaled(ptr(d_q), ptr(d_y), n, fmt, ptr(d_s), stream())
    np.testing.assert_array_equal(host(d_y, np.float32), O.dequantize_ocp(host(d_q, np.uint8), float(scale[0]), fmt))


def test_ocp_nan_and_specials(nq):
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = O.special_floats()
    d_x, d_s = dev(x), dev(np.array([1.0], np.float32))
    for fmt in (0, 1, 2):
        d_q = empty(x.size)
        nq.quantize_scaled(ptr(d_x), 0, ptr(d_q), x.size, fmt, ptr(d_s), stream())
        np.testing.assert_array_equal(host(d_q, np.uint8), O.quantize_ocp(x, 1.0, fmt), err_msg=f"fmt {fmt}")


def test_invalid_arguments(nq):
    from nova_b200.capi import NqError
    with pytest.raises(NqError):
        nq.quantize_f32_to_int8(0, 0, 10, 1.0, 0.0, 1, 0)
    nq.quantize_f32_to_int8(0, 0, 0, 1.0, 0.0, 1, 0)  # n == 0 is a no-op


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("off", [0, 4])
def test_fake_quantize_bit_exact(nq, n, off):
    """QAT FakeQuantize::forward over a device array (nq_fake_quantize_int8):
    bit-identical to the oracle (itself pinned to the reference's host code),
    on the vector body, the tail and unaligned pointers."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    x = rand(n, 7 + n, 5.0)
    x[: min(n, 3)] = [0.025, -0.075, np.nan][: min(n, 3)]
    for scale, zp in [(0.05, 0.0), (0.5, 2.0), (0.0, 0.5)]:
        d_x, d_y = dev(x, off), empty(4 * n, off)
        nq.fake_quantize_int8(ptr(d_x), ptr(d_y), n, scale, zp, stream())
        got = host(d_y, np.float32)
        np.testing.assert_array_equal(got.view(np.uint32), O.fake_quantize(x, scale, zp).view(np.uint32))


def test_fake_quantize_reference_golden(nq):
    import os
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "qat_fake_quant.npz"))
    for i in range(5):
        x, y, (scale, zp) = g[f"x{i}"], g[f"y{i}"], g[f"p{i}"]
        d_x, d_y = dev(x), empty(4 * x.size)
        nq.fake_quantize_int8(ptr(d_x), ptr(d_y), x.size, float(scale), float(zp), stream())
        np.testing.assert_array_equal(host(d_y, np.float32).view(np.uint32), y.view(np.uint32))


@pytest.mark.parametrize("fmt", [0, 1])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_fp8_activation_vs_oracle(nq, fmt, op):
    """FP8 activations on reference-codec codes (nq_fp8_activation,
    fp8_activation.hpp:26-98): every code, plus a long random array through
    the 16-code vector path, its tail and an unaligned pointer.  relu and leaky
    relu are bit-exact; gelu and sigmoid use CUDA's erff / expf against the
    host libm of the oracle, so a code may differ by one step where the fp32
    result sits within a few ulp of a rounding boundary (at most 1 in 256)."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    rng = np.random.default_rng(11 + op)
    for codes, off in [(np.arange(256, dtype=np.uint8), 0),
                       (rng.integers(0, 256, (1 << 20) + 7, dtype=np.uint8), 0),
                       (rng.integers(0, 256, 1000, dtype=np.uint8), 3)]:
        d_x, d_y = dev(codes, off), empty(codes.size, off)
        nq.fp8_activation(ptr(d_x), ptr(d_y), codes.size, fmt, op, 0.01, stream())
        got = host(d_y, np.uint8)
        ref = O.fp8_activation(codes, fmt, op, 0.01)
        diff = got != ref
        if op in (0, 3):
            assert not diff.any()
        else:
            assert diff.mean() <= 1 / 256
            assert (np.abs(got[diff].astype(int) - ref[diff].astype(int)) <= 1).all()
    assert nq.device_error_flags() == 0
