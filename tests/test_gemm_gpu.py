"""tcgen05 GEMMs against the CPU oracle.

INT8 (kind::i8): the int32 accumulators must be exact and the scaled
fp32/bf16 outputs bit-identical to the oracle's epilogue (same operation
order, one rounding per step).
FP8 (kind::f8f6f4): products of two FP8 values are exact in fp32, only the
summation order differs from the oracle's sequential FMA; the bar is a max
relative error of 1e-2 per element (with |ref| floored at 1e-2 * rms(ref)),
and in practice the observed error is far smaller (asserted separately for
fp32 outputs at 1e-4)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FP8_TOL = 1e-2
FP8_TOL_F32_OBSERVED = 1e-4


@pytest.fixture(scope="module")
def nq(cuda):
    import nova_b200.capi as capi
    return capi


def fp8_operand(shape, seed, fmt):
    import oracle_lib as O
    x = np.random.default_rng(seed).standard_normal(shape).astype(np.float32)
    qmax = 448.0 if fmt == 0 else 57344.0
    s = float(np.abs(x).max() / qmax)
    return O.quantize_ocp(x, s, fmt), s


def int8_operand(shape, seed):
    return np.random.default_rng(seed).integers(-127, 128, size=shape, dtype=np.int8)


def rel_err(got, ref):
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    floor = 1e-2 * np.sqrt(np.mean(ref * ref)) + 1e-30
    return float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), floor)))


def run_gemm(nq, a, b, m, n, k, fa, fb, b_layout, out_dtype, alpha=1.0, row=None, col=None, bias=None,
             simt=False):
    from gpu_util import dev, empty, host, ptr, stream
    d_a, d_b = dev(a), dev(b)
    esize = {0: 4, 1: 2, 2: 4, 3: 1}[out_dtype]
    d_o = empty(m * n * esize)
    d_r = dev(row) if row is not None else None
    d_c = dev(col) if col is not None else None
    d_bi = dev(bias) if bias is not None else None
    desc = nq.make_desc(m, n, k, fa, fb, b_layout, out_dtype, alpha, ptr(d_r) if d_r is not None else 0,
                        ptr(d_c) if d_c is not None else 0, ptr(d_bi) if d_bi is not None else 0)
    (nq.gemm_simt if simt else nq.gemm)(desc, ptr(d_a), ptr(d_b), ptr(d_o), stream())
    dt = {0: np.float32, 1: np.uint16, 2: np.int32, 3: np.int8}[out_dtype]
    out = host(d_o, dt, (m, n))
    assert nq.device_error_flags() == 0
    return out


SHAPES = [(128, 256, 128), (256, 512, 256), (200, 272, 176), (128, 1024, 1024), (384, 768, 4096), (64, 16, 32)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("b_layout", [0, 1])
def test_int8_gemm_exact(nq, m, n, k, b_layout):
    import oracle_lib as O
    a = int8_operand((m, k), m + k)
    b = int8_operand((k, n) if b_layout == 0 else (n, k), n + k + 1)
    acc = run_gemm(nq, a, b, m, n, k, 2, 2, b_layout, 2)
    np.testing.assert_array_equal(acc, O.gemm_i8_acc(a, b, b_layout == 0))
    rs = (np.random.default_rng(1).random(m) * 0.01 + 1e-3).astype(np.float32)
    cs = (np.random.default_rng(2).random(n) * 0.01 + 1e-3).astype(np.float32)
    bias = np.random.default_rng(3).standard_normal(n).astype(np.float32)
    for out_dtype in (0, 1):
        got = run_gemm(nq, a, b, m, n, k, 2, 2, b_layout, out_dtype, 0.75, rs, cs, bias)
        np.testing.assert_array_equal(got, O.epilogue(acc, out_dtype == 1, 0.75, rs, cs, bias))


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("b_layout", [0, 1])
@pytest.mark.parametrize("fa,fb", [(0, 0), (1, 1), (0, 1)])
def test_fp8_gemm_vs_oracle(nq, m, n, k, b_layout, fa, fb):
    import oracle_lib as O
    a, sa = fp8_operand((m, k), 10 + m, fa)
    b, sb = fp8_operand((k, n) if b_layout == 0 else (n, k), 20 + n, fb)
    ref_acc = O.gemm_fp8_acc(a, b, fa, fb, b_layout == 0)
    alpha = np.float32(sa) * np.float32(sb)
    got32 = run_gemm(nq, a, b, m, n, k, fa, fb, b_layout, 0, float(alpha))
    ref32 = O.epilogue(ref_acc, False, float(alpha))
    assert rel_err(got32, ref32) <= FP8_TOL_F32_OBSERVED
    got16 = run_gemm(nq, a, b, m, n, k, fa, fb, b_layout, 1, float(alpha))
    ref16 = O.epilogue(ref_acc, True, float(alpha))
    assert rel_err(O.bf16_bits_to_f32(got16), O.bf16_bits_to_f32(ref16)) <= FP8_TOL


def test_fp8_gemm_scales_bias_bf16(nq):
    import oracle_lib as O
    m, n, k = 256, 512, 384
    a, _ = fp8_operand((m, k), 1, 0)
    b, _ = fp8_operand((n, k), 2, 0)
    rs = (np.random.default_rng(5).random(m) + 0.5).astype(np.float32)
    cs = (np.random.default_rng(6).random(n) + 0.5).astype(np.float32)
    bias = np.random.default_rng(7).standard_normal(n).astype(np.float32)
    got = run_gemm(nq, a, b, m, n, k, 0, 0, 1, 1, 0.001, rs, cs, bias)
    ref = O.epilogue(O.gemm_fp8_acc(a, b, 0, 0, False), True, 0.001, rs, cs, bias)
    assert rel_err(O.bf16_bits_to_f32(got), O.bf16_bits_to_f32(ref)) <= FP8_TOL


@pytest.mark.parametrize("m,n,k", [(4, 4, 4), (33, 17, 9), (100, 40, 30), (16, 24, 1000)])
def test_simt_path_exact(nq, m, n, k):
    """Shapes the TMA path cannot take run the SIMT kernel: sequential-k FMA,
    bit-identical to the oracle."""
    import oracle_lib as O
    a, _ = fp8_operand((m, k), m, 0)
    b, _ = fp8_operand((k, n), n, 0)
    got = run_gemm(nq, a, b, m, n, k, 0, 0, 0, 0, 1.0)
    np.testing.assert_array_equal(got, O.epilogue(O.gemm_fp8_acc(a, b, 0, 0, True), False, 1.0))
    ai, bi = int8_operand((m, k), 1), int8_operand((k, n), 2)
    np.testing.assert_array_equal(run_gemm(nq, ai, bi, m, n, k, 2, 2, 0, 2), O.gemm_i8_acc(ai, bi, True))


def test_reference_fp8_gemm_cases(nq):
    """fp8_gemm_test.cpp: 4x4 times identity (:58-108), 8x8 identity
    (:110-162), config scaling (:210-275) through FP8GEMM::forward's entry
    point, codes made by the reference codec FP8E4M3(float)."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    eye4 = np.eye(4, dtype=np.float32)
    a = np.arange(1, 17, dtype=np.float32).reshape(4, 4)
    for (x, y, sa, sb, expect) in [(a, eye4, 1.0, 1.0, a), (np.eye(8, dtype=np.float32), np.eye(8, dtype=np.float32),
                                                            1.0, 1.0, np.eye(8, dtype=np.float32)),
                                   (np.tile(np.arange(1, 5, dtype=np.float32), (4, 1)), eye4, 2.0, 0.5,
                                    np.tile(np.arange(1, 5, dtype=np.float32), (4, 1)))]:
        m, k = x.shape
        n = y.shape[1]
        qa, qb = O.quantize_compat(x), O.quantize_compat(y)
        d_a, d_b, d_c = dev(qa), dev(qb), empty(4 * m * n)
        nq.fp8_gemm_forward(ptr(d_a), ptr(d_b), ptr(d_c), m, k, n, sa, sb, 1.0, stream())
        c = host(d_c, np.float32, (m, n))
        np.testing.assert_allclose(c, expect, rtol=0.05, atol=1e-6)
    assert nq.lib.nq_fp8_gemm_workspace_size(128, 256, 128) >= max(128 * 256, 256 * 128, 128 * 128 * 4)


def test_c1_shape_fp8_forward(nq):
    """FP8GEMM::forward M=128, K=1024, N=1024, fp32 out."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    m, k, n = 128, 1024, 1024
    a, sa = fp8_operand((m, k), 1, 0)
    b, sb = fp8_operand((k, n), 0, 0)
    d_a, d_b, d_c = dev(a), dev(b), empty(4 * m * n)
    nq.fp8_gemm_forward(ptr(d_a), ptr(d_b), ptr(d_c), m, k, n, sa, sb, 1.0, stream())
    got = host(d_c, np.float32, (m, n))
    ref = O.epilogue(O.gemm_fp8_acc(a, b, 0, 0, True), False, float(np.float32(sa) * np.float32(sb)))
    assert rel_err(got, ref) <= FP8_TOL_F32_OBSERVED


def test_large_fp8_gemm_torch_check(nq):
    """4096^3 checked against a torch fp64 matmul of
    the decoded operands: too large for the C oracle in a test."""
    import torch
    from gpu_util import ptr, stream
    m = n = k = 4096
    g = torch.Generator(device="cuda").manual_seed(2)
    A = torch.randn(m, k, device="cuda", generator=g)
    B = torch.randn(k, n, device="cuda", generator=g)
    sa, sb = float(A.abs().max() / 448), float(B.abs().max() / 448)
    qa = (A / sa).to(torch.float8_e4m3fn)
    qb = (B / sb).to(torch.float8_e4m3fn)
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    desc = nq.make_desc(m, n, k, 0, 0, 0, 1, float(np.float32(sa) * np.float32(sb)))
    nq.gemm(desc, qa.data_ptr(), qb.data_ptr(), out.data_ptr(), stream())
    ref = (qa.double() @ qb.double()) * (float(np.float32(sa) * np.float32(sb)))
    ref_bf = ref.to(torch.bfloat16).double()
    err = ((out.double() - ref_bf).abs() / torch.maximum(ref_bf.abs(), 1e-2 * ref_bf.pow(2).mean().sqrt())).max()
    assert float(err) <= FP8_TOL
    assert nq.device_error_flags() == 0


@pytest.mark.parametrize("m,n,k", [(2, 2, 3), (128, 256, 512), (200, 272, 176)])
def test_int8_requant_epilogue_matches_quantized_matmul(nq, m, n, k):
    """NQ_S8 epilogue == QuantizedMatmul::forward (quantize_ops.hpp:54-81)."""
    import oracle_lib as O
    a, b = int8_operand((m, k), 5), int8_operand((k, n), 6)
    sa, sb = 0.01, 0.02
    got = run_gemm(nq, a, b, m, n, k, 2, 2, 0, 3, float(np.float32(sa) * np.float32(sb)))
    exp = np.empty((m, n), np.int8)
    O.lib.orc_quantized_matmul(O.ptr(a), O.ptr(b), O.ptr(exp), m, k, n, sa, sb)
    np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("m,k,n", [(37, 300, 70), (1, 64, 1), (9, 1000, 3001), (64, 129, 256)])
def test_mixed_precision_matmul(nq, m, k, n):
    """QuantizedMatmul::mixed_precision (quantize_ops.hpp:83-102): identical
    roundings to the reference host loop (rows and columns that fill no whole
    8 x 128 block, k past one 64-deep stage)."""
    from gpu_util import dev, empty, host, ptr, stream
    rng = np.random.default_rng(9 + m + k + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.integers(-127, 128, (k, n), dtype=np.int8)
    s = (rng.random(k) * 0.1).astype(np.float32)
    d_a, d_b, d_s, d_o = dev(a), dev(b), dev(s), empty(4 * m * n)
    nq.mixed_precision_matmul(ptr(d_a), ptr(d_b), ptr(d_s), ptr(d_o), m, k, n, stream())
    got = host(d_o, np.float32, (m, n))
    exp = np.zeros((m, n), np.float32)
    for p in range(k):
        exp = (exp + a[:, p:p + 1] * (b[p:p + 1, :].astype(np.float32) * s[p])).astype(np.float32)
    np.testing.assert_array_equal(got, exp)


# Shapes of the CTA-pair kernel (74 co-resident pairs on a B200) with and
# without a stream-K part (K >= 48 k-blocks and a last wave at most half
# full): fewer tiles than pairs with every tile cut across 4-5 pairs
# (300 x 2048 x 8192), whole waves plus 1.16 waves shared out (2560 x 4096 x
# 8192), and whole-tile schedules (C4 at M = 256, 4096^3, ragged edges,
# shallow K).
SK_SHAPES = [(2560, 4096, 8192, 0), (300, 2048, 8192, 1), (256, 28672, 8192, 1), (4096, 4096, 4096, 0),
             (1000, 1040, 2048, 0), (2560, 2048, 1024, 1), (4352, 4096, 512, 0), (8192, 14336, 256, 1)]


@pytest.mark.parametrize("m,n,k,b_layout", SK_SHAPES)
def test_stream_k_int8_exact_vs_torch(nq, m, n, k, b_layout):
    """Tiles whose k-blocks are shared out across CTA pairs (stream-K): the
    parked int32 partial sums added by the finishing pair must be exact.
    Checked against torch._int_mm (exact int32 accumulation)."""
    import torch
    from gpu_util import stream
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
    b = torch.randint(-127, 128, (k, n) if b_layout == 0 else (n, k), dtype=torch.int8, device="cuda", generator=g)
    out = torch.empty(m, n, dtype=torch.int32, device="cuda")
    desc = nq.make_desc(m, n, k, 2, 2, b_layout, 2, 1.0)
    nq.gemm(desc, a.data_ptr(), b.data_ptr(), out.data_ptr(), stream())
    ref = torch._int_mm(a, b if b_layout == 0 else b.t().contiguous())
    assert torch.equal(out, ref)
    assert nq.device_error_flags() == 0


@pytest.mark.parametrize("m,n,k,b_layout", [(2560, 2048, 1024, 0), (8192, 14336, 512, 0), (2560, 4096, 8192, 0),
                                            (300, 2048, 8192, 1), (1000, 1040, 2048, 0), (4096, 4096, 4096, 0)])
@pytest.mark.parametrize("out_dtype", [0, 1])
def test_stream_k_fp8_vs_torch(nq, m, n, k, b_layout, out_dtype):
    """FP8 stream-K: the fp32 parts summed in pair order stay within the
    observed fp32 bound of an fp64 product; bf16 outputs within the FP8 bar;
    two launches give bit-identical results (the fixup order is fixed)."""
    import torch
    from gpu_util import stream
    g = torch.Generator(device="cuda").manual_seed(7)
    qa = (torch.randn(m, k, device="cuda", generator=g) * 50).to(torch.float8_e4m3fn)
    qb = (torch.randn(k, n, device="cuda", generator=g) * 50).to(torch.float8_e4m3fn)
    bb = qb if b_layout == 0 else qb.t().contiguous()
    dt = torch.float32 if out_dtype == 0 else torch.bfloat16
    out = torch.empty(m, n, dtype=dt, device="cuda")
    out2 = torch.empty_like(out)
    desc = nq.make_desc(m, n, k, 0, 0, b_layout, out_dtype, 1e-3)
    nq.gemm(desc, qa.data_ptr(), bb.data_ptr(), out.data_ptr(), stream())
    nq.gemm(desc, qa.data_ptr(), bb.data_ptr(), out2.data_ptr(), stream())
    ref = (qa.double() @ qb.double()) * 1e-3
    err = ((out.double() - ref).abs() / torch.maximum(ref.abs(), 1e-2 * ref.pow(2).mean().sqrt())).max()
    # fp32 outputs: the summation-order error of fp32 accumulation grows with
    # k (the observed 1e-4 holds per 4096 terms); bf16 outputs: the FP8 bar
    f32_bound = FP8_TOL_F32_OBSERVED * max(1.0, k / 4096)
    assert float(err) <= (f32_bound if out_dtype == 0 else FP8_TOL)
    assert torch.equal(out.view(torch.int16 if out_dtype else torch.int32),
                       out2.view(torch.int16 if out_dtype else torch.int32))
    assert nq.device_error_flags() == 0


@pytest.mark.parametrize("m", [1, 16, 17, 32, 40, 64, 200, 256])
@pytest.mark.parametrize("b_layout", [1, 0])
def test_decode_int8_exact_vs_oracle(nq, m, b_layout):
    """Decode-shaped INT8 (BASELINE configs[3] pattern at reduced N/K): the
    swap-AB stream-K path with int32 red.add partials must be exact, and the
    scaled bf16 output bit-identical to the oracle epilogue."""
    import oracle_lib as O
    n, k = 4096, 4096
    a = int8_operand((m, k), m)
    b = int8_operand((k, n) if b_layout == 0 else (n, k), 99)
    acc = O.gemm_i8_acc(a, b, b_layout == 0)
    np.testing.assert_array_equal(run_gemm(nq, a, b, m, n, k, 2, 2, b_layout, 2), acc)
    rs = (np.random.default_rng(1).random(m) * 0.01 + 1e-3).astype(np.float32)
    cs = (np.random.default_rng(2).random(n) * 0.01 + 1e-3).astype(np.float32)
    got = run_gemm(nq, a, b, m, n, k, 2, 2, b_layout, 1, 1.0, rs, cs)
    np.testing.assert_array_equal(got, O.epilogue(acc, True, 1.0, rs, cs))


@pytest.mark.parametrize("m,n,k", [(7, 4112, 4112), (40, 4352, 3856), (64, 4240, 4000)])
@pytest.mark.parametrize("b_layout", [1, 0])
def test_decode_ragged_k_and_n(nq, m, n, k, b_layout):
    """The decode path with K not a multiple of the 128-byte k-block (the last
    k-block is zero-filled by the TMA) and N not a multiple of the 128-row weight
    slice: int32 exact, bf16 bit-identical to the oracle epilogue."""
    import oracle_lib as O
    a = int8_operand((m, k), 31)
    b = int8_operand((k, n) if b_layout == 0 else (n, k), 32)
    acc = O.gemm_i8_acc(a, b, b_layout == 0)
    np.testing.assert_array_equal(run_gemm(nq, a, b, m, n, k, 2, 2, b_layout, 2), acc)
    rs = (np.random.default_rng(33).random(m) * 0.01 + 1e-3).astype(np.float32)
    cs = (np.random.default_rng(34).random(n) * 0.01 + 1e-3).astype(np.float32)
    got = run_gemm(nq, a, b, m, n, k, 2, 2, b_layout, 1, 1.0, rs, cs)
    np.testing.assert_array_equal(got, O.epilogue(acc, True, 1.0, rs, cs))


@pytest.mark.parametrize("m", [5, 33, 64])
@pytest.mark.parametrize("n", [4096, 4112])
def test_decode_every_output_type(nq, m, n):
    """The decode path for each output type: int32 exact, fp32 and bf16 (with
    row / column scales and bias) bit-identical to the oracle epilogue, int8
    equal to QuantizedMatmul::forward; n = 4112 leaves a last weight slice of
    16 rows, which the bulk output store clips."""
    import oracle_lib as O
    k = 4096
    a, b = int8_operand((m, k), 21), int8_operand((k, n), 22)
    acc = O.gemm_i8_acc(a, b, True)
    np.testing.assert_array_equal(run_gemm(nq, a, b, m, n, k, 2, 2, 0, 2), acc)
    rng = np.random.default_rng(23)
    rs = (rng.random(m) * 0.01 + 1e-3).astype(np.float32)
    cs = (rng.random(n) * 0.01 + 1e-3).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    for out_dtype, bf in ((0, False), (1, True)):
        got = run_gemm(nq, a, b, m, n, k, 2, 2, 0, out_dtype, 0.5, rs, cs, bias)
        np.testing.assert_array_equal(got, O.epilogue(acc, bf, 0.5, rs, cs, bias))
    sa, sb = 0.01, 0.02
    got = run_gemm(nq, a, b, m, n, k, 2, 2, 0, 3, float(np.float32(sa) * np.float32(sb)))
    exp = np.empty((m, n), np.int8)
    O.lib.orc_quantized_matmul(O.ptr(a), O.ptr(b), O.ptr(exp), m, k, n, sa, sb)
    np.testing.assert_array_equal(got, exp)


@pytest.mark.parametrize("m", [16, 32, 64, 256])
def test_decode_fp8_vs_oracle(nq, m):
    import oracle_lib as O
    n, k = 4096, 4096
    a, sa = fp8_operand((m, k), 3, 0)
    b, sb = fp8_operand((n, k), 4, 0)
    alpha = float(np.float32(sa) * np.float32(sb))
    got = run_gemm(nq, a, b, m, n, k, 0, 0, 1, 0, alpha)
    ref = O.epilogue(O.gemm_fp8_acc(a, b, 0, 0, False), False, alpha)
    assert rel_err(got, ref) <= FP8_TOL_F32_OBSERVED


def test_decode_config3_full_size_vs_torch(nq):
    """BASELINE configs[3] at full size (K=8192, N=28672) for M=16: exact int32
    against torch._int_mm."""
    import torch
    from gpu_util import stream
    m, k, n = 16, 8192, 28672
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
    out = torch.empty(m, n, dtype=torch.int32, device="cuda")
    nq.gemm(nq.make_desc(m, n, k, 2, 2, 1, 2, 1.0), x.data_ptr(), w.data_ptr(), out.data_ptr(), stream())
    xm = torch.zeros(32, k, dtype=torch.int8, device="cuda")
    xm[:m] = x
    ref = torch._int_mm(xm, w.t().contiguous())[:m]
    assert torch.equal(out, ref)
    assert nq.device_error_flags() == 0


def test_decode_flags_across_launches_streams_and_graphs(nq):
    """The decode path's stream-K fixup flags live in a per-stream buffer that
    each launch leaves cleared (no memset per launch), and in a memset node of
    their own inside a graph capture: launches of different shapes back to back
    on one stream, on two streams at once, and a captured graph replayed three
    times must all stay exact against torch._int_mm."""
    import torch
    k, n = 8192, 28672
    g = torch.Generator(device="cuda").manual_seed(5)
    w = torch.randint(-127, 128, (n, k), dtype=torch.int8, device="cuda", generator=g)
    wt = w.t().contiguous()
    cases = {}
    for m in (16, 32, 7):
        x = torch.randint(-127, 128, (m, k), dtype=torch.int8, device="cuda", generator=g)
        xm = torch.zeros(32, k, dtype=torch.int8, device="cuda")
        xm[:m] = x
        cases[m] = (x, torch._int_mm(xm, wt)[:m])
    outs = {m: torch.empty(m, n, dtype=torch.int32, device="cuda") for m in cases}

    def launch(m, stream):
        x, _ = cases[m]
        nq.gemm(nq.make_desc(m, n, k, 2, 2, 1, 2, 1.0), x.data_ptr(), w.data_ptr(), outs[m].data_ptr(),
                stream.cuda_stream)

    def check():
        for m, (_, ref) in cases.items():
            assert torch.equal(outs[m], ref), m
            outs[m].fill_(0)

    s0 = torch.cuda.current_stream()
    for _ in range(3):
        for m in (16, 32, 7, 16):
            launch(m, s0)
    torch.cuda.synchronize()
    check()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    s1.wait_stream(s0)
    s2.wait_stream(s0)
    for _ in range(4):
        launch(16, s1)
        launch(32, s2)
    launch(7, s1)
    torch.cuda.synchronize()
    check()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        cs = torch.cuda.current_stream()
        for m in (16, 32, 7):
            launch(m, cs)
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        check()
    del graph
    launch(16, s0)                      # the stream's own flags are still clear
    torch.cuda.synchronize()
    assert torch.equal(outs[16], cases[16][1])
    assert nq.device_error_flags() == 0


def run_swiglu(nq, a, b, m, n, k, b_layout, out_dtype, alpha, row=None, col=None, bias=None):
    from gpu_util import dev, empty, host, ptr, stream
    d_a, d_b = dev(a), dev(b)
    d_o = empty(m * (n // 2) * (4 if out_dtype == 0 else 2))
    keep = [dev(v) if v is not None else None for v in (row, col, bias)]
    desc = nq.make_desc(m, n, k, 0, 0, b_layout, out_dtype, alpha, *[ptr(t) if t is not None else 0 for t in keep],
                        epilogue=nq.EPI_SWIGLU)
    nq.gemm(desc, ptr(d_a), ptr(d_b), ptr(d_o), stream())
    out = host(d_o, np.float32 if out_dtype == 0 else np.uint16, (m, n // 2))
    assert nq.device_error_flags() == 0
    return out


@pytest.mark.parametrize("m,n,k", [(256, 512, 256), (200, 1024, 512), (64, 256, 128), (384, 2048, 1024), (16, 768, 384)])
@pytest.mark.parametrize("b_layout", [0, 1])
def test_swiglu_epilogue_vs_oracle(nq, m, n, k, b_layout):
    """Gate/up GEMM with the fused silu(g) * u epilogue (the TP MLP's first
    layer): same accumulators as the plain GEMM, then the oracle's SwiGLU on
    the scaled values; fp32 out within 1e-4, bf16 out within the FP8 bar."""
    import oracle_lib as O
    a, sa = fp8_operand((m, k), 30 + m, 0)
    b, sb = fp8_operand((k, n) if b_layout == 0 else (n, k), 40 + n, 0)
    rs = (np.random.default_rng(8).random(m) + 0.5).astype(np.float32) * np.float32(sa)
    cs = (np.random.default_rng(9).random(n) + 0.5).astype(np.float32) * np.float32(sb)
    bias = (np.random.default_rng(10).standard_normal(n) * 0.1).astype(np.float32)
    acc = O.gemm_fp8_acc(a, b, 0, 0, b_layout == 0)
    got32 = run_swiglu(nq, a, b, m, n, k, b_layout, 0, 1.0, rs, cs, bias)
    ref32 = O.swiglu_epilogue(acc, False, 1.0, rs, cs, bias)
    assert rel_err(got32, ref32) <= FP8_TOL_F32_OBSERVED
    got16 = run_swiglu(nq, a, b, m, n, k, b_layout, 1, 1.0, rs, cs)
    ref16 = O.swiglu_epilogue(acc, True, 1.0, rs, cs)
    assert rel_err(O.bf16_bits_to_f32(got16), O.bf16_bits_to_f32(ref16)) <= FP8_TOL


def test_swiglu_epilogue_rejects_unsupported(nq):
    from gpu_util import empty, ptr, stream
    buf = empty(1 << 20)
    for n, fmt, od in [(384, 0, 1), (512, 2, 1), (512, 0, 3)]:
        desc = nq.make_desc(128, n, 128, fmt, fmt, 0, od, 1.0, epilogue=nq.EPI_SWIGLU)
        with pytest.raises(nq.NqError, match="UNSUPPORTED"):
            nq.gemm(desc, ptr(buf), ptr(buf), ptr(buf), stream())


@pytest.mark.parametrize("m,k,n", [(256, 512, 384), (200, 272, 176), (64, 128, 96), (33, 40, 24), (300, 1000, 130)])
@pytest.mark.parametrize("gfmt", [0, 1])
def test_fp8_backward_exact_vs_oracle(nq, m, k, n, gfmt):
    """nq_fp8_gemm_backward: grad_a = g . B^T and grad_b = A^T . g (the
    transposes FP8GEMM::backward omits), E4M3 operands, E4M3 or E5M2 gradient;
    fp32 outputs against the oracle's accumulators on the transposed operands."""
    import oracle_lib as O
    from gpu_util import dev, empty, host, ptr, stream
    a, sa = fp8_operand((m, k), 50 + m, 0)
    b, sb = fp8_operand((k, n), 60 + n, 0)
    g, sg = fp8_operand((m, n), 70 + k, gfmt)
    d_a, d_b, d_g = dev(a), dev(b), dev(g)
    d_ga, d_gb = empty(4 * m * k), empty(4 * k * n)
    nq.fp8_gemm_backward(ptr(d_g), gfmt, ptr(d_a), ptr(d_b), ptr(d_ga), ptr(d_gb), m, k, n, sg, sa, sb, stream())
    ga, gb = host(d_ga, np.float32, (m, k)), host(d_gb, np.float32, (k, n))
    ref_ga = O.epilogue(O.gemm_fp8_acc(g, b, gfmt, 0, False), False, float(np.float32(sg) * np.float32(sb)))
    ref_gb = O.epilogue(O.gemm_fp8_acc(np.ascontiguousarray(a.T), g, 0, gfmt, True), False,
                        float(np.float32(sa) * np.float32(sg)))
    assert rel_err(ga, ref_ga) <= FP8_TOL_F32_OBSERVED
    assert rel_err(gb, ref_gb) <= FP8_TOL_F32_OBSERVED
    # either gradient alone
    d_ga2 = empty(4 * m * k)
    nq.fp8_gemm_backward(ptr(d_g), gfmt, ptr(d_a), ptr(d_b), ptr(d_ga2), 0, m, k, n, sg, sa, sb, stream())
    np.testing.assert_array_equal(host(d_ga2, np.float32, (m, k)), ga)
    assert nq.device_error_flags() == 0
