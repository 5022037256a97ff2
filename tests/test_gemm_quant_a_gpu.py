"""nq_gemm_quant_a: the W8A8 GEMM with the per-token activation quantization
fused into the kernel (one launch), against the two-launch path it replaces
(nq_quantize_rows, then nq_gemm with the per-token scales as row scales).

Bars: the codes and scales the kernel writes are bit-identical to
nq_quantize_rows' (which the quantize tests pin to the oracle); the GEMM
output is bit-identical to the two-launch path (the same codes, scales and
accumulation); at the full BASELINE configs[2] shape (8192 x 4096 x 14336,
41 outlier channels x20, per-channel E4M3 weights) the output is also checked
against an fp64 product of the decoded codes (max relative error 1e-2, |ref|
floored at 1e-2 rms, the FP8 bar)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nq(cuda):
    import nova_b200.capi as capi
    return capi


def _case(m, k, n, b_layout, seed, outliers=0):
    import torch
    import nova_b200.capi as nq
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=g)
    if outliers:
        ch = torch.randperm(k, generator=torch.Generator().manual_seed(seed + 1))[:outliers].cuda()
        x[:, ch] *= 20.0
    x = x.to(torch.bfloat16)
    w = torch.randn(k, n, device="cuda", generator=g).mul_(0.02)
    wq = torch.empty(k, n, dtype=torch.uint8, device="cuda")
    ws = torch.empty(n, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    nq.quantize_cols(w.data_ptr(), wq.data_ptr(), ws.data_ptr(), k, n, nq.E4M3, s)
    if b_layout == 1:
        wq = wq.t().contiguous()
    return x, wq, ws


def _two_launch(nq, x, wq, ws, m, k, n, b_layout, out_dtype, epilogue=0):
    import torch
    s = torch.cuda.current_stream().cuda_stream
    xq = torch.empty(m, k, dtype=torch.uint8, device="cuda")
    xs = torch.empty(m, device="cuda")
    nq.quantize_rows(x.data_ptr(), nq.BF16, xq.data_ptr(), xs.data_ptr(), m, k, nq.E4M3, s)
    n_out = n // 2 if epilogue else n
    y = torch.empty(m, n_out, dtype=torch.bfloat16 if out_dtype == nq.BF16 else torch.float32, device="cuda")
    d = nq.make_desc(m, n, k, nq.E4M3, nq.E4M3, b_layout, out_dtype, 1.0, xs.data_ptr(), ws.data_ptr(), 0, epilogue)
    nq.gemm(d, xq.data_ptr(), wq.data_ptr(), y.data_ptr(), s)
    return xq, xs, y


def _fused(nq, x, wq, ws, m, k, n, b_layout, out_dtype, epilogue=0):
    import torch
    s = torch.cuda.current_stream().cuda_stream
    xq = torch.full((m, k), 0xAB, dtype=torch.uint8, device="cuda")     # stale contents must not leak
    xs = torch.full((m,), -3.0, device="cuda")
    n_out = n // 2 if epilogue else n
    y = torch.empty(m, n_out, dtype=torch.bfloat16 if out_dtype == nq.BF16 else torch.float32, device="cuda")
    d = nq.make_desc(m, n, k, nq.E4M3, nq.E4M3, b_layout, out_dtype, 1.0, 0, ws.data_ptr(), 0, epilogue)
    nq.gemm_quant_a(d, x.data_ptr(), xq.data_ptr(), xs.data_ptr(), wq.data_ptr(), y.data_ptr(), s)
    return xq, xs, y


@pytest.mark.parametrize("m,k,n,b_layout,out_dtype", [
    (300, 256, 512, 0, 1), (1000, 512, 768, 1, 1), (130, 4096, 256, 0, 0), (1000, 8192, 512, 0, 1),
    (2048, 1024, 2048, 1, 0), (257, 4112, 272, 0, 1)])
def test_fused_quantize_equals_two_launches(nq, m, k, n, b_layout, out_dtype):
    import torch
    x, wq, ws = _case(m, k, n, b_layout, seed=m + k + n, outliers=max(1, k // 100))
    for rep in range(2):
        rq, rs, ry = _two_launch(nq, x, wq, ws, m, k, n, b_layout, out_dtype)
        fq, fs, fy = _fused(nq, x, wq, ws, m, k, n, b_layout, out_dtype)
        torch.cuda.synchronize()
        assert nq.device_error_flags() == 0
        assert torch.equal(fq, rq), "codes"
        assert torch.equal(fs, rs), "scales"
        view = torch.int16 if out_dtype == 1 else torch.int32
        assert torch.equal(fy.view(view), ry.view(view)), "output"


@pytest.mark.parametrize("m,k,n,b_layout", [(512, 512, 1024, 0), (300, 4096, 768, 1)])
def test_fused_quantize_swiglu(nq, m, k, n, b_layout):
    import torch
    x, wq, ws = _case(m, k, n, b_layout, seed=3)
    rq, rs, ry = _two_launch(nq, x, wq, ws, m, k, n, b_layout, nq.BF16, epilogue=nq.EPI_SWIGLU)
    fq, fs, fy = _fused(nq, x, wq, ws, m, k, n, b_layout, nq.BF16, epilogue=nq.EPI_SWIGLU)
    torch.cuda.synchronize()
    assert nq.device_error_flags() == 0
    assert torch.equal(fq, rq) and torch.equal(fs, rs)
    assert torch.equal(fy.view(torch.int16), ry.view(torch.int16))


def test_config2_full_size(nq):
    """X 8192 x 4096 bf16 ~N(0,1), 41 of 4096 channels
    x20; W 4096 x 14336 ~N(0,0.02), per-output-channel E4M3; bf16 out."""
    import torch
    m, k, n = 8192, 4096, 14336
    x, wq, ws = _case(m, k, n, 0, seed=4, outliers=41)
    rq, rs, ry = _two_launch(nq, x, wq, ws, m, k, n, 0, nq.BF16)
    fq, fs, fy = _fused(nq, x, wq, ws, m, k, n, 0, nq.BF16)
    torch.cuda.synchronize()
    assert nq.device_error_flags() == 0
    assert torch.equal(fq, rq) and torch.equal(fs, rs)
    assert torch.equal(fy.view(torch.int16), ry.view(torch.int16))
    # against an fp64 product of the decoded codes, in row blocks
    f8 = torch.float8_e4m3fn
    wd = wq.view(f8).double() * ws.double()[None, :]
    worst = 0.0
    for r0 in range(0, m, 1024):
        ref = (fq[r0:r0 + 1024].view(f8).double() * fs[r0:r0 + 1024].double()[:, None]) @ wd
        got = fy[r0:r0 + 1024].double()
        floor = 1e-2 * ref.pow(2).mean().sqrt()
        worst = max(worst, float(((got - ref).abs() / torch.maximum(ref.abs(), floor)).max()))
    assert worst <= 1e-2, worst


def test_fused_quantize_argument_checks(nq):
    from nova_b200.capi import NqError
    d = nq.make_desc(256, 256, 256, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0, 16, 0, 0)
    with pytest.raises(NqError, match="row_scale must be NULL"):
        nq.gemm_quant_a(d, 16, 16, 16, 16, 16, 0)
    d = nq.make_desc(256, 256, 256, nq.INT8, nq.INT8, nq.B_KN, nq.BF16, 1.0)
    with pytest.raises(NqError):
        nq.gemm_quant_a(d, 16, 16, 16, 16, 16, 0)
    d = nq.make_desc(256, 256, 200, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0)
    with pytest.raises(NqError, match="k, n % 16"):
        nq.gemm_quant_a(d, 16, 16, 16, 16, 16, 0)
