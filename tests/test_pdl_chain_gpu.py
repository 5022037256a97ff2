"""Back-to-back launches with programmatic dependent launch.

The per-token quantize, the pair GEMM and the decode GEMM start their prologue
while the previous kernel of the stream finishes and wait (griddepcontrol.wait)
before touching memory it may write.  Here each GEMM reads the codes and scales
the quantize launch right before it produced, from inputs that change every
step; run back to back on one stream, every output must equal the output of the
same step run alone between two synchronizations (all kernels are
deterministic), so a GEMM that read its operands early would show up as a
mismatch."""
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nq(cuda):
    import nova_b200.capi as capi
    return capi


@pytest.mark.parametrize("tokens", [16, 64, 512])
def test_quantize_then_gemm_back_to_back(nq, tokens):
    import torch
    K, N, steps = 4096, 8192, 6
    g = torch.Generator(device="cuda").manual_seed(tokens)
    w = torch.randn(K, N, device="cuda", generator=g).mul_(0.02)
    wq = torch.empty(K, N, dtype=torch.uint8, device="cuda")
    ws = torch.empty(N, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    nq.quantize_cols(w.data_ptr(), wq.data_ptr(), ws.data_ptr(), K, N, nq.E4M3, s)
    xs = [torch.randn(tokens, K, device="cuda", generator=g).to(torch.bfloat16) for _ in range(steps)]
    xq = torch.empty(tokens, K, dtype=torch.uint8, device="cuda")
    sx = torch.empty(tokens, device="cuda")
    outs = [torch.empty(tokens, N, dtype=torch.bfloat16, device="cuda") for _ in range(steps)]
    desc = nq.make_desc(tokens, N, K, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0, sx.data_ptr(), ws.data_ptr(), 0)

    def step(i):
        nq.quantize_rows(xs[i].data_ptr(), nq.BF16, xq.data_ptr(), sx.data_ptr(), tokens, K, nq.E4M3, s)
        nq.gemm(desc, xq.data_ptr(), wq.data_ptr(), outs[i].data_ptr(), s)

    refs = []
    for i in range(steps):
        torch.cuda.synchronize()
        step(i)
        torch.cuda.synchronize()
        refs.append(outs[i].clone())
        outs[i].zero_()
    torch.cuda.synchronize()
    for _ in range(3):
        for i in range(steps):
            step(i)
        torch.cuda.synchronize()
        for i in range(steps):
            assert torch.equal(outs[i].view(torch.int16), refs[i].view(torch.int16)), i
            outs[i].zero_()
    assert nq.device_error_flags() == 0
