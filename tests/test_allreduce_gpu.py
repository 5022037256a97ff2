"""The GEMM-fused all-reduce kernels (nq_gemm_allreduce, nq_allreduce_finish)
on ONE GPU, through the C ABI: tp = 1, the rank's own buffers standing in
for the peers' (the peer path).  A one-rank all-reduce is the identity on the
bf16 partial (an fp32 sum of one bf16 value rounds back to it), so the
reduced output must equal the plain bf16 GEMM bit for bit.

Covered here, with no second GPU:
  * signal + job + finish in one kernel (RowParallelLayer::forward as one
    launch, tensor_parallel_layers.cpp:370-416) against nq_gemm;
  * counters and targets that wrap past 2^32 (compared modulo 2^32);
  * bounded waits that run out: a job whose tile counters nothing raises and
    a finish whose target nothing reaches, under a 20 ms wait limit
    (nq_set_peer_wait_limit).  The kernel returns, the stream completes, and
    bit 0 of the device error word is set -- the device-side analogue of the
    reference's safe_stream_wait deadline (src/cuda/nccl/nccl_error.cpp:13-83).
"""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def nq(cuda):
    import nova_b200.capi as capi
    capi.device_error_flags()   # start clean
    return capi


def _operands(m, n, k, seed):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = torch.randint(0, 256, (m, k), dtype=torch.uint8, device="cuda", generator=g)
    b = torch.randint(0, 256, (k, n), dtype=torch.uint8, device="cuda", generator=g)
    # keep the codes finite and moderate: clear NaN patterns (0x7F / 0xFF) and the top exponents
    a = torch.where((a & 0x7F) >= 0x70, a & 0x8F, a)
    b = torch.where((b & 0x7F) >= 0x70, b & 0x8F, b)
    rs = torch.rand(m, device="cuda", generator=g) + 0.5
    cs = torch.rand(n, device="cuda", generator=g) * 1e-2 + 1e-3
    return a, b, rs, cs


def _counters(m, n, flag0, done0):
    import torch
    tiles = max(1, m // 256 + (m % 256 > 0)) * (n // 256)
    flags = torch.full((tiles,), flag0, dtype=torch.int64, device="cuda").to(torch.int32) \
        if flag0 < (1 << 31) else torch.full((tiles,), flag0 - (1 << 32), dtype=torch.int32, device="cuda")
    done = torch.tensor([done0 if done0 < (1 << 31) else done0 - (1 << 32)], dtype=torch.int32, device="cuda")
    return flags, done


def _desc_tp1(nq, m, n, flags, done, partial, out, epoch, done_target, signal=True, job=True, finish=True):
    d = nq.AllreduceDesc()
    d.tp, d.rank, d.epoch = 1, 0, epoch & 0xFFFFFFFF
    if signal:
        d.signal = 1
        d.signal_flags[0] = flags.data_ptr()
    if job:
        d.m, d.n = m, n
        d.flags = flags.data_ptr()
        d.peer_partial[0], d.peer_out[0], d.peer_done[0] = partial.data_ptr(), out.data_ptr(), done.data_ptr()
    if finish:
        d.done = done.data_ptr()
        d.done_target = done_target & 0xFFFFFFFF
    return d


@pytest.mark.parametrize("m,n,k", [(512, 512, 256), (300, 768, 512), (1024, 1024, 1024)])
@pytest.mark.parametrize("start", ["zero", "wrap"])
def test_fused_row_parallel_tp1_equals_gemm(nq, m, n, k, start):
    import torch
    a, b, rs, cs = _operands(m, n, k, seed=m + n + k)
    s = torch.cuda.current_stream().cuda_stream
    desc = nq.make_desc(m, n, k, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 0.5, rs.data_ptr(), cs.data_ptr(), 0)
    ref = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    nq.gemm(desc, a.data_ptr(), b.data_ptr(), ref.data_ptr(), s)
    per_forward = nq.allreduce_done_per_job(m, n, 1)
    tiles = nq.gemm_allreduce_counters(m, n)
    # "wrap": the counters start so close to 2^32 that the 2nd and 3rd forwards wrap
    if start == "zero":
        e0, flag0, done0 = 0, 0, 0
    else:
        e0 = (1 << 32) - 2
        flag0 = e0 % (1 << 32)                       # tp = 1: one count per tile and epoch
        done0 = (e0 * per_forward) % (1 << 32)
    flags, done = _counters(m, n, flag0, done0)
    assert flags.numel() == tiles
    partial = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    for i in range(1, 5):
        epoch = e0 + i
        out.zero_()
        d = _desc_tp1(nq, m, n, flags, done, partial, out, epoch, epoch * per_forward)
        nq.gemm_allreduce(desc, C.byref(d), a.data_ptr(), b.data_ptr(), partial.data_ptr(), s)
        torch.cuda.synchronize()
        assert nq.device_error_flags() == 0, f"a wait timed out at forward {i}"
        assert torch.equal(partial.view(torch.int16), ref.view(torch.int16))
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16)), f"forward {i}"
        got_done = int(done.item()) & 0xFFFFFFFF
        assert got_done == (epoch * per_forward) % (1 << 32)
        assert (flags.to(torch.int64) & 0xFFFFFFFF).eq(epoch % (1 << 32)).all()


def test_finish_without_a_gemm_tp1(nq):
    """A GEMM that only signals, then nq_allreduce_finish runs the job and the
    completion wait (the last chunk of the pipeline without a host GEMM)."""
    import torch
    m, n, k = 512, 768, 256
    a, b, rs, cs = _operands(m, n, k, seed=5)
    s = torch.cuda.current_stream().cuda_stream
    desc = nq.make_desc(m, n, k, nq.E4M3, nq.E4M3, nq.B_NK, nq.BF16, 1.0, rs.data_ptr(), cs.data_ptr(), 0)
    bnk = b.reshape(n, k).contiguous()
    ref = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    nq.gemm(desc, a.data_ptr(), bnk.data_ptr(), ref.data_ptr(), s)
    flags, done = _counters(m, n, 0, 0)
    partial = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    per_job = nq.allreduce_done_per_job(m, n, 0)
    for epoch in (1, 2):
        d1 = _desc_tp1(nq, m, n, flags, done, partial, out, epoch, 0, signal=True, job=False, finish=False)
        nq.gemm_allreduce(desc, C.byref(d1), a.data_ptr(), bnk.data_ptr(), partial.data_ptr(), s)
        d2 = _desc_tp1(nq, m, n, flags, done, partial, out, epoch, epoch * per_job, signal=False)
        nq.allreduce_finish(C.byref(d2), s)
        torch.cuda.synchronize()
        assert nq.device_error_flags() == 0
        assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
        assert int(done.item()) == epoch * per_job


@pytest.fixture
def short_peer_wait(nq):
    old = nq.peer_wait_limit()
    nq.set_peer_wait_limit(20_000_000)           # 20 ms
    assert nq.peer_wait_limit() == 20_000_000
    yield
    nq.set_peer_wait_limit(0)                    # back to the default
    assert nq.peer_wait_limit() == old == 5_000_000_000


def test_wait_for_tiles_nobody_signals_times_out(nq, short_peer_wait):
    """A job whose tile counters no GEMM ever raises: every reducer warp gives
    up after the limit, the kernel returns and reports the timeout."""
    import torch
    m, n = 512, 512
    flags, done = _counters(m, n, 0, 0)
    partial = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    out = torch.full((m, n), 7.0, dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    d = _desc_tp1(nq, m, n, flags, done, partial, out, 1, 0, signal=False, job=True, finish=False)
    t0 = time.perf_counter()
    nq.allreduce_finish(C.byref(d), s)
    torch.cuda.synchronize()                      # the stream completes
    dt = time.perf_counter() - t0
    assert (nq.device_error_flags() & 1) == 1
    assert nq.device_error_flags() == 0           # cleared by the read above
    assert dt < 2.0, dt                           # bounded by the 20 ms limit, not the 5 s default
    assert torch.all(out == 7.0)                  # nothing was reduced
    assert int(done.item()) == 0


def test_finish_target_never_reached_times_out(nq, short_peer_wait):
    """A completion wait whose target nothing reaches (a peer that never
    joined): the waiting thread gives up after the limit and flags it; the
    next launch on the same context runs normally."""
    import torch
    m, n = 256, 256
    flags, done = _counters(m, n, 0, 0)
    partial = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    d = _desc_tp1(nq, m, n, flags, done, partial, out, 1, 5, signal=False, job=False, finish=True)
    t0 = time.perf_counter()
    nq.allreduce_finish(C.byref(d), s)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 2.0
    assert nq.device_error_flags() == 1
    # the context is still usable: a normal GEMM right after
    a, b, rs, cs = _operands(256, 256, 256, seed=9)
    desc = nq.make_desc(256, 256, 256, nq.E4M3, nq.E4M3, nq.B_KN, nq.BF16, 1.0, 0, 0, 0)
    o1 = torch.empty(256, 256, dtype=torch.bfloat16, device="cuda")
    nq.gemm(desc, a.data_ptr(), b.data_ptr(), o1.data_ptr(), s)
    o2 = torch.empty_like(o1)
    nq.gemm_simt(desc, a.data_ptr(), b.data_ptr(), o2.data_ptr(), s)
    torch.cuda.synchronize()
    assert nq.device_error_flags() == 0
    d1, d2 = o1.float(), o2.float()
    assert torch.max(torch.abs(d1 - d2) / torch.clamp(torch.abs(d2), min=float(1e-2 * d2.abs().max()))).item() <= 1e-2
