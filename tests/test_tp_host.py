"""Host logic of the tensor-parallel MLP, on CPU: weight sharding as the
reference's set_weight slices it (tensor_parallel_layers.cpp:111-136,
:344-368), the packed gate/up column order of the SwiGLU GEMM, the token
chunking of the overlapped all-reduce, and the chunked all-reduce pipeline
itself run by two gloo ranks on oracle-computed partials."""
import os
import socket

import numpy as np
import pytest

from nova_b200 import tp


def test_shards_partition_the_weight():
    w = np.arange(8 * 12, dtype=np.float32).reshape(8, 12)
    for t in (1, 2, 4):
        cols = [tp.shard_columns(w, r, t) for r in range(t)]
        rows = [tp.shard_rows(w, r, t) for r in range(t)]
        np.testing.assert_array_equal(np.concatenate(cols, axis=1), w)
        np.testing.assert_array_equal(np.concatenate(rows, axis=0), w)
        assert cols[-1].shape == (8, 12 // t) and rows[-1].shape == (8 // t, 12)
    with pytest.raises(ValueError):
        tp.shard_columns(w, 0, 5)
    with pytest.raises(ValueError):
        tp.shard_rows(w, 0, 3)


def test_pack_order_is_block_interleaved_permutation():
    for il in (128, 384, 3584):
        o = tp.swiglu_pack_order(il)
        assert sorted(o.tolist()) == list(range(2 * il))
        blocks = o.reshape(-1, 256)
        assert (blocks[:, :128] < il).all() and (blocks[:, 128:] >= il).all()
        np.testing.assert_array_equal(blocks[:, 128:] - il, blocks[:, :128])
    with pytest.raises(ValueError):
        tp.swiglu_pack_order(200)


@pytest.mark.parametrize("tokens,chunks", [(16384, 4), (300, 4), (256, 8), (1, 4), (1000, 1), (4097, 3)])
def test_chunk_bounds_cover_tokens(tokens, chunks):
    b = tp.chunk_bounds(tokens, chunks)
    assert b[0][0] == 0 and b[-1][1] == tokens
    assert all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))
    assert all((r0 % 256) == 0 and r1 > r0 for r0, r1 in b)
    assert len(b) <= chunks
    assert tp.chunk_bounds(0, 4) == []


@pytest.mark.parametrize("tokens,tp_", [(16384, 8), (16384, 4), (16384, 2), (300, 8), (1, 4), (4097, 8), (16384, 1)])
def test_plan_chunks_cover_tokens(tokens, tp_):
    b = tp.plan_chunks(tokens, 2 * 28672 // tp_, 8192, 8192, 28672 // tp_, tp_)
    assert b[0][0] == 0 and b[-1][1] == tokens
    assert all(b[i][1] == b[i + 1][0] for i in range(len(b) - 1))
    assert all((r0 % 256) == 0 and r1 > r0 for r0, r1 in b)
    assert 1 <= len(b) <= 8
    if tp_ == 1:
        assert b == [(0, tokens)]
    assert tp.plan_chunks(0, 256, 256, 256, 256, 4) == []


def test_mlp_chunk_rows_option():
    mlp = tp.TensorParallelMLP(256, 512, chunk_rows=512)
    assert mlp._bounds(1300) == [(0, 512), (512, 1024), (1024, 1300)]
    mlp = tp.TensorParallelMLP(256, 512, chunks=3)
    assert mlp._bounds(1300) == tp.chunk_bounds(1300, 3)
    mlp = tp.TensorParallelMLP(256, 512, chunk_rows="plan")
    assert mlp._bounds(1300) == [(0, 1300)]      # tp = 1: one chunk
    for bad in (0, -256, 300, "many"):
        with pytest.raises(ValueError):
            tp.TensorParallelMLP(256, 512, chunk_rows=bad)


def test_packed_swiglu_equals_separate_gate_up():
    """The packed GEMM's accumulators are the separate gate/up accumulators
    permuted (bit-identical), and the SwiGLU epilogue on them equals
    silu(g) * u of the separately scaled values."""
    import oracle_lib as O
    rng = np.random.default_rng(0)
    T, H, il = 64, 128, 256
    x = rng.standard_normal((T, H)).astype(np.float32)
    g = (rng.standard_normal((H, il)) * 0.02).astype(np.float32)
    u = (rng.standard_normal((H, il)) * 0.02).astype(np.float32)
    xq, sx = O.quantize_rows(x, 0)
    gq, gs = O.quantize_cols(g, 0)
    uq, us = O.quantize_cols(u, 0)
    order = tp.swiglu_pack_order(il)
    pq = np.ascontiguousarray(np.concatenate([gq, uq], axis=1)[:, order])
    ps = np.concatenate([gs, us])[order]
    pq2, ps2 = O.quantize_cols(np.ascontiguousarray(np.concatenate([g, u], axis=1)[:, order]), 0)
    np.testing.assert_array_equal(pq, pq2)
    np.testing.assert_array_equal(ps, ps2)
    acc = O.gemm_fp8_acc(xq, pq, 0, 0, True)
    ga, ua = O.gemm_fp8_acc(xq, gq, 0, 0, True), O.gemm_fp8_acc(xq, uq, 0, 0, True)
    np.testing.assert_array_equal(acc, np.concatenate([ga, ua], axis=1)[:, order])
    h = O.swiglu_epilogue(acc, False, 1.0, sx, ps)
    gv = ga * sx[:, None] * gs[None, :]
    uv = ua * sx[:, None] * us[None, :]
    ref = np.vectorize(lambda a, b: O.lib.orc_silu_mul(float(a), float(b)), otypes=[np.float32])(gv, uv)
    np.testing.assert_allclose(h, ref, rtol=2e-6, atol=1e-30)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, case):
    import torch
    import torch.distributed as dist
    import oracle_lib as O
    from nova_b200 import tp as tpm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, H, I = case
        rng = np.random.default_rng(7)
        x = O.f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
        wg = (rng.standard_normal((H, I)) * 0.02).astype(np.float32)
        wu = (rng.standard_normal((H, I)) * 0.02).astype(np.float32)
        wd = (rng.standard_normal((I, H)) * 0.02).astype(np.float32)
        _, part = O.tp_mlp_partial(x, wg, wu, wd, rank, world)
        out = torch.zeros(T, H, dtype=torch.float32)
        src = torch.from_numpy(O.bf16_bits_to_f32(part))
        seen = []

        def compute(r0, r1):
            seen.append((r0, r1))
            out[r0:r1] = src[r0:r1]
            return out[r0:r1]

        tpm.reduce_pipeline(tpm.chunk_bounds(T, 4), compute, None, world)
        assert seen == tpm.chunk_bounds(T, 4)
        want = sum(O.bf16_bits_to_f32(O.tp_mlp_partial(x, wg, wu, wd, r, world)[1]) for r in range(world))
        np.testing.assert_array_equal(out.numpy(), want)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(600, 256, 512)])
def test_reduce_pipeline_two_gloo_ranks(case):
    import torch.multiprocessing as mp
    mp.start_processes(_gloo_rank, args=(2, _free_port(), case), nprocs=2, join=True, start_method="spawn")


def test_fused_allreduce_descriptors():
    """The descriptors the chunked MLP pipeline hands to nq_gemm_allreduce:
    per-chunk counter offsets, job rows offset into the symmetric buffers,
    the completion target of an epoch (host logic only, fake addresses)."""
    import nova_b200.capi as nq
    ar = object.__new__(tp.SymmetricAllReduce)
    ar.nq, ar.tp, ar.rank = nq, 4, 1
    T, n = 1300, 512
    bounds = tp.chunk_bounds(T, 3)
    assert len(bounds) == 3
    offs, tiles = [], 0
    for r0, r1 in bounds:
        offs.append(tiles)
        tiles += nq.gemm_allreduce_counters(r1 - r0, n)

    class FakeT:
        def __init__(self, p):
            self.p = p

        def data_ptr(self):
            return self.p

    per_forward = sum(nq.allreduce_done_per_job(r1 - r0, n, int(c == len(bounds) - 1))
                      for c, (r0, r1) in enumerate(bounds))
    st = tp._ArState(m=T, n=n, bounds=bounds, offs=offs, flags=FakeT(1 << 20), done=FakeT(2 << 20),
                     partial=FakeT(3 << 20), out=FakeT(4 << 20), pf=[(10 + r) << 20 for r in range(4)],
                     pd=[(20 + r) << 20 for r in range(4)], pp=[(30 + r) << 20 for r in range(4)],
                     po=[(40 + r) << 20 for r in range(4)], mcp=50 << 20, mco=60 << 20, mcd=70 << 20,
                     use_mc=True, per_forward=per_forward, epoch=0)
    ar.begin(st)
    ar.begin(st)
    assert st.epoch == 2
    d = ar.desc(st, signal=1)
    assert d.signal == 1 and d.m == 0 and d.done_target == 0 and d.epoch == 2
    assert [d.signal_flags[r] for r in range(4)] == [((10 + r) << 20) + 4 * offs[1] for r in range(4)]
    r0, r1 = bounds[2]
    d = ar.desc(st, signal=2, job=2, finish=True)
    assert (d.m, d.n) == (r1 - r0, n)
    assert d.flags == (1 << 20) + 4 * offs[2]
    assert d.mc_partial == (50 << 20) + 2 * r0 * n and d.mc_out == (60 << 20) + 2 * r0 * n
    assert d.mc_done == 70 << 20 and d.done == 2 << 20
    assert d.done_target == 2 * per_forward
    assert [d.peer_partial[r] for r in range(4)] == [((30 + r) << 20) + 2 * r0 * n for r in range(4)]
    st.use_mc = False
    d = ar.desc(st, job=0)
    assert d.mc_partial is None and d.peer_out[3] == (43 << 20)
    last = nq.gemm_allreduce_counters(bounds[-1][1] - bounds[-1][0], n)
    assert per_forward == 5 * (tiles - last) + 4 * last
    # counters wrap: near 2^32 forwards the epoch and the completion target are
    # the use count and its counter total modulo 2^32, and the finish is keyed
    # on `done`, so a target that wraps to exactly 0 still waits
    for epoch in ((1 << 32) - 2, (1 << 32) - 1, 1 << 32, (1 << 32) + 1):
        st.epoch = epoch - 1
        ar.begin(st)
        d = ar.desc(st, signal=2, job=2, finish=True)
        assert d.epoch == epoch % (1 << 32)
        assert d.done_target == (epoch * per_forward) % (1 << 32) and d.done == 2 << 20
    st.per_forward, st.epoch = 1 << 31, 2
    d = ar.desc(st, finish=True)
    assert d.done_target == 0 and d.done == 2 << 20


def _counter_reached(v, want):
    """The kernels' counter compare (gemm.cu counter_reached): v has reached
    want when their difference modulo 2^32, read as a signed 32-bit value, is
    not negative."""
    diff = (v - want) % (1 << 32)
    return diff < (1 << 31)


def test_counter_compare_wraps():
    """A counter that wrapped past 2^32 still compares right against a target
    that wrapped too, and one a forward short of it still waits."""
    per_forward, tp_ = 5 * 2048, 8
    for epoch in (1, 2, (1 << 32) // per_forward, (1 << 32) // per_forward + 1, (1 << 32) - 1):
        target = (epoch * per_forward) % (1 << 32)
        assert _counter_reached(target, target)
        assert not _counter_reached((target - 1) % (1 << 32), target)
        assert not _counter_reached((target - per_forward) % (1 << 32), target)
        assert _counter_reached((target + per_forward) % (1 << 32), target)   # a peer already one forward on
        flag_want = (epoch * tp_) % (1 << 32)
        assert _counter_reached(flag_want, flag_want)
        assert not _counter_reached((flag_want - 1) % (1 << 32), flag_want)


def test_layer_argument_checks_without_gpu():
    """Shape and option errors are raised on the host before any device work
    (the reference throws std::invalid_argument, tensor_parallel_layers.cpp)."""
    with pytest.raises(ValueError):
        tp.TensorParallelMLP(256, 200)            # intermediate not a multiple of 128
    with pytest.raises(ValueError):
        tp.TensorParallelMLP(250, 256)            # hidden not a multiple of 16
    with pytest.raises(ValueError):
        tp.TensorParallelMLP(256, 256, overlap="sideways")
    with pytest.raises(ValueError):
        tp.RowParallelLayer(256, 256, allreduce="carrier-pigeon")
    mlp = tp.TensorParallelMLP(256, 512)
    assert (mlp.tp, mlp.rank, mlp.chunks, mlp.I_local) == (1, 0, 1, 512)
    assert mlp.down.fused is None                 # tp = 1: no all-reduce at all
    with pytest.raises(RuntimeError):
        mlp.forward(None, None, 1, 4)             # weights not set
