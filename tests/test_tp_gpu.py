"""Tensor-parallel FP8 layers and the SwiGLU MLP on the GPU against the
oracle's restatement (oracle_lib.tp_mlp_partial / tp_down_partial).  tp = 1
runs in this process; tp = 2 runs tests/tp_worker.py under torchrun over
NCCL when the box has two GPUs.

Tolerances.  The SwiGLU intermediate h (bf16) and the output computed from
the GPU's own h (oracle_lib.tp_down_partial) are within 1e-2 per element
(max relative error, |ref| floored at 1e-2 rms): only the accumulation order
and one bf16 rounding differ.  Against the all-oracle pipeline the output is
compared normwise (1e-2): a 1-ulp bf16 difference in h can move single FP8
codes of the second quantization, a per-element effect the norm averages.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def rel_err(got, ref):
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    floor = 1e-2 * np.sqrt(np.mean(ref * ref)) + 1e-30
    return float(np.max(np.abs(got - ref) / np.maximum(np.abs(ref), floor)))


def weights(T, H, I, seed=7):
    import oracle_lib as O
    rng = np.random.default_rng(seed)
    x = O.f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    wg = (rng.standard_normal((H, I)) * 0.02).astype(np.float32)
    wu = (rng.standard_normal((H, I)) * 0.02).astype(np.float32)
    wd = (rng.standard_normal((I, H)) * 0.02).astype(np.float32)
    return x, wg, wu, wd


def to_dev_bf16(bits):
    import torch
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()


def bits(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().view(torch.int16).numpy().view(np.uint16)


def norm_err(got, ref):
    got = got.astype(np.float64)
    ref = ref.astype(np.float64)
    return float(np.linalg.norm(got - ref) / np.linalg.norm(ref))


def check_mlp(got_bits, h_bits_per_rank, x, wg, wu, wd, tp):
    """Returns (max h error, output error vs the GPU-h oracle, normwise
    output error vs the all-oracle pipeline).  The second is taken relative
    to sum_r |partial_r| per element (floored at 1e-2 of its rms): the
    condition of a sum whose terms may cancel."""
    import oracle_lib as O
    h_err, from_h, mag, full = 0.0, 0.0, 0.0, 0.0
    for r in range(tp):
        h_ref, part = O.tp_mlp_partial(x, wg, wu, wd, r, tp)
        h_err = max(h_err, rel_err(O.bf16_bits_to_f32(h_bits_per_rank[r]), O.bf16_bits_to_f32(h_ref)))
        p = O.bf16_bits_to_f32(O.tp_down_partial(h_bits_per_rank[r], wd, r, tp)).astype(np.float64)
        from_h, mag = from_h + p, mag + np.abs(p)
        full = full + O.bf16_bits_to_f32(part).astype(np.float64)
    got = O.bf16_bits_to_f32(got_bits).astype(np.float64)
    floor = 1e-2 * np.sqrt(np.mean(mag * mag)) + 1e-30
    out_err = float(np.max(np.abs(got - from_h) / np.maximum(mag, floor)))
    return h_err, out_err, norm_err(got, full)


@pytest.mark.parametrize("T,H,I,overlap,chunks", [(300, 256, 512, "full", None), (512, 512, 1024, "down", 3),
                                                  (600, 256, 512, "full", 3), (64, 256, 256, "full", 4)])
def test_tp1_mlp_vs_oracle(cuda, T, H, I, overlap, chunks):
    import torch
    import nova_b200.capi as nq
    from nova_b200.tp import TensorParallelMLP
    x, wg, wu, wd = weights(T, H, I)
    mlp = TensorParallelMLP(H, I, overlap=overlap, chunks=chunks)
    mlp.set_weight(wg, wu, wd)
    xin = to_dev_bf16(x)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    mlp.forward(xin, out, 1, T)
    h_err, out_err, full_err = check_mlp(bits(out), [bits(mlp._h[T])], x, wg, wu, wd, 1)
    assert h_err <= 1e-2 and out_err <= 1e-2 and full_err <= 1e-2, (h_err, out_err, full_err)
    assert nq.device_error_flags() == 0


def test_column_and_row_layers_tp1(cuda):
    import torch
    import oracle_lib as O
    from nova_b200.tp import ColumnParallelLayer, RowParallelLayer
    T, K, N = 200, 384, 512
    rng = np.random.default_rng(3)
    x = O.f32_to_bf16_bits(rng.standard_normal((T, K)).astype(np.float32))
    w = (rng.standard_normal((K, N)) * 0.02).astype(np.float32)
    xq, sx = O.quantize_rows(x, 0, bf16=True)
    wq, ws = O.quantize_cols(w, 0)
    ref = O.bf16_bits_to_f32(O.epilogue(O.gemm_fp8_acc(xq, wq, 0, 0, True), True, 1.0, sx, ws))
    for layer in (ColumnParallelLayer(K, N), RowParallelLayer(K, N)):
        layer.set_weight(w)
        out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
        layer.forward(to_dev_bf16(x), out, 2, T // 2)
        assert rel_err(O.bf16_bits_to_f32(bits(out)), ref) <= 1e-2
        with pytest.raises(ValueError):
            layer.forward(to_dev_bf16(x), out, 1, T + 1)


def test_tp2_mlp_nccl_vs_oracle(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE=os.environ.get("NCCL_NVLS_ENABLE", "1"))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(ROOT, "tests", "tp_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_WORKER_OK" in r.stdout
