"""Tensor-parallel FP8 layers and the SwiGLU MLP on the GPU against the
oracle's restatement (oracle_lib.tp_mlp_partial).  tp = 1 runs in this
process; tp = 2 runs tests/tp_worker.py under torchrun over NCCL when the
box has two GPUs.  Tolerances: the SwiGLU intermediate h (bf16) within
1e-2 relative (the FP8 bar), the MLP output within 2e-2 (h's bf16 rounding
can move single FP8 codes of the second quantization)."""
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


@pytest.mark.parametrize("T,H,I,overlap", [(300, 256, 512, "full"), (512, 512, 1024, "down"), (64, 256, 256, "full")])
def test_tp1_mlp_vs_oracle(cuda, T, H, I, overlap):
    import torch
    import oracle_lib as O
    import nova_b200.capi as nq
    from nova_b200.tp import TensorParallelMLP
    x, wg, wu, wd = weights(T, H, I)
    mlp = TensorParallelMLP(H, I, overlap=overlap)
    mlp.set_weight(wg, wu, wd)
    xin = to_dev_bf16(x)
    out = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    mlp.forward(xin, out, 1, T)
    h_ref, out_ref = O.tp_mlp_partial(x, wg, wu, wd, 0, 1)
    assert rel_err(O.bf16_bits_to_f32(bits(mlp._h[T])), O.bf16_bits_to_f32(h_ref)) <= 1e-2
    assert rel_err(O.bf16_bits_to_f32(bits(out)), O.bf16_bits_to_f32(out_ref)) <= 2e-2
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
