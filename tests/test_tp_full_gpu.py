"""BASELINE configs[4] at full size on one GPU (tp = 1): the FP8 SwiGLU MLP
with hidden 8192, intermediate 28672 and 16384 tokens, weights ~N(0, 0.02),
x ~N(0, 1) bf16 -- the parity check bench.py reports in its tp_mlp block
(bench.tp_parity), on 64 sampled token rows:

  * per-token codes and scales of x and h bit-identical to a torch
    re-derivation of nq_quantize_rows' arithmetic;
  * h and the output within the FP8 bar (max relative error 1e-2, |ref|
    floored at 1e-2 rms) of fp64 sums over the GPU's own codes;
  * normwise within 0.1 of an fp32 computation with the unquantized weights
    (tensor_parallel_layers.cpp:561-579 in fp32).
"""
import os
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_c5_tp1_full_size_parity(cuda):
    import torch
    sys.path.insert(0, ROOT)
    import bench
    from nova_b200.tp import TensorParallelMLP
    T, H, I = 16384, 8192, 28672
    g = torch.Generator(device="cuda").manual_seed(11)
    mlp = TensorParallelMLP(H, I)
    wg = torch.randn(H, I, device="cuda", generator=g).mul_(0.02)
    wu = torch.randn(H, I, device="cuda", generator=g).mul_(0.02)
    wd = torch.randn(I, H, device="cuda", generator=g).mul_(0.02)
    mlp.set_weight(wg, wu, wd)
    x = torch.randn(T, H, device="cuda", generator=g).to(torch.bfloat16)
    y = torch.empty(T, H, dtype=torch.bfloat16, device="cuda")
    mlp.forward(x, y, 1, T)
    rows = sorted(set(int(v) for v in torch.linspace(0, T - 1, 64).round().tolist()))
    res = bench.tp_parity(mlp, x, y, (wg, wu, wd), rows, 1)
    assert res["ok"], res
    assert res["codes_bit_exact"] and res["device_errors"] == 0
