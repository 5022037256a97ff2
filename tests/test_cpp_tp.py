"""The drop-in C++ tensor-parallel layers (include/cuda/neural/
tensor_parallel_layers.h over include/cuda/nccl/nccl_context.h), run by
tests/cpp/test_tp.cpp with one host thread per GPU as the reference's own
tests do (tests/neural/tensor_parallel_multigpu_test.cpp:578-621), checked
against the oracle restatement of the same W8A8 FP8 pipeline.

Bars:
  * ColumnParallelLayer, RowParallelLayer at tp = 1: element-wise within the
    FP8 bar (max relative error 1e-2, |ref| floored at 1e-2 rms) of the
    oracle's GEMM on the same codes and scales;
  * RowParallelLayer at tp > 1, relative to sum_r |partial_r| (the condition
    of a sum whose terms cancel): the fp32 ncclAllReduce path within 1e-3 of
    the oracle's fp32 partials summed; the GEMM-fused path (bf16 partials
    summed in fp32, one bf16 rounding) within 2^-7 + 2^-8 + 1e-3 -- each
    rank's partial may round one bf16 ulp apart from the oracle's, plus the
    final rounding;
  * TensorParallelMLP: normwise within 1e-2 of the all-oracle pipeline (a
    1-ulp bf16 difference in h can move single FP8 codes of the second
    quantization, which the norm averages), and every rank's output
    bit-identical.
"""
import os
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "tests", "cpp", "bin", "test_tp")


def _exe():
    if not os.path.exists(EXE):
        pytest.fail("tests/cpp/bin/test_tp is not built: run __graft_entry__.build()")
    return EXE


def test_cpp_tp_host_checks():
    """Shape and argument errors, the uninitialized context's behaviour and
    NcclResult, before any device work (std::invalid_argument as the
    reference throws, tensor_parallel_layers.cpp:36-52)."""
    r = subprocess.run([_exe(), "checks"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failures" in r.stdout


def _load(d, name, shape):
    return np.fromfile(os.path.join(d, name), dtype=np.float32).reshape(shape)


def _rel(got, ref, mag=None):
    got, ref = got.astype(np.float64), ref.astype(np.float64)
    mag = np.abs(ref) if mag is None else mag
    floor = 1e-2 * np.sqrt(np.mean(mag * mag)) + 1e-30
    return float(np.max(np.abs(got - ref) / np.maximum(mag, floor)))


def _mlp_partials(x, wg, wu, wd, h, inter, tp, bf16_partial):
    """Each rank's partial of the drop-in MLP on the oracle: per-token E4M3
    of the fp32 input, the rank's gate / up shards packed in 128-column
    blocks and zero-padded to a multiple of 128, SwiGLU to bf16 h, per-token
    E4M3 of h, the zero-padded down shard."""
    import oracle_lib as O
    L = inter // tp
    pad = (L + 127) // 128 * 128
    xq, sx = O.quantize_rows(np.ascontiguousarray(x), 0)
    parts = []
    for r in range(tp):
        packed = np.zeros((h, 2 * pad), np.float32)
        for c in range(L):
            b, col = divmod(c, 128)
            packed[:, 256 * b + col] = wg[:, r * L + c]
            packed[:, 256 * b + 128 + col] = wu[:, r * L + c]
        gq, gs = O.quantize_cols(packed, 0)
        hb = O.swiglu_epilogue(O.gemm_fp8_acc(xq, gq, 0, 0, True), True, 1.0, sx, gs)
        hq, sh = O.quantize_rows(np.ascontiguousarray(hb), 0, bf16=True)
        down = np.zeros((pad, h), np.float32)
        down[:L] = wd[r * L:(r + 1) * L]
        dq, ds = O.quantize_cols(down, 0)
        acc = O.gemm_fp8_acc(hq, dq, 0, 0, True)
        p = O.epilogue(acc, bf16_partial, 1.0, sh, ds)
        parts.append(O.bf16_bits_to_f32(p) if bf16_partial else p)
    return parts


def _lin_partials(x, w, m, k, n, tp, row, bf16_partial):
    import oracle_lib as O
    if not row:
        xq, sx = O.quantize_rows(np.ascontiguousarray(x), 0)
        wq, ws = O.quantize_cols(np.ascontiguousarray(w[:, :n // tp]), 0)
        return [O.epilogue(O.gemm_fp8_acc(xq, wq, 0, 0, True), False, 1.0, sx, ws)]
    kl = k // tp
    parts = []
    for r in range(tp):
        xq, sx = O.quantize_rows(np.ascontiguousarray(x[:, r * kl:(r + 1) * kl]), 0)
        wq, ws = O.quantize_cols(np.ascontiguousarray(w[r * kl:(r + 1) * kl]), 0)
        p = O.epilogue(O.gemm_fp8_acc(xq, wq, 0, 0, True), bf16_partial, 1.0, sx, ws)
        parts.append(O.bf16_bits_to_f32(p) if bf16_partial else p)
    return parts


def _run_and_check(tp, tmp_path):
    r = subprocess.run([_exe(), "run", str(tp), str(tmp_path)], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    report = []
    for line in r.stdout.splitlines():
        if not line.startswith("case "):
            continue
        f = dict(kv.split("=") for kv in line.split()[2:])
        name, m, tp_ = line.split()[1], int(f["m"]), int(f["tp"])
        if name.startswith("mlp"):
            h, inter, fused = int(f["h"]), int(f["inter"]), f["fused"] == "1"
            x = _load(tmp_path, f"{name}_x.bin", (m, h))
            wg, wu = _load(tmp_path, f"{name}_wg.bin", (h, inter)), _load(tmp_path, f"{name}_wu.bin", (h, inter))
            wd = _load(tmp_path, f"{name}_wd.bin", (inter, h))
            ref = sum(p.astype(np.float64) for p in _mlp_partials(x, wg, wu, wd, h, inter, tp_, fused))
            outs = [_load(tmp_path, f"{name}_out{q}.bin", (m, h)) for q in range(tp_)]
            err = float(np.linalg.norm(outs[0] - ref) / np.linalg.norm(ref))
            report.append((name, err))
            assert err <= 1e-2, (name, err)
        else:
            k, n = int(f["k"]), int(f["n"])
            row = name.startswith("row")
            x = _load(tmp_path, f"{name}_x.bin", (m, k))
            w = _load(tmp_path, f"{name}_w.bin", (k, n))
            fused = row and tp_ > 1 and not name.endswith("nccl") and n % 256 == 0
            parts = [p.astype(np.float64) for p in _lin_partials(x, w, m, k, n, tp_, row, fused)]
            ref = sum(parts)
            mag = sum(np.abs(p) for p in parts)
            ncol = n // tp_ if not row else n
            outs = [_load(tmp_path, f"{name}_out{q}.bin", (m, ncol)) for q in range(tp_)]
            bound = 1e-2 if tp_ == 1 or not row else (2.0 ** -7 + 2.0 ** -8 + 1e-3 if fused else 1e-3)
            err = _rel(outs[0], ref, mag)
            report.append((name, err))
            assert err <= bound, (name, err, bound)
            if not row:
                continue
        for q in range(1, tp_):
            assert np.array_equal(outs[q], outs[0]), f"{name}: rank {q} output differs from rank 0"
    assert len(report) == 8, r.stdout
    if tp > 1 and "peer_access=1" in r.stdout:
        # with peer access the 512-wide MLP reduces inside its down GEMM
        assert "case mlp_mid m=200 h=512 inter=%d tp=%d fused=1" % (768 * tp, tp) in r.stdout, r.stdout
        assert "case mlp_mid_nccl m=200 h=512 inter=%d tp=%d fused=0" % (768 * tp, tp) in r.stdout, r.stdout
    print(r.stdout, report)
    return report


@pytest.mark.gpu
def test_cpp_tp_one_gpu(cuda, tmp_path):
    """tp = 1 on an uninitialized context: the reference's single-GPU
    fall-back (tensor_parallel_layers_test.cpp:150-235) on FP8."""
    _run_and_check(1, tmp_path)


@pytest.mark.gpu
def test_cpp_tp_two_gpus(cuda, tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    _run_and_check(2, tmp_path)
