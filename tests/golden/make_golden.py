"""Generates tests/golden/*.npz from the reference's OWN host code
(pplmx/nova headers compiled by oracle/Makefile into
oracle/_ref/libnova_ref_host.so):

  fp8_codec.npz      FP8E4M3(float) / FP8E5M2(float) codes of seeded and edge
                     inputs, and operator float of all 256 codes
                     (include/cuda/quantize/fp8_types.hpp:64-207)
  from_float.npz     QuantizedTensor<int8_t>::FromFloat (quantize_tensor.hpp:160-191)
  quantized_matmul.npz  QuantizedMatmul::forward (quantize_ops.hpp:54-81)
  qat_fake_quant.npz FakeQuantize::forward (qat.hpp:64-72) at several scales and
                     zero points, edge inputs included

Run from the repository root after `make -C oracle ref`:
    python tests/golden/make_golden.py          # every fixture
    python tests/golden/make_golden.py qat      # qat_fake_quant.npz only
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
import oracle_lib as O  # noqa: E402


def main():
    r = O.ref_host()
    if r is None:
        raise SystemExit("oracle/_ref/libnova_ref_host.so missing: run `make -C oracle ref` first")
    rng = np.random.default_rng(20261201)
    # inputs: edge values, a log-uniform sweep over every exponent the codecs
    # touch, and raw random bit patterns
    edge = O.special_floats()
    mag = np.exp2(rng.uniform(-24, 20, 6000)).astype(np.float32)
    sweep = mag * np.where(rng.random(6000) < 0.5, -1, 1).astype(np.float32)
    bits = rng.integers(0, 1 << 32, 2000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    x = np.concatenate([edge, sweep, bits]).astype(np.float32)
    e4 = np.array([r.ref_e4m3_encode(float(v)) for v in x], np.uint8)
    e5 = np.array([r.ref_e5m2_encode(float(v)) for v in x], np.uint8)
    d4 = np.array([r.ref_e4m3_decode(c) for c in range(256)], np.float32)
    d5 = np.array([r.ref_e5m2_decode(c) for c in range(256)], np.float32)
    np.savez_compressed(os.path.join(HERE, "fp8_codec.npz"), x=x, e4m3=e4, e5m2=e5, dec_e4m3=d4, dec_e5m2=d5)

    cases = {}
    for i, (n, scale) in enumerate([(1000, 0.0), (1000, 0.05), (37, 0.0), (64, 1e-3)]):
        v = (rng.standard_normal(n) * (3.0 if i % 2 == 0 else 1.0)).astype(np.float32)
        v[: min(4, n)] = [0.5 * 0.05, -1.5 * 0.05, 2.5 * 0.05, 1000.0][: min(4, n)]
        q = np.empty(n, np.int8)
        s = C.c_float()
        assert r.ref_from_float_int8(v.ctypes.data, n, scale, q.ctypes.data, C.byref(s)) == 1
        cases[f"x{i}"], cases[f"scale_in{i}"], cases[f"q{i}"], cases[f"scale{i}"] = v, np.float32(scale), q, np.float32(s.value)
    np.savez_compressed(os.path.join(HERE, "from_float.npz"), **cases)

    mm = {}
    for i, (m, k, n, sa, sb) in enumerate([(2, 3, 2, 0.1, 0.2), (8, 16, 12, 0.01, 0.02), (5, 64, 7, 0.003, 0.004)]):
        a = rng.integers(-127, 128, (m, k), dtype=np.int8)
        b = rng.integers(-127, 128, (k, n), dtype=np.int8)
        out = np.empty((m, n), np.int8)
        r.ref_quantized_matmul(a.ctypes.data, b.ctypes.data, out.ctypes.data, m, k, n, sa, sb)
        mm[f"a{i}"], mm[f"b{i}"], mm[f"out{i}"], mm[f"s{i}"] = a, b, out, np.array([sa, sb], np.float32)
    np.savez_compressed(os.path.join(HERE, "quantized_matmul.npz"), **mm)
    print("golden fixtures written to", HERE)


def qat():
    r = O.ref_host()
    if r is None:
        raise SystemExit("oracle/_ref/libnova_ref_host.so missing: run `make -C oracle ref` first")
    rng = np.random.default_rng(20261202)
    edge = O.special_floats()
    out = {}
    for i, (scale, zp) in enumerate([(0.05, 0.0), (0.5, 2.0), (1e-8, 0.0), (3.0, -1.25), (0.0, 0.5)]):
        x = np.concatenate([edge, (rng.standard_normal(3000) * 8.0).astype(np.float32),
                            (np.arange(-300, 301, dtype=np.float32) * 0.5 * np.float32(max(scale, 1e-6)) + zp)])
        x = x.astype(np.float32)
        y = np.empty_like(x)
        r.ref_fake_quantize(x.ctypes.data, y.ctypes.data, x.size, scale, zp)
        out[f"x{i}"], out[f"y{i}"], out[f"p{i}"] = x, y, np.array([scale, zp], np.float32)
    np.savez_compressed(os.path.join(HERE, "qat_fake_quant.npz"), **out)
    print("qat_fake_quant.npz written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "qat":
        qat()
    else:
        main()
        qat()
