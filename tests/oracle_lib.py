"""ctypes binding of the CPU oracle (oracle/liboracle.so) and, when built,
of the reference's own code under oracle/_ref/.  Test infrastructure."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE = os.path.join(ROOT, "oracle", "liboracle.so")
REF_HOST = os.path.join(ROOT, "oracle", "_ref", "libnova_ref_host.so")
REF_GPU = os.path.join(ROOT, "oracle", "_ref", "libnova_ref_gpu.so")

_p, _sz, _f, _i = C.c_void_p, C.c_size_t, C.c_float, C.c_int

lib = C.CDLL(ORACLE)
for name, res, args in [
    ("orc_e4m3_compat_encode", C.c_uint8, [_f]), ("orc_e5m2_compat_encode", C.c_uint8, [_f]),
    ("orc_e4m3_ocp_encode", C.c_uint8, [_f]), ("orc_e5m2_ocp_encode", C.c_uint8, [_f]),
    ("orc_e4m3_compat_decode", _f, [C.c_uint8]), ("orc_e5m2_compat_decode", _f, [C.c_uint8]),
    ("orc_e4m3_ocp_decode", _f, [C.c_uint8]), ("orc_e5m2_ocp_decode", _f, [C.c_uint8]),
    ("orc_f32_to_bf16", C.c_uint16, [_f]), ("orc_bf16_to_f32", _f, [C.c_uint16]),
    ("orc_quantize_f32_to_fp8_compat", None, [_p, _p, _sz, _i]),
    ("orc_dequantize_fp8_compat", None, [_p, _p, _sz, _f, _i]),
    ("orc_quantize_scaled_fp8_compat", None, [_p, _p, _sz, _f]),
    ("orc_quantize_f32_to_int8", None, [_p, _p, _sz, _f, _f, _i]),
    ("orc_dequantize_int8_to_f32", None, [_p, _p, _sz, _f, _f, _i]),
    ("orc_quantize_int8_with_calibration", None, [_p, _p, _sz, _f, _f]),
    ("orc_quantize_int8_half_away", None, [_p, _p, _sz, _f]),
    ("orc_quantize_ocp", None, [_p, _p, _sz, _f, _i]),
    ("orc_dequantize_ocp", None, [_p, _p, _sz, _f, _i]),
    ("orc_compute_minmax", None, [_p, _sz, _p, _p]),
    ("orc_amax", _f, [_p, _sz]),
    ("orc_build_histogram", None, [_p, _p, _sz, _f, _f, _i]),
    ("orc_minmax_calibrate", None, [_p, _sz, _i, _p]),
    ("orc_histogram_threshold", _f, [_p, _i, _f, _f, _f]),
    ("orc_histogram_calibrate", None, [_p, _sz, _i, _f, _i, _p, _p]),
    ("orc_mse_calibrate", None, [_p, _sz, _i, _p]),
    ("orc_quantize_rows", None, [_p, _i, _p, _p, _sz, _sz, _i]),
    ("orc_quantize_cols", None, [_p, _p, _p, _sz, _sz, _i]),
    ("orc_fp8_gemm_reference", None, [_p, _p, _p, _i, _i, _i, _f, _f, _f, _i]),
    ("orc_gemm_fp8_acc", None, [_p, _p, _p, _i, _i, _i, _i, _i, _i]),
    ("orc_gemm_i8_acc", None, [_p, _p, _p, _i, _i, _i, _i]),
    ("orc_epilogue", None, [_p, _i, _p, _i, _i, _i, _f, _p, _p, _p]),
    ("orc_quantized_matmul", None, [_p, _p, _p, _i, _i, _i, _f, _f]),
    ("orc_quantized_tensor_from_float", _i, [_p, _sz, _f, _p, _p]),
    ("orc_fp8_gemm_reference_rows_mt", _i, [_p, _p, _p, _i, _i, _i, _f, _f, _f, _i, _i, _i]),
    ("orc_swiglu_epilogue", None, [_p, _p, _i, _i, _i, _f, _p, _p, _p]),
    ("orc_silu_mul", _f, [_f, _f]),
    ("orc_fake_quantize_int8", None, [_p, _p, _sz, _f, _f]),
    ("orc_fp8_activation", None, [_p, _p, _sz, _i, _i, _f]),
]:
    fn = getattr(lib, name)
    fn.restype = res
    fn.argtypes = args


def ptr(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data


def quantize_compat(x, fmt=0):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.size, np.uint8)
    lib.orc_quantize_f32_to_fp8_compat(ptr(x), ptr(q), x.size, fmt)
    return q.reshape(x.shape)


def dequantize_compat(q, scale, fmt=0):
    q = np.ascontiguousarray(q, np.uint8)
    y = np.empty(q.size, np.float32)
    lib.orc_dequantize_fp8_compat(ptr(q), ptr(y), q.size, scale, fmt)
    return y.reshape(q.shape)


def quantize_int8(x, scale, zp=0.0, sym=True):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.size, np.int8)
    lib.orc_quantize_f32_to_int8(ptr(x), ptr(q), x.size, scale, zp, int(sym))
    return q.reshape(x.shape)


def dequantize_int8(q, scale, zp=0.0, sym=True):
    q = np.ascontiguousarray(q, np.int8)
    y = np.empty(q.size, np.float32)
    lib.orc_dequantize_int8_to_f32(ptr(q), ptr(y), q.size, scale, zp, int(sym))
    return y.reshape(q.shape)


def quantize_ocp(x, scale, fmt):
    x = np.ascontiguousarray(x, np.float32)
    q = np.empty(x.size, np.uint8)
    lib.orc_quantize_ocp(ptr(x), ptr(q), x.size, scale, fmt)
    return q.reshape(x.shape)


def dequantize_ocp(q, scale, fmt):
    q = np.ascontiguousarray(q, np.uint8)
    y = np.empty(q.size, np.float32)
    lib.orc_dequantize_ocp(ptr(q), ptr(y), q.size, scale, fmt)
    return y.reshape(q.shape)


def minmax(x):
    x = np.ascontiguousarray(x, np.float32)
    lo, hi = C.c_float(), C.c_float()
    lib.orc_compute_minmax(ptr(x), x.size, C.byref(lo), C.byref(hi))
    return lo.value, hi.value


def histogram(x, lo, hi, bins):
    x = np.ascontiguousarray(x, np.float32)
    h = np.empty(bins, np.uint32)
    lib.orc_build_histogram(ptr(x), ptr(h), x.size, lo, hi, bins)
    return h


def minmax_calibrate(x, sym=True):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(5, np.float32)
    lib.orc_minmax_calibrate(ptr(x), x.size, int(sym), ptr(out))
    return out


def quantize_rows(x, fmt, bf16=False):
    x = np.ascontiguousarray(x)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.uint8)
    s = np.empty(rows, np.float32)
    lib.orc_quantize_rows(ptr(x), int(bf16), ptr(q), ptr(s), rows, cols, fmt)
    return q, s


def quantize_cols(x, fmt):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.uint8)
    s = np.empty(cols, np.float32)
    lib.orc_quantize_cols(ptr(x), ptr(q), ptr(s), rows, cols, fmt)
    return q, s


def f32_to_bf16_bits(x):
    x = np.ascontiguousarray(x, np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    r[nan] = ((x.view(np.uint32)[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def gemm_fp8_acc(a, b, fmt_a, fmt_b, b_kn):
    m, k = a.shape
    n = b.shape[1] if b_kn else b.shape[0]
    acc = np.empty((m, n), np.float32)
    lib.orc_gemm_fp8_acc(ptr(np.ascontiguousarray(a)), ptr(np.ascontiguousarray(b)), ptr(acc), m, k, n,
                         fmt_a, fmt_b, int(b_kn))
    return acc


def gemm_i8_acc(a, b, b_kn):
    m, k = a.shape
    n = b.shape[1] if b_kn else b.shape[0]
    acc = np.empty((m, n), np.int32)
    lib.orc_gemm_i8_acc(ptr(np.ascontiguousarray(a)), ptr(np.ascontiguousarray(b)), ptr(acc), m, k, n, int(b_kn))
    return acc


def epilogue(acc, out_bf16, alpha, row_scale=None, col_scale=None, bias=None):
    m, n = acc.shape
    acc = np.ascontiguousarray(acc)
    out = np.empty((m, n), np.uint16 if out_bf16 else np.float32)
    rs = np.ascontiguousarray(row_scale, np.float32) if row_scale is not None else None
    cs = np.ascontiguousarray(col_scale, np.float32) if col_scale is not None else None
    bs = np.ascontiguousarray(bias, np.float32) if bias is not None else None
    lib.orc_epilogue(ptr(acc), int(acc.dtype == np.int32), ptr(out), int(out_bf16), m, n, alpha,
                     ptr(rs) if rs is not None else None, ptr(cs) if cs is not None else None,
                     ptr(bs) if bs is not None else None)
    return out


def fp8_gemm_reference(a, b, sa, sb, so, fmt=0):
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), np.float32)
    lib.orc_fp8_gemm_reference(ptr(np.ascontiguousarray(a)), ptr(np.ascontiguousarray(b)), ptr(c), m, k, n,
                               sa, sb, so, fmt)
    return c


def ref_host():
    """The reference's own host code (None when oracle/_ref was not built)."""
    if not os.path.exists(REF_HOST):
        return None
    r = C.CDLL(REF_HOST)
    r.ref_e4m3_encode.restype = C.c_uint8
    r.ref_e4m3_encode.argtypes = [_f]
    r.ref_e5m2_encode.restype = C.c_uint8
    r.ref_e5m2_encode.argtypes = [_f]
    r.ref_e4m3_decode.restype = _f
    r.ref_e4m3_decode.argtypes = [C.c_uint8]
    r.ref_e5m2_decode.restype = _f
    r.ref_e5m2_decode.argtypes = [C.c_uint8]
    r.ref_e4m3_encode_array.argtypes = [_p, _p, _sz]
    r.ref_from_float_int8.restype = _i
    r.ref_from_float_int8.argtypes = [_p, _sz, _f, _p, _p]
    r.ref_quantized_matmul.argtypes = [_p, _p, _p, _i, _i, _i, _f, _f]
    r.ref_fake_quantize.argtypes = [_p, _p, _sz, _f, _f]
    r.ref_amp_load.restype = _i
    r.ref_amp_load.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(_i), C.POINTER(_f), C.POINTER(_f), C.POINTER(_i)]
    r.ref_amp_save_two.argtypes = [C.c_char_p]
    return r


def ref_gpu():
    """The reference's own GPU kernels built for sm_100a (None if absent)."""
    if not os.path.exists(REF_GPU):
        return None
    r = C.CDLL(REF_GPU)
    for name, args in [
        ("ref_gpu_quantize_f32_to_int8", [_p, _p, _sz, _f, _f, _i]),
        ("ref_gpu_dequantize_int8_to_f32", [_p, _p, _sz, _f, _f, _i]),
        ("ref_gpu_quantize_with_calibration", [_p, _p, _sz, _f, _f]),
        ("ref_gpu_quantize_fp8", [_p, _p, _sz, _i]),
        ("ref_gpu_dequantize_fp8", [_p, _p, _sz, _f, _i]),
        ("ref_gpu_compute_minmax", [_p, _sz, _p, _p]),
        ("ref_gpu_build_histogram", [_p, _p, _sz, _f, _f, _i]),
        ("ref_gpu_fp8_gemm", [_p, _p, _p, _i, _i, _i, _f, _f, _f]),
        ("ref_gpu_minmax_calibrate", [_p, _sz, _i, _p]),
        ("ref_gpu_mse_calibrate", [_p, _sz, _i, _p]),
    ]:
        fn = getattr(r, name)
        fn.restype = _i
        fn.argtypes = args
    return r


def special_floats():
    """Edge values of the codecs: zeros, infinities, NaN, max/min normals of
    every format, rounding ties and values around every threshold."""
    f = np.finfo(np.float32)
    base = [0.0, -0.0, np.inf, -np.inf, np.nan, f.max, -f.max, f.tiny, -f.tiny, 1e-45, -1e-45,
            240.0, 248.0, 256.0, 250.0, 15.9, 7.99, 0.0019, 0.001, 448.0, 464.0, 480.0, 500.0,
            57344.0, 61440.0, 65536.0, 1.0 / 64, 1.0 / 512, 1.0 / 1024, 2.0 ** -10, 2.0 ** -9, 2.0 ** -16,
            2.0 ** -17, 1.0625, 1.1875, 0.5, 1.5, 2.5, 126.5, 127.5, 128.5, -126.5, -127.5, 1000.0, -1000.0]
    grid = []
    for e in range(-20, 18):
        for m in range(0, 16):
            grid.append((1.0 + m / 16.0) * 2.0 ** e)
            grid.append((1.0 + (m + 0.5) / 16.0) * 2.0 ** e)
    v = np.array(base + grid, np.float32)
    return np.concatenate([v, -v])


def swiglu_epilogue(acc, out_bf16, alpha, row_scale=None, col_scale=None, bias=None):
    m, n = acc.shape
    acc = np.ascontiguousarray(acc, np.float32)
    out = np.empty((m, n // 2), np.uint16 if out_bf16 else np.float32)
    rs = np.ascontiguousarray(row_scale, np.float32) if row_scale is not None else None
    cs = np.ascontiguousarray(col_scale, np.float32) if col_scale is not None else None
    bs = np.ascontiguousarray(bias, np.float32) if bias is not None else None
    lib.orc_swiglu_epilogue(ptr(acc), ptr(out), int(out_bf16), m, n, alpha, ptr(rs) if rs is not None else None,
                            ptr(cs) if cs is not None else None, ptr(bs) if bs is not None else None)
    return out


def tp_mlp_partial(x_bits, wg, wu, wd, rank, tp):
    """One rank's row-parallel partial of the W8A8 FP8 SwiGLU MLP, restated on
    the oracle: per-token E4M3 quantize of x (bf16 bits, T x H); gate/up
    column shards (tensor_parallel_layers.cpp:111-136) with per-column E4M3
    scales, packed in alternating 128-column blocks; the GEMM accumulators
    and the SwiGLU epilogue (activations.cu:80-92) to bf16 h; per-token
    quantize of h; the down row shard (:344-368) with per-column scales; bf16
    partial.  Returns (h bits, partial bits)."""
    T, H = x_bits.shape
    I = wg.shape[1]
    il = I // tp
    xq, sx = quantize_rows(x_bits, 0, bf16=True)
    g = wg[:, rank * il:(rank + 1) * il]
    u = wu[:, rank * il:(rank + 1) * il]
    j = np.arange(il // 128)[:, None]
    c = np.arange(128)[None, :]
    order = np.concatenate([j * 128 + c, il + j * 128 + c], axis=1).reshape(-1)
    gu = np.ascontiguousarray(np.concatenate([g, u], axis=1)[:, order])
    gq, gs = quantize_cols(gu, 0)
    h = swiglu_epilogue(gemm_fp8_acc(xq, gq, 0, 0, True), True, 1.0, sx, gs)
    return h, tp_down_partial(h, wd, rank, tp)


def tp_down_partial(h_bits, wd, rank, tp):
    """The row-parallel half of tp_mlp_partial: per-token quantize of this
    rank's h (bf16 bits, T x I/tp), down row shard with per-column scales,
    bf16 partial (T x H)."""
    il = wd.shape[0] // tp
    hq, sh = quantize_rows(np.ascontiguousarray(h_bits), 0, bf16=True)
    dq, ds = quantize_cols(np.ascontiguousarray(wd[rank * il:(rank + 1) * il]), 0)
    return epilogue(gemm_fp8_acc(hq, dq, 0, 0, True), True, 1.0, sh, ds)


def fake_quantize(x, scale, zero_point):
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib.orc_fake_quantize_int8(ptr(x), ptr(y), x.size, scale, zero_point)
    return y


def fp8_activation(codes, fmt, op, alpha=0.01):
    codes = np.ascontiguousarray(codes, np.uint8)
    out = np.empty_like(codes)
    lib.orc_fp8_activation(ptr(codes), ptr(out), codes.size, fmt, op, alpha)
    return out
