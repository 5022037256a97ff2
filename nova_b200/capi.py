"""ctypes binding of the C ABI (include/nova_q.h) for tests and benchmarks.

Every function takes raw device pointers (ints, e.g. torch.Tensor.data_ptr())
and a cudaStream_t handle (int).  Status codes are turned into NqError.
"""
from __future__ import annotations

import ctypes as C
import os

from . import LIB_PATH

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python -m nova_b200.build` "
                      "(the CUDA extension is required; there is no CPU fallback)")

lib = C.CDLL(LIB_PATH)

E4M3, E5M2, INT8 = 0, 1, 2
F32, BF16, S32, S8 = 0, 1, 2, 3
B_KN, B_NK = 0, 1

_p, _sz, _f, _i, _u32p = C.c_void_p, C.c_size_t, C.c_float, C.c_int, C.POINTER(C.c_uint32)


class NqError(RuntimeError):
    def __init__(self, status: int, where: str):
        self.status = status
        msg = lib.nq_last_error().decode(errors="replace")
        name = lib.nq_status_string(status).decode()
        super().__init__(f"{where}: {name}: {msg}")


class GemmDesc(C.Structure):
    _fields_ = [("m", C.c_int), ("n", C.c_int), ("k", C.c_int), ("a_format", C.c_int), ("b_format", C.c_int),
                ("b_layout", C.c_int), ("out_dtype", C.c_int), ("alpha", C.c_float), ("row_scale", C.c_void_p),
                ("col_scale", C.c_void_p), ("bias", C.c_void_p), ("epilogue", C.c_int)]


MAX_TP = 8


class AllreduceDesc(C.Structure):
    _fields_ = [("tp", C.c_int), ("rank", C.c_int), ("epoch", C.c_uint32),
                ("signal", C.c_int), ("signal_flags", C.c_void_p * MAX_TP),
                ("m", C.c_int), ("n", C.c_int), ("flags", C.c_void_p),
                ("mc_partial", C.c_void_p), ("mc_out", C.c_void_p), ("mc_done", C.c_void_p),
                ("peer_partial", C.c_void_p * MAX_TP), ("peer_out", C.c_void_p * MAX_TP),
                ("peer_done", C.c_void_p * MAX_TP),
                ("done", C.c_void_p), ("done_target", C.c_uint32)]


_SIGS = {
    "nq_quantize_f32_to_fp8e4m3": [_p, _p, _sz, _p],
    "nq_quantize_f32_to_fp8e5m2": [_p, _p, _sz, _p],
    "nq_dequantize_fp8e4m3_to_f32": [_p, _p, _sz, _f, _p],
    "nq_dequantize_fp8e5m2_to_f32": [_p, _p, _sz, _f, _p],
    "nq_quantize_batched_f32_to_fp8e4m3": [_p, _p, _i, _p, _p, _p],
    "nq_dequantize_batched_fp8e4m3_to_f32": [_p, _p, _i, _p, _p, _p],
    "nq_quantize_f32_to_int8": [_p, _p, _sz, _f, _f, _i, _p],
    "nq_dequantize_int8_to_f32": [_p, _p, _sz, _f, _f, _i, _p],
    "nq_quantize_f32_to_int8_with_calibration": [_p, _p, _sz, _f, _f, _p],
    "nq_quantize_f32_to_int8_round_away": [_p, _p, _sz, _f, _p],
    "nq_fake_quantize_int8": [_p, _p, _sz, _f, _f, _p],
    "nq_fp8_activation": [_p, _p, _sz, _i, _i, _f, _p],
    "nq_compute_minmax": [_p, _sz, _p, _p, _p],
    "nq_build_histogram": [_p, _p, _sz, _f, _f, _i, _p],
    "nq_minmax_async": [_p, _sz, _p, _p],
    "nq_amax_scale_async": [_p, _i, _sz, _i, _p, _p],
    "nq_minmax_rows": [_p, _i, _i, _p, _p, _p],
    "nq_quantize_scaled": [_p, _i, _p, _sz, _i, _p, _p],
    "nq_dequantize_scaled": [_p, _p, _sz, _i, _p, _p],
    "nq_calibrate_quantize": [_p, _i, _p, _sz, _i, _p, _p],
    "nq_quantize_rows": [_p, _i, _p, _p, _i, _i, _i, _p],
    "nq_quantize_cols": [_p, _p, _p, _i, _i, _i, _p],
    "nq_quantize_cols_noalloc": [_p, _p, _p, _i, _i, _i, _p],
    "nq_gemm": [C.POINTER(GemmDesc), _p, _p, _p, _p],
    "nq_gemm_simt": [C.POINTER(GemmDesc), _p, _p, _p, _p],
    "nq_gemm_quant_a": [C.POINTER(GemmDesc), _p, _p, _p, _p, _p, _p],
    "nq_convert_bf16_to_f32": [_p, _p, _sz, _p],
    "nq_gemm_allreduce": [C.POINTER(GemmDesc), C.POINTER(AllreduceDesc), _p, _p, _p, _p],
    "nq_allreduce_finish": [C.POINTER(AllreduceDesc), _p],
    "nq_fp8_gemm_forward": [_p, _p, _p, _i, _i, _i, _f, _f, _f, _p],
    "nq_fp8e5m2_gemm_forward": [_p, _p, _p, _i, _i, _i, _f, _f, _f, _p],
    "nq_device_error_flags": [_u32p, _i],
    "nq_set_peer_wait_limit": [C.c_uint64],
    "nq_mixed_precision_matmul": [_p, _p, _p, _p, _i, _i, _i, _p],
    "nq_fp8_gemm_backward": [_p, _i, _p, _p, _p, _p, _i, _i, _i, _f, _f, _f, _p],
}

lib.nq_status_string.restype = C.c_char_p
lib.nq_status_string.argtypes = [C.c_int]
lib.nq_last_error.restype = C.c_char_p
lib.nq_last_error.argtypes = []
lib.nq_version.restype = C.c_int
lib.nq_fp8_gemm_workspace_size.restype = C.c_size_t
lib.nq_fp8_gemm_workspace_size.argtypes = [_i, _i, _i]
lib.nq_gemm_allreduce_counters.restype = C.c_int
lib.nq_gemm_allreduce_counters.argtypes = [_i, _i]
gemm_allreduce_counters = lib.nq_gemm_allreduce_counters
lib.nq_peer_wait_limit.restype = C.c_uint64
lib.nq_peer_wait_limit.argtypes = []
peer_wait_limit = lib.nq_peer_wait_limit
lib.nq_allreduce_done_per_job.restype = C.c_int
lib.nq_allreduce_done_per_job.argtypes = [_i, _i, _i]
allreduce_done_per_job = lib.nq_allreduce_done_per_job


def _wrap(name, argtypes):
    fn = getattr(lib, name)
    fn.argtypes = argtypes
    fn.restype = C.c_int

    def call(*args):
        st = fn(*args)
        if st != 0:
            raise NqError(st, name)
        return st

    call.__name__ = name
    call.raw = fn
    return call


for _n, _a in _SIGS.items():
    _short = _n[3:] if _n != "nq_device_error_flags" else "device_error_flags_"
    globals()[_short] = _wrap(_n, _a)   # nq_gemm -> capi.gemm


def exported_symbols():
    return sorted(list(_SIGS) + ["nq_status_string", "nq_last_error", "nq_version", "nq_fp8_gemm_workspace_size",
                                 "nq_gemm_allreduce_counters", "nq_allreduce_done_per_job", "nq_peer_wait_limit"])


EPI_NONE, EPI_SWIGLU = 0, 1
ACT_RELU, ACT_GELU, ACT_SIGMOID, ACT_LEAKY_RELU = 0, 1, 2, 3


def make_desc(m, n, k, a_format=E4M3, b_format=E4M3, b_layout=B_KN, out_dtype=BF16, alpha=1.0,
              row_scale=0, col_scale=0, bias=0, epilogue=EPI_NONE) -> GemmDesc:
    return GemmDesc(m, n, k, a_format, b_format, b_layout, out_dtype, alpha, row_scale or None,
                    col_scale or None, bias or None, epilogue)


def device_error_flags(clear: bool = True) -> int:
    v = C.c_uint32(0)
    device_error_flags_(C.byref(v), int(clear))  # noqa: F821 (defined by the loop above)
    return v.value
