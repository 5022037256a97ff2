"""The C ABI library loads and exports every entry point include/*.h declares
(CPU only: no kernel is launched)."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for d, _, files in os.walk(inc):
        for f in files:
            if f.endswith(".h"):
                txt = open(os.path.join(d, f)).read()
                txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
                names |= set(re.findall(r"\b(nq_[a-z0-9_]+)\s*\(", txt))
    return names


def test_library_exports_every_declared_symbol():
    import nova_b200.capi as capi
    out = subprocess.run(["nm", "-D", "--defined-only", capi.LIB_PATH if hasattr(capi, "LIB_PATH") else
                          os.path.join(ROOT, "nova_b200", "libnova_q.so")], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (nq_\w+)", out))
    declared = declared_symbols()
    assert declared, "no declarations found"
    assert declared <= exported, f"declared but not exported: {sorted(declared - exported)}"
    assert exported <= declared, f"exported but not declared: {sorted(exported - declared)}"
    for name in declared:
        assert hasattr(capi.lib, name)


def test_status_strings_and_errors_without_gpu():
    import ctypes as C
    import nova_b200.capi as capi
    assert capi.lib.nq_status_string(0) == b"NQ_SUCCESS"
    assert capi.lib.nq_status_string(6) == b"NQ_ERROR_DEVICE_TIMEOUT"
    assert capi.lib.nq_version() >= 100
    # argument errors are reported before any device work
    st = capi.quantize_f32_to_int8.raw(None, None, 10, 1.0, 0.0, 1, None)
    assert st == 1 and b"null" in capi.lib.nq_last_error()
    assert capi.quantize_f32_to_int8.raw(None, None, 0, 1.0, 0.0, 1, None) == 0
    d = capi.make_desc(16, 16, 16, capi.E4M3, capi.INT8)
    assert capi.gemm.raw(C.byref(d), 16, 16, 16, None) == 1
    assert capi.lib.nq_fp8_gemm_workspace_size(128, 256, 128) == 128 * 256 + 256 * 128 + 128 * 128 * 4


def test_gemm_allreduce_argument_checks_without_gpu():
    """nq_gemm_allreduce / nq_allreduce_finish validate their descriptors
    before touching a device."""
    import ctypes as C
    import nova_b200.capi as capi
    assert capi.lib.nq_gemm_allreduce_counters(16384, 8192) == 64 * 32
    assert capi.lib.nq_gemm_allreduce_counters(300, 512) == 2 * 2
    assert capi.lib.nq_gemm_allreduce_counters(0, 512) == 0
    assert capi.lib.nq_allreduce_done_per_job(300, 512, 0) == 4 * 5
    assert capi.lib.nq_allreduce_done_per_job(300, 512, 1) == 4 * 4
    d = capi.make_desc(256, 512, 256)
    ar = capi.AllreduceDesc()
    ar.tp, ar.rank, ar.epoch = 2, 0, 1
    run = lambda: capi.gemm_allreduce.raw(C.byref(d), C.byref(ar), 16, 16, 16, None)
    assert capi.gemm_allreduce.raw(None, C.byref(ar), 16, 16, 16, None) == 1     # null descriptor
    ar.tp = 9
    assert run() == 1                                                              # tp > NQ_MAX_TP
    ar.tp, ar.signal = 2, 1
    assert run() == 1                                                              # signal without counters
    ar.signal_flags[0], ar.signal_flags[1] = 64, 128
    d.n = 384
    assert run() == 2                                                              # signalling needs n % 256 == 0
    d.n, d.out_dtype = 512, capi.F32
    assert run() == 2                                                              # bf16 output only
    d.out_dtype = capi.BF16
    ar.m, ar.n = 256, 512
    assert run() == 1                                                              # job without counters
    ar.flags = 256
    assert run() == 1                                                              # job without peer pointers
    assert capi.allreduce_finish.raw(C.byref(ar), None) == 1                       # finish cannot signal
    ar.signal, ar.m, ar.done_target = 0, 0, 5
    assert capi.allreduce_finish.raw(C.byref(ar), None) == 0                       # no job, no `done`: nothing to do
    ar.rank = 2
    assert capi.allreduce_finish.raw(C.byref(ar), None) == 1                       # rank >= tp


def test_fp8_backward_argument_checks_without_gpu():
    import nova_b200.capi as capi
    assert capi.fp8_gemm_backward.raw(16, 2, 16, 16, 16, 16, 4, 4, 4, 1.0, 1.0, 1.0, None) == 1   # INT8 grads
    assert capi.fp8_gemm_backward.raw(16, 0, 16, 16, 16, 16, -1, 4, 4, 1.0, 1.0, 1.0, None) == 1  # negative size
    assert capi.fp8_gemm_backward.raw(None, 0, 16, 16, 16, 16, 4, 4, 4, 1.0, 1.0, 1.0, None) == 1  # null grad
    assert capi.fp8_gemm_backward.raw(16, 0, 16, None, 16, None, 4, 4, 4, 1.0, 1.0, 1.0, None) == 1  # grad_a needs B
    assert capi.fp8_gemm_backward.raw(16, 0, 16, 16, 16, 16, 0, 4, 4, 1.0, 1.0, 1.0, None) == 0   # empty


def test_no_device_is_an_error_not_a_crash():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import nova_b200.capi as capi
    st = capi.quantize_f32_to_int8.raw(16, 32, 10, 1.0, 0.0, 1, None)
    assert st in (3, 5)


def test_cpp_headers_compile():
    """The drop-in C++ headers compile on their own (syntax check)."""
    inc = os.path.join(ROOT, "include")
    hdrs = []
    for d, _, files in os.walk(os.path.join(inc, "cuda")):
        hdrs += [os.path.join(d, f) for f in files if f.endswith(".hpp")]
    if not hdrs:
        pytest.skip("no C++ headers")
    # qat.hpp and quantize_ops.hpp both declare nova::quantize::Precision with
    # different enumerators, as in the reference: one of them per translation unit
    for skip in ("qat.hpp", "quantize_ops.hpp"):
        tu = [h for h in sorted(hdrs) if os.path.basename(h) != skip]
        src = "".join(f'#include "{h}"\n' for h in tu) + "int main(){return 0;}\n"
        r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", inc, "-I", "/usr/local/cuda/include", "-x",
                            "c++", "-"], input=src, capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
