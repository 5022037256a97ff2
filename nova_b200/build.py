"""Build recipe of libnova_q.so (sm_100a) and its test-side companions.

    python -m nova_b200.build          # library + oracle (+ reference pins)

The library is compiled in-tree so that the .so ships with the repository
snapshot; objects go to nova_b200/_build/.  Only the nq_* C ABI is exported
(linker version script).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libnova_q.so")
SOURCES = ["runtime.cu", "elementwise.cu", "reduce.cu", "gemm.cu"]
HEADERS = ["nq_internal.h", "ptx.cuh", "codec.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2"] + ARCH


def reference_dir():
    """The pplmx/nova source tree used only to build the test-side pins under
    oracle/_ref/: $NOVA_REFERENCE_DIR, else a checkout named `reference` beside
    this repository; None when neither exists (the pins are then skipped and
    any prebuilt oracle/_ref/ files are used as they are)."""
    cand = os.environ.get("NOVA_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")
    return cand if os.path.isdir(os.path.join(cand, "include", "cuda", "quantize")) else None


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libnova_q")
    return cand


def _newer(src_files, target) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(f) > t for f in src_files)


def _run(cmd, cwd=None):
    r = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r


def build_library(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = _nvcc()
    deps = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(ROOT, "include", "nova_q.h")]
    jobs = []
    for s in SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s.replace(".cu", ".o"))
        if _newer([src] + deps, obj):
            jobs.append([nvcc] + NVCC_FLAGS + ["-c", src, "-o", obj])
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        for r in ex.map(_run, jobs):
            if verbose and r.stderr:
                print(r.stderr, file=sys.stderr)
    objs = [os.path.join(BUILD, s.replace(".cu", ".o")) for s in SOURCES]
    if _newer(objs, LIB):
        vs = os.path.join(BUILD, "exports.map")
        with open(vs, "w") as f:
            f.write("{ global: nq_*; local: *; };\n")
        _run([nvcc, "-shared"] + ARCH + ["-o", LIB] + objs + ["-Xlinker", f"--version-script={vs}"])
    return LIB


def build_oracle() -> None:
    """CPU oracle (test infrastructure) and, where the pplmx/nova sources are
    present, the reference's own code under oracle/_ref/ (checker only)."""
    _run(["make", "-s", "-C", os.path.join(ROOT, "oracle")])
    ref = reference_dir()
    if ref:
        _run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref", f"REF={ref}"])


def build_cpp_tests() -> None:
    """C++ programs that exercise the drop-in headers over libnova_q.so."""
    src_dir = os.path.join(ROOT, "tests", "cpp")
    out_dir = os.path.join(src_dir, "bin")
    os.makedirs(out_dir, exist_ok=True)
    for name in sorted(os.listdir(src_dir)):
        if not name.endswith(".cpp"):
            continue
        src = os.path.join(src_dir, name)
        exe = os.path.join(out_dir, name[:-4])
        hdrs = []
        for d, _, fs in os.walk(os.path.join(ROOT, "include")):
            hdrs += [os.path.join(d, f) for f in fs]
        if _newer([src, LIB] + hdrs, exe):
            # the TP layers' context holds NCCL communicators
            nccl = ["-lnccl", "-pthread"] if "nccl" in open(src).read() else []
            _run(["g++", "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                  src, "-o", exe, "-L", HERE, "-lnova_q", f"-Wl,-rpath,{HERE}", "-L", "/usr/local/cuda/lib64",
                  "-lcudart", f"-Wl,-rpath,/usr/local/cuda/lib64"] + nccl)


def build_all(verbose: bool = False) -> None:
    build_library(verbose)
    build_oracle()
    build_cpp_tests()


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print(LIB)
