"""Build recipe for the in-tree sm_100a libraries.

``python -m decode_opt_b200.build`` compiles ``csrc/dg_capi.cu`` into
``decode_opt_b200/libdecode_gemm_b200.so`` for ``sm_100a`` only.  The library
links the CUDA runtime statically and resolves ``cuTensorMapEncodeTiled``
through the runtime's driver entry-point query, so it loads on hosts without a
GPU (the CPU test suite checks its exported symbols there).

It then compiles ``tests/cpp/dg_drop_in_check.cu`` against the C++ headers
(``include/decode_gemm.cuh``, ``include/weight_prepack.cuh``) and the
library into ``decode_opt_b200/dg_drop_in_check``, the program the GPU tests
run to check the C++ interface, and ``csrc/dg_cublaslt_fp8.cu`` into
``decode_opt_b200/dg_cublaslt_fp8``, the cuBLASLt FP8 baseline bench.py runs
in its own process (linked to the CUDA toolkit's cuBLASLt, which declares the
128-block scale modes; torch's bundled cuBLAS is never loaded beside it).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIB_NAME = "libdecode_gemm_b200.so"
LIB_PATH = os.path.join(HERE, LIB_NAME)
DROP_IN_SRC = os.path.join(ROOT, "tests", "cpp", "dg_drop_in_check.cu")
DROP_IN_BIN = os.path.join(HERE, "dg_drop_in_check")
CUBLASLT_SRC = os.path.join(CSRC, "dg_cublaslt_fp8.cu")
CUBLASLT_BIN = os.path.join(HERE, "dg_cublaslt_fp8")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
SOURCES = ("dg_capi.cu", "dg_probe.cu", "dg_quant.cu")


def nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = os.path.join(cuda_home, "bin", "nvcc")
    return cand if os.path.exists(cand) else (shutil.which("nvcc") or "nvcc")


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))] + [
        os.path.join(INCLUDE, f) for f in sorted(os.listdir(INCLUDE))]


def needs_build(target: str = LIB_PATH, extra=()) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in list(_sources()) + list(extra))


def build(verbose: bool = False, ptxas_verbose: bool = False, force: bool = False) -> str:
    lib = build_library(verbose, ptxas_verbose, force)
    build_drop_in_check(verbose, force)
    build_cublaslt_bench(verbose, force)
    return lib


def cuda_lib_dir() -> str:
    return os.path.join(os.path.dirname(os.path.dirname(os.path.realpath(nvcc()))), "lib64")


def build_cublaslt_bench(verbose: bool = False, force: bool = False) -> str:
    """The cuBLASLt FP8 baseline program (block-scaled and per-tensor)."""
    if not force and os.path.exists(CUBLASLT_BIN) and os.path.getmtime(CUBLASLT_BIN) > os.path.getmtime(CUBLASLT_SRC):
        return CUBLASLT_BIN
    libdir = cuda_lib_dir()
    cmd = [nvcc(), "-std=c++17", "-O3", *ARCH_FLAGS, CUBLASLT_SRC, "-o", CUBLASLT_BIN + ".tmp", "-L", libdir,
           "-lcublasLt", "-Xlinker", f"-rpath,{libdir}"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(CUBLASLT_BIN + ".tmp", CUBLASLT_BIN)
    return CUBLASLT_BIN


def build_drop_in_check(verbose: bool = False, force: bool = False) -> str:
    """The C++-interface check program, linked to the in-tree library (found
    next to it at run time)."""
    if not force and not needs_build(DROP_IN_BIN, (DROP_IN_SRC, LIB_PATH)):
        return DROP_IN_BIN
    cmd = [nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS, "-I", INCLUDE, "-I", CSRC, DROP_IN_SRC,
           "-o", DROP_IN_BIN + ".tmp", "-L", HERE, "-ldecode_gemm_b200", "-Xlinker", "-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(DROP_IN_BIN + ".tmp", DROP_IN_BIN)
    return DROP_IN_BIN


def build_library(verbose: bool = False, ptxas_verbose: bool = False, force: bool = False) -> str:
    if not force and not needs_build():
        return LIB_PATH
    cmd = [nvcc(), "-std=c++17", "-O3", "-lineinfo", *ARCH_FLAGS,
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "static",
           "-I", CSRC, "-I", INCLUDE,
           *[os.path.join(CSRC, f) for f in SOURCES], "-o", LIB_PATH + ".tmp"]
    if ptxas_verbose:
        cmd[1:1] = ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(LIB_PATH + ".tmp", LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv, force="-f" in sys.argv)
