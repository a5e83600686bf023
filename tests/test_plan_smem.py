"""The planner's shared-memory size of every accepted plan equals the kernel's
carve-up (tests/cpp/dg_plan_smem_check.cu, host-only, built with nvcc; no
GPU): a plan that under-counts would let the kernel address shared memory
past its launch's allocation."""

import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else shutil.which("nvcc")


@pytest.mark.skipif(_nvcc() is None, reason="needs nvcc")
def test_plan_smem_matches_kernel_carve_up(tmp_path):
    exe = str(tmp_path / "dg_plan_smem_check")
    cmd = [_nvcc(), "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a",
           "-I", os.path.join(ROOT, "decode_opt_b200", "csrc"), "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "cpp", "dg_plan_smem_check.cu"), "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert " 0 failure(s)" in run.stdout
