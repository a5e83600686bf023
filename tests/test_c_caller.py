"""The C ABI from plain C: tests/c/dg_c_caller.c compiled with gcc as C99
(-pedantic -Wall -Wextra -Werror) against include/decode_gemm_b200.h, linked to
the in-tree library and run (no GPU needed for what it checks)."""

import os
import shutil
import subprocess

import pytest

from decode_opt_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_plain_c_caller(tmp_path):
    lib_dir = os.path.dirname(_lib.LIB_PATH)
    assert os.path.exists(_lib.LIB_PATH), "build the library first (__graft_entry__.build())"
    exe = str(tmp_path / "dg_c_caller")
    cmd = ["gcc", "-std=c99", "-pedantic", "-Wall", "-Wextra", "-Werror",
           "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c", "dg_c_caller.c"), "-o", exe,
           "-L", lib_dir, "-ldecode_gemm_b200", f"-Wl,-rpath,{lib_dir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "0 failure(s)" in run.stdout
