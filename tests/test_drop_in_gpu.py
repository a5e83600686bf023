"""The C++ interface (include/decode_gemm.cuh, include/weight_prepack.cuh) on
the GPU: the reference-shaped calls launch<Cfg>, launch_with_maps<Cfg> and a
caller's own cudaLaunchKernelEx of fp8_decode_gemm<Cfg> (the reference
bench's direct launch) give bit-identical outputs that match the oracle, for
KernelConfigs of every batch class (M_TILE 8..128), raw and packed weights,
split-K 2 and 4, BM 56 to 256, ragged N, and any M <= M_TILE."""

import json
import os
import subprocess

import numpy as np
import pytest

from helpers import check_against_oracle, smoke_case

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "decode_opt_b200",
                   "dg_drop_in_check")
CFG_M_TILE = {"s0_mt8": 8, "s5_mt8_bm56_sk2": 8, "mt32_sk4": 32, "mt64_bm256": 64, "mt128_bm128_epi": 128}


@pytest.mark.parametrize("m", [1, 5, 8, 20, 32, 40, 64, 100, 128])
def test_cpp_interface_three_launch_paths(m, tmp_path):
    assert os.path.exists(BIN), "dg_drop_in_check missing: run python -m decode_opt_b200.build"
    n, k = 1000, 2048
    w, ws, a, as_, ref = smoke_case(n, k, 31, m)
    (tmp_path / "meta.txt").write_text(f"{m} {n} {k}\n")
    np.ascontiguousarray(w).tofile(tmp_path / "w.bin")
    np.ascontiguousarray(ws, dtype=np.float32).tofile(tmp_path / "ws.bin")
    np.ascontiguousarray(a).tofile(tmp_path / "a.bin")
    np.ascontiguousarray(as_, dtype=np.float32).tofile(tmp_path / "as.bin")
    proc = subprocess.run([BIN, str(tmp_path)], capture_output=True, text=True, timeout=300)
    assert proc.returncode == 0, proc.stderr
    lines = [json.loads(ln) for ln in proc.stdout.splitlines() if ln.startswith("{")]
    assert {r["cfg"] for r in lines} == {c for c, mt in CFG_M_TILE.items() if m <= mt}
    for r in lines:
        assert r["rc"] == [0, 0, 0], r
        assert r["launch_eq_with_maps"] and r["launch_eq_direct"] and r["sem_clean"], r
        bits = np.fromfile(tmp_path / f"out_{r['cfg']}.bin", dtype=np.uint16).reshape(m, n)
        got = (bits.astype(np.uint32) << 16).view(np.float32)
        ok, rl2, worst = check_against_oracle(got, ref)
        assert ok, (r["cfg"], rl2, worst)
