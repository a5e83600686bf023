"""Build-level drop-in check: the reference's own bench (bench/*.cu,
unmodified, canonical variants) compiled against include/decode_gemm.cuh and
include/weight_prepack.cuh instead of its SM90 kernel headers and linked to
the sm_100a library (oracle/Makefile, target refbench, built by build() when
the reference checkout is present).  Its --list registers every canonical
variant without touching a GPU; its main() stops on any device but SM90
(bench/bench_decode.cu:1982), so that is as far as it runs on B200."""

import os
import subprocess

import pytest

BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                   "bench_decode_b200")


@pytest.mark.skipif(not os.path.exists(BIN), reason="reference bench not built (no reference checkout at build time)")
def test_reference_bench_links_and_registers_its_variants():
    proc = subprocess.run([BIN, "--list"], capture_output=True, text=True, timeout=120)
    assert proc.returncode == 0, proc.stderr
    out = proc.stdout
    assert "registered variants: 226 (canonical=226 tune=0)" in out
    for mt, n in ((8, 49), (16, 47), (32, 47), (64, 47), (128, 36)):
        assert f"M_TILE={mt:>3} canonical={n:<3d}" in out
    assert "S0 baseline     M_TILE=8;BM=64;WG=4;REG=112" in out
