"""bench.py's output contract, on the CPU through its reference arm
(`--impl reference`: the reference's host GEMM on all host cores): stdout
carries exactly one JSON line with the contract's keys, one process and under
torch.distributed.run with two ranks (rank 0 alone measures and prints; the
other rank exits 0 without work)."""

import json
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# torchrun's own parser would take --n / --m / --k for prefixes of its options,
# so the runs keep the default C2 shape and bound the sample by time instead.
SMALL = ["--impl", "reference", "--steps", "1", "--warmup", "1", "--ref-seconds", "2"]


def _one_json_line(stdout: str) -> dict:
    lines = [ln for ln in stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, f"stdout must carry exactly one line, got {len(lines)}: {lines[:3]}"
    return json.loads(lines[0])


def _check_reference_line(d: dict, n_gpus: int):
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference"
    assert d["n_gpus"] == n_gpus and d["steps"] == 1 and d["warmup"] == 1
    assert d["unit"] == "GB/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["N"] == 7168 and d["config"]["K"] == 16384 and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == d["value"] and cb["unit"] == d["unit"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_reference_arm_prints_one_contract_line():
    r = subprocess.run([sys.executable, "bench.py", *SMALL], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    _check_reference_line(_one_json_line(r.stdout), 1)


def test_reference_arm_under_torchrun_rank0_prints_once():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(port), "bench.py", "--gpus", "2", *SMALL]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    _check_reference_line(_one_json_line(r.stdout), 2)
