"""GPU test of the measurement probes (decode_opt_b200/probe.py, the rebuild
of the reference's tools/peak_bw_probe.cu): a reduced sweep must report a
plausible achievable HBM read figure -- at least half and at most the B200's
8 TB/s spec -- and an L2 self-test far above it (the harness tells L2 hits
from DRAM reads, reference tools/peak_bw_probe.cu:190-211); the JSON
document carries the reference's fields; the tcgen05.mma probe reports a
positive cost for every shape and issuer count."""

import json

import pytest

pytestmark = pytest.mark.gpu


def test_quick_probe_sweep(tmp_path):
    from decode_opt_b200 import probe
    out = tmp_path / "peak_bw.json"
    probe.main(["--quick", "--json", str(out)])
    doc = json.loads(out.read_text())
    best = doc["measured_best_gbps"]
    assert 4000.0 <= best <= probe.SPEC_GBPS, best
    assert doc["l2_selftest_gbps"] >= 1.4 * best, (doc["l2_selftest_gbps"], best)
    for key in ("spec_gbps", "measured_best_gbps", "method", "best", "configs", "naive", "l2_selftest"):
        assert key in doc
    feasible = [c for c in doc["configs"] if c["feasible"]]
    assert feasible and all(c["gbps"] > 0 and len(c["round_us"]) == 7 for c in feasible)
    # every HBM figure is a cold read: none above the spec
    assert all(c["gbps"] <= probe.SPEC_GBPS for c in feasible + doc["naive"])
    for r in doc["mma"]:
        assert r["issue_cycles"] > 0 and r["complete_cycles"] >= r["issue_cycles"], r
    # No shape beats the FP8 dense tensor peak: one 128 x 256 x 32 MMA per
    # 128 cycles, 8192 MACs per cycle per SM.
    assert max(r["mac_per_cycle"] for r in doc["mma"]) <= 8192 * 1.05
