"""The bench_decode sweep on the GPU: every canonical row, split-K factor row
and PDL-placement row of a small model passes the fp32 check, the files have
the reference's layout, and --resume re-measures nothing."""

import json
import math
import os

import pytest

from decode_opt_b200 import bench_decode as bd

pytestmark = pytest.mark.gpu


def _rows(path):
    with open(path) as f:
        lines = f.read().splitlines()
    return lines[0], [bd.split_csv_line(ln) for ln in lines[1:] if ln.strip()]


def test_sweep_rows_pass_and_resume(tmp_path):
    out = str(tmp_path)
    args = ["--models", "qwen36", "--ms", "1,8,128", "--steps", "0,3,5,6,7", "--reps", "2", "--iso-samples", "3",
            "--b2b-batch", "6", "--out", out, "--splitk-factor-sweep", "--pdl-placement", "--check-launcher",
            "--weight-cache-gb", "3"]
    assert bd.main(args) == 0
    csv = bd.newest_csv(out, "bench_")
    header, rows = _rows(csv)
    assert header == bd.CSV_HEADER
    assert len(rows) == 3 * 5 * 3
    col = {h: i for i, h in enumerate(header.split(","))}
    for r in rows:
        assert r[col["pass"]] == "1", r
        assert float(r[col["rel_l2"]]) <= bd.REL_L2_THRESHOLD
        lat = float(r[col["latency_us_p50"]])
        assert 0.5 < lat < 5000.0
        bw = float(r[col["bandwidth_gbps"]])
        assert bw == pytest.approx(bd.modeled_bytes(2048, 4096, int(r[col["M"]])) / (lat * 1e-6) / 1e9, rel=1e-3)
    assert {(r[col["step"]], r[col["step_name"]]) for r in rows} == {("0", "baseline"), ("3", "prepack"),
                                                                     ("5", "splitk"), ("6", "b200"),
                                                                     ("7", "b200_indep")}
    dh, drows = _rows(bd.detail_path_of(csv))
    assert dh == bd.DETAIL_HEADER and len(drows) == len(rows)
    dcol = {h: i for i, h in enumerate(dh.split(","))}
    for r in drows:
        assert math.isfinite(float(r[dcol["rel_l2_launcher"]]))
        assert int(r[dcol["weight_sets"]]) >= 5
    with open(os.path.splitext(csv)[0] + ".json") as f:
        summary = json.load(f)
    assert summary["kernel_backend"] == bd.KERNEL_BACKEND and summary["skipped"] == []
    fh, frows = _rows(os.path.join(out, "splitk_factor_sweep.csv"))
    assert fh == bd.FACTOR_HEADER and len(frows) == 3 * 4 * 3
    assert all(r[col["pass"]] == "1" for r in frows)
    assert {r[-1] for r in frows} == {"1", "2", "4", "8"}
    ph, prows = _rows(os.path.join(out, "ablation_pdl_placement.csv"))
    assert ph == bd.PLACEMENT_HEADER and len(prows) == 3 * 3 * 3
    assert all(r[col["pass"]] == "1" for r in prows)

    # resume: every canonical row is already there, nothing is re-measured
    assert bd.main(["--models", "qwen36", "--ms", "1,8,128", "--steps", "0,3,5,6,7", "--reps", "2",
                    "--iso-samples", "3", "--b2b-batch", "6", "--out", out, "--resume"]) == 0
    _, rows2 = _rows(csv)
    assert rows2 == rows


def test_tune_best_table(tmp_path):
    out = str(tmp_path)
    assert bd.main(["--models", "qwen36", "--ms", "4", "--tune-only", "--protocols", "PDL", "--reps", "1",
                    "--b2b-batch", "4", "--out", out, "--weight-cache-gb", "3"]) == 0
    tune = [n for n in os.listdir(out) if n.startswith("tune_") and n.endswith("_best.csv")]
    assert len(tune) == 1
    header, rows = _rows(os.path.join(out, tune[0]))
    assert header == bd.TUNE_BEST_HEADER
    assert 1 <= len(rows) <= 108
    ranks = [int(r[7]) for r in rows]
    assert ranks == list(range(1, len(rows) + 1)) and rows[0][8] == "1"
    lat = [float(r[10]) for r in rows]
    assert lat == sorted(lat)
