"""The bandwidth-vs-M figures (no GPU): the reference's curve rule (step 0
from B2B, later steps from PDL, another protocol only as a marked fallback),
bandwidth recomputed from N, K, M and p50, failed rows dropped, and the SVG's
reference lines (spec, measured peak only when given, compute roof only where
it is below the spec)."""

import json
import xml.etree.ElementTree as ET

import pytest

from decode_opt_b200 import bench_decode as bd
from decode_opt_b200 import plot

NS = "{http://www.w3.org/2000/svg}"


def _write_csv(path, rows):
    with open(path, "w") as f:
        f.write(bd.CSV_HEADER + "\n")
        for model, n, k, m, step, proto, p50, passed in rows:
            r = bd.CsvRow(model=model, N=n, K=k, M=m, m_tile=bd.m_tile_for(m), step=step,
                          step_name=bd.STEP_NAMES[step], passed=passed, config="C")
            r.fill_stats(proto, bd.TimingStats(p50, p50, p50, p50, 1))
            f.write(bd.row_main(r) + "\n")


def test_curve_rule_and_bandwidth(tmp_path):
    p = str(tmp_path / "bench_x.csv")
    _write_csv(p, [
        ("a", 2048, 4096, 1, 0, "B2B", 10.0, "1"), ("a", 2048, 4096, 1, 0, "PDL", 5.0, "1"),
        ("a", 2048, 4096, 8, 0, "B2B", 11.0, "1"),
        ("a", 2048, 4096, 1, 6, "PDL", 4.0, "1"), ("a", 2048, 4096, 1, 6, "B2B", 3.0, "1"),
        ("a", 2048, 4096, 8, 6, "ISO", 9.0, "1"),                    # no PDL row at M=8: fallback
        ("a", 2048, 4096, 16, 6, "PDL", 1.0, "0"),                   # failed row: dropped
    ])
    (mc,) = plot.build_curves(plot.load_rows([p]))
    assert (mc.model, mc.n, mc.k) == ("a", 2048, 4096)
    c0, c6 = mc.curves[0], mc.curves[6]
    assert c0.protocol == "B2B" and not c0.fallback
    assert [m for m, _ in c0.points] == [1, 8]
    assert c0.points[0][1] == pytest.approx(plot.moved_bytes(2048, 4096, 1) / 10e-6 / 1e9)
    assert c6.fallback and [m for m, _ in c6.points] == [1, 8]
    assert c6.points[0][1] == pytest.approx(plot.moved_bytes(2048, 4096, 1) / 4e-6 / 1e9)
    assert plot.build_curves(plot.load_rows([p]), steps=[6])[0].curves.keys() == {6}


def test_roof_formula():
    # B200 FP8 roof is far above the spec at decode sizes; a tiny peak makes it bind
    assert plot.roof_gbps(128, 7168, 16384, plot.FP8_DENSE_TFLOPS, 8000.0) == 8000.0
    m, n, k, tf = 128, 7168, 16384, 10.0
    want = plot.moved_bytes(n, k, m) / (2.0 * m * n * k / (tf * 1e12)) / 1e9
    assert plot.roof_gbps(m, n, k, tf, 8000.0) == pytest.approx(want)


def test_svg_files_and_reference_lines(tmp_path, capsys):
    p = str(tmp_path / "bench_20260101T000000Z.csv")
    rows = []
    for model in ("a", "b"):
        for step in (0, 4, 6, 7):
            for m in (1, 8, 64, 128):
                rows.append((model, 7168, 16384, m, step, "B2B" if step == 0 else "PDL", 20.0 + m / 8, "1"))
    _write_csv(p, rows)
    peaks = tmp_path / "peaks.json"
    peaks.write_text(json.dumps({"hbm_gbs": 6555.2}))
    out = tmp_path / "figs"
    assert plot.main([p, "--out", str(out), "--peaks", str(peaks)]) == 0
    names = sorted(x.name for x in out.iterdir())
    assert names == ["fig_bw_vs_M_a.svg", "fig_bw_vs_M_b.svg", "fig_main_bw_vs_M.svg"]
    root = ET.parse(out / "fig_main_bw_vs_M.svg").getroot()
    classes = [g.get("class") for g in root.iter() if g.get("class")]
    assert classes.count("ref-spec") == 2 and classes.count("ref-measured") == 2
    assert "ref-roof" not in classes                     # the roof never drops below 8 TB/s here
    assert {c for c in classes if c.startswith("step-")} == {"step-0", "step-4", "step-6", "step-7"}
    text = " ".join(t.text or "" for t in root.iter(NS + "text"))
    assert "measured HBM peak 6555 GB/s" in text and "8000 GB/s" in text
    # no peaks file: the measured line is left out, never invented
    out2 = tmp_path / "figs2"
    assert plot.main([p, "--out", str(out2), "--peaks", str(tmp_path / "none.json"), "--tflops", "10"]) == 0
    root2 = ET.parse(out2 / "fig_bw_vs_M_a.svg").getroot()
    classes2 = [g.get("class") for g in root2.iter() if g.get("class")]
    assert "ref-measured" not in classes2 and "ref-roof" in classes2
    assert "measured line is left out" in capsys.readouterr().err


def test_newest_csv_default(tmp_path):
    _write_csv(str(tmp_path / "bench_20260101T000000Z.csv"), [("a", 64, 128, 1, 6, "PDL", 1.0, "1")])
    _write_csv(str(tmp_path / "bench_20260102T000000Z.csv"), [("z", 64, 128, 1, 6, "PDL", 1.0, "1")])
    (tmp_path / "bench_20260103T000000Z_detail.csv").write_text("x\n")
    assert plot.newest_csv(str(tmp_path)).endswith("bench_20260102T000000Z.csv")
    assert plot.main(["--results", str(tmp_path), "--peaks", ""]) == 0
    assert (tmp_path / "fig_bw_vs_M_z.svg").exists()
    assert plot.main(["--results", str(tmp_path / "empty")]) == 2
