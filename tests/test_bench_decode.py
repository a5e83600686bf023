"""Host logic of the bench_decode harness (no GPU): option parsing, the step
ladder, CSV formats, percentiles, resume and purge (the reference's
bench/bench_decode.cu:98-312, :582-603, :1117-1476 and bench/configs.cuh)."""

import math
import os

import pytest

from decode_opt_b200 import bench_decode as bd


def test_parse_int_ranges():
    assert bd.parse_int_ranges("all", 0, 7) == list(range(8))
    assert bd.parse_int_ranges("", 1, 3) == [1, 2, 3]
    assert bd.parse_int_ranges("0-3,5", 0, 6) == [0, 1, 2, 3, 5]
    assert bd.parse_int_ranges("3-1", 0, 6) == [1, 2, 3]
    assert bd.parse_int_ranges("1,2,200,2", 1, 128) == [1, 2]
    assert bd.parse_int_ranges("4,all", 0, 2) == [0, 1, 2]
    assert bd.parse_int_ranges("x", 1, 128) == []           # atoi("x") = 0: out of range


def test_parse_args_defaults_and_flags():
    o = bd.parse_args([])
    assert o.steps == list(range(8)) and o.ms == [1, 2, 4, 8, 16, 32, 64, 128]
    assert o.reps == 3 and o.iso_samples == 0 and o.b2b_batch == 0 and o.out_dir == "results"
    assert bd.wanted_protocols(o) == ["ISO", "B2B", "PDL"]
    o = bd.parse_args(["--protocols", "iso,pdl", "--models", "qwen36,glm52", "--ms", "1-4", "--reps", "0"])
    assert bd.wanted_protocols(o) == ["ISO", "PDL"] and o.models == ["qwen36", "glm52"]
    assert o.ms == [1, 2, 3, 4] and o.reps == 1
    o = bd.parse_args(["--resume", "x.csv", "--verbose"])
    assert o.resume and o.resume_path == "x.csv" and o.verbose
    o = bd.parse_args(["--resume", "--verbose"])
    assert o.resume and o.resume_path == "" and o.verbose
    o = bd.parse_args(["--resume", "--no-resume"])
    assert not o.resume
    o = bd.parse_args(["--splitk-factor-sweep"])
    assert o.splitk_factors == [1, 2, 4, 8]
    o = bd.parse_args(["--splitk-factors", "1-8"])
    assert o.splitk_factors == [1, 2, 4, 8]
    o = bd.parse_args(["--tune-out", "t.csv"])
    assert o.tune and o.tune_out == "t.csv"
    o = bd.parse_args(["--demo", "--models", "a,b"])
    assert o.steps == [0, 1] and o.ms == [1, 8] and o.reps == 1 and o.models == ["a"]
    for bad in (["--bogus"], ["--reps"], ["--protocols", "XYZ"]):
        with pytest.raises(SystemExit) as e:
            bd.parse_args(bad)
        assert e.value.code == 2


def test_timing_plan_big_k():
    o = bd.parse_args([])
    assert bd.plan_for(16384, o) == bd.TimingPlan(3, 20, 50)
    assert bd.plan_for(4096, o) == bd.TimingPlan(3, 30, 90)
    o = bd.parse_args(["--iso-samples", "7", "--b2b-batch", "11"])
    assert bd.plan_for(16384, o) == bd.TimingPlan(3, 7, 11)


def test_models_table_and_json(tmp_path):
    ms = bd.builtin_models()
    assert [(m.id, m.N, m.K) for m in ms] == [("kimi_k3", 7168, 12288), ("qwen36", 2048, 4096),
                                              ("glm52", 6144, 16384), ("deepseek_v4_pro", 7168, 16384),
                                              ("minimax_m3", 6144, 8192)]
    p = tmp_path / "models.json"
    p.write_text('{"models": [{"id": "x", "display": "X", "hidden": 512, "gemm": {"layer": "o", "N": 512, '
                 '"K": 1024}}]}')
    got, note = bd.load_models(str(p))
    assert got == [bd.ModelShape("x", "X", "o", 512, 512, 1024)] and note == str(p)
    got, note = bd.load_models(str(tmp_path / "missing.json"))
    assert got == ms and note.startswith("FALLBACK")
    sel, missing = bd.select_models(ms, ["glm52", "nope"])
    assert [m.id for m in sel] == ["glm52"] and missing == ["nope"]


def test_choose_bm_and_splitk_rule():
    # bench/configs.cuh comments: N=6144 -> BM48 (128 tiles), 7168 -> BM56, 2048 -> BM32
    assert bd.choose_bm(7168) == 56
    assert bd.choose_bm(6144) == 48
    assert bd.choose_bm(2048) == 32
    assert bd.splitk_worth_it(7168, 56, 148)          # 128 tiles -> 256 >= 148
    assert not bd.splitk_worth_it(7168, 56, 78)       # H20: 128 tiles already a wave
    assert not bd.splitk_worth_it(2048, 32, 148)      # 64 tiles -> 128 < 148


def test_canonical_ladder():
    kc = bd.canonical_kernel_config(0, 8, 7168, 16384, 1, 148)
    assert bd.config_string(kc) == ("M_TILE=8;BM=64;WG=4;REG=112;STG=2;TILES=1;SUBS=1;PREPACK=0;PDL=0;EPI=0;"
                                    "SPLITK=0;SK=1;PR=32;SPW=0;PLA=0;SISM=1")
    kc = bd.canonical_kernel_config(4, 8, 7168, 16384, 8, 148)
    assert (kc.OUTPUT_ROWS_PER_CTA, kc.NUM_MATH_WG, kc.MATH_REGS, kc.STAGES_PER_WG, kc.SUBS_PER_STAGE,
            kc.PREPACK, kc.PDL, kc.kSplitKFactor) == (56, 2, 80, 3, 2, True, True, 1)
    assert bd.canonical_kernel_config(5, 8, 7168, 16384, 1, 148).kSplitKFactor == 1      # M < 8
    assert bd.canonical_kernel_config(5, 8, 7168, 16384, 8, 148).kSplitKFactor == 2
    kc = bd.canonical_kernel_config(2, 128, 6144, 16384, 100, 148)
    assert (kc.OUTPUT_ROWS_PER_CTA, kc.MATH_REGS, kc.SUBS_PER_STAGE, kc.TILES_PER_CTA, kc.kScaleInSmem,
            kc.PREPACK) == (48, 168, 1, 2, False, False)
    kc = bd.canonical_kernel_config(5, 16, 7168, 16384, 16, 148, splitk=8)
    assert kc.kSplitKFactor == 8 and "SPLITK=1;SK=8" in bd.config_string(kc)
    # K/(128*SUBS*S) must divide: K = 1024 with SUBS=2 cannot take S=8
    assert bd.canonical_kernel_config(5, 16, 7168, 1024, 16, 148, splitk=8).kSplitKFactor == 1
    assert "," not in bd.config_string(kc)


def test_b200_config_string():
    cfg = dict(m_tile=8, block_n=256, subs=2, stages=2, layout=2, pdl=True, split_k=1, grid_ctas=-1, epi_warps=0,
               flags=4, timeout_ns=0)
    assert bd.b200_config_string(cfg) == ("B200;M_TILE=8;BN=256;SUBS=2;STAGES=2;LAYOUT=swizzled;GRID=streamk;"
                                          "PDL=1;SK=1;ACT_EARLY=1")
    assert len(bd.tune_grid(1)) == 108 and all(c["m_tile"] == 8 for c in bd.tune_grid(3))


def test_number_formats_and_fields():
    assert bd.f4(1.23456789) == "1.2346" and bd.f3(2.0) == "2.000" and bd.f6(0.5) == "0.500000"
    assert bd.fe6(0.00123456) == "1.234560e-03"
    for f in (bd.f4, bd.f3, bd.f6, bd.fe6):
        assert f(float("nan")) == "nan" and f(float("inf")) == "nan"
    assert bd.csv_field("a;b") == "a;b"
    assert bd.csv_field('a,"b"') == '"a,""b"""'


def test_row_main_and_detail():
    r = bd.CsvRow(model="deepseek_v4_pro", N=7168, K=16384, M=1, m_tile=8, step=6, step_name="b200",
                  config="B200;BN=256", rel_l2=1.1e-3, passed="1", clocks_mhz=1965, reps=3, iso_samples=20,
                  b2b_batch=50, pdl_batch=50)
    r.fill_stats("PDL", bd.TimingStats(23.5, 23.4, 23.3, 23.45, 3))
    line = bd.row_main(r)
    f = line.split(",")
    assert bd.CSV_HEADER.count(",") + 1 == 16 == len(f)
    assert f[:9] == ["deepseek_v4_pro", "7168", "16384", "1", "8", "6", "b200", "PDL", "23.5000"]
    bw = (7168 * 16384 + 16384 + 2 * 7168) / 23.5e-6 / 1e9
    assert f[10] == f"{bw:.3f}" and f[11] == f"{bw / 8000.0:.6f}"
    assert f[12:] == ["1965", "1.100000e-03", "1", "B200;BN=256"]
    d = bd.row_detail(r).split(",")
    assert len(d) == bd.DETAIL_HEADER.count(",") + 1 == 35
    assert bd.split_csv_line(line + "\r\n") == f


def test_percentile_rule():
    v = [float(i) for i in range(1, 11)]
    assert bd.percentile(v, 0.5) == 5.0 and bd.percentile(v, 0.3) == 3.0
    assert bd.percentile([7.0], 0.3) == 7.0 and math.isnan(bd.percentile([], 0.5))
    s = bd.summarize([3.0, 1.0, 2.0, 4.0])
    assert (s.p50_us, s.p30_us, s.min_us, s.mean_us, s.n) == (2.0, 2.0, 1.0, 2.5, 4)


def _row(model, m, step, proto, p50, config="C"):
    r = bd.CsvRow(model=model, N=64, K=128, M=m, m_tile=8, step=step, step_name="s", config=config)
    r.fill_stats(proto, bd.TimingStats(p50, p50, p50, p50, 1))
    return bd.row_main(r)


def test_purge_and_resume(tmp_path):
    p = str(tmp_path / "bench_20260101T000000Z.csv")
    w = bd.CsvWriter(p, bd.CSV_HEADER)
    for proto in bd.PROTOCOLS:                     # complete group
        w.write(_row("a", 1, 0, proto, 2.0))
    w.write(_row("a", 8, 0, "ISO", 2.0))            # missing B2B, PDL
    w.write(_row("a", 8, 0, "B2B", 2.0))
    for proto in bd.PROTOCOLS:                     # one nan latency
        w.write(_row("b", 1, 1, proto, float("nan") if proto == "PDL" else 1.0, config='x,"y"'))
    w.close()
    assert bd.purge_incomplete_groups(p, []) == (3, 5, 2)
    assert bd.purge_incomplete_groups(p, []) == (3, 0, 0)
    done = bd.DoneSet()
    assert done.load(p, False) and done.rows == 3
    probe = bd.CsvRow(model="a", N=64, K=128, M=1, m_tile=8, step=0, protocol="PDL", config="C")
    assert done.has(False, probe) and not done.has(True, probe)
    probe.config = "other"
    assert not done.has(False, probe)
    # purge against the requested protocols only
    p2 = str(tmp_path / "bench_20260102T000000Z.csv")
    w = bd.CsvWriter(p2, bd.CSV_HEADER)
    w.write(_row("a", 1, 0, "PDL", 2.0))
    w.close()
    assert bd.purge_incomplete_groups(p2, ["PDL"]) == (1, 0, 0)
    w = bd.CsvWriter(p2, bd.CSV_HEADER, append=True)
    assert w.rows == 1
    w.close()
    open(str(tmp_path / "bench_20260103T000000Z_detail.csv"), "w").close()
    assert bd.newest_csv(str(tmp_path), "bench_") == p2
    assert bd.newest_csv(str(tmp_path / "none"), "bench_") is None


def test_csv_lock(tmp_path):
    p = str(tmp_path / "x.csv")
    a, b = bd.CsvLock(p), bd.CsvLock(p)
    assert a.acquire()
    assert not b.acquire()
    a.release()
    assert b.acquire()
    b.release()
    assert not os.path.exists(p + ".lock")


def test_block_quantize_matches_formula():
    torch = pytest.importorskip("torch")
    g = torch.Generator().manual_seed(5)
    x = torch.randn((130, 256), generator=g) / 16.0
    q, s = bd.block_quantize(x, 128)
    assert q.shape == (130, 256) and q.dtype == torch.uint8 and s.shape == (2, 2)
    blk = x[:128, 128:256]
    np = pytest.importorskip("numpy")
    want_scale = np.float32(max(np.float32(blk.abs().max()), np.float32(1e-4))) / np.float32(448.0)
    assert float(s[0, 1]) == float(want_scale)                          # fp32 arithmetic, exact
    v = np.float32(x[3, 200]) / np.float32(s[0, 1])
    want = torch.tensor([max(-448.0, min(448.0, float(v)))]).to(torch.float8_e4m3fn).view(torch.uint8)
    assert int(q[3, 200]) == int(want[0])
    back = bd.dequantize(q, s, 128)
    assert float((back - x).abs().max()) <= float(s.max()) * 32        # e4m3 step at 448 is 32
    qa, sa = bd.block_quantize(x[:3], 1)
    assert sa.shape == (3, 2)


def test_list_runs_without_gpu(capsys):
    assert bd.main(["--list", "--models", "qwen36"]) == 0
    out = capsys.readouterr().out
    assert "qwen36" in out and "S6 b200" in out and "S7 b200_indep" in out and "108 configurations" in out
    assert bd.main(["--list", "--models", "nope"]) == 2
