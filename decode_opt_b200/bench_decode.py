"""Sweep harness for the sm_100a decode GEMM with the reference's CLI and CSV.

    python -m decode_opt_b200.bench_decode [--models all|id,...] [--steps all|0-6]
        [--ms all|1,2,4,...] [--protocols ISO,B2B,PDL] [--reps R] [--out DIR]
        [--tune] [--splitk-ablation] [--pdl-placement] [--splitk-factor-sweep]
        [--resume [CSV]] [--list] [--demo] ...

The rebuild of the reference's `bench_decode` (bench/bench_decode.cu:98-312
options, :1145-1480 CSV/resume, :1527-1700 measurement): for every model shape
W[N, K], batch size M and step of the optimisation ladder it times one launch
configuration under up to three protocols and writes one row per protocol to
a CSV with the reference's 16 columns, column order and number formats
(bench/bench_decode.cu:1167-1213), a detail sidecar with the reference's 35
columns (`<csv>_detail.csv`) and a JSON summary (`<csv>.json`).

Steps (the reference's ladder, bench/configs.cuh:42-43 and :255-288, plus one
B200 step):

  0 baseline    1 pdl    2 blockk    3 prepack    4 tile_stage    5 splitk
      the reference's canonical KernelConfig of the step, run by the sm_100a
      kernel with the reference's schedule (one CTA per BM-row output tile,
      times the split-K factor); the ring depth WG*STG is reduced when it
      does not fit in shared memory (STAGES_SM100 in the config column);
  6 b200
      the B200 schedule for dependent launches (``default_config``): cluster
      split-K -- each tile's K range split over one thread-block cluster and
      reduced through distributed shared memory, as many clusters as one
      wave holds -- with the descriptor-ready swizzled weight layout and the
      early PDL trigger; activations are read after griddepcontrol.wait;
  7 b200_indep
      the B200 schedule for independent inputs (FLAG_INDEPENDENT_INPUTS:
      activations read before griddepcontrol.wait, writes after; fewer CTAs
      per GEMM), under which back-to-back GEMMs of the PDL protocol stream
      side by side -- the reference kernel, which never waits on the grid
      dependency, is timed the same way.

S5 turns 2-way split-K on where the reference's rule says it pays: M >= 8 and
the tile count in [ceil(SMs/2), SMs) (bench/configs.cuh:398-406), with this
GPU's SM count in place of the H20's 78.

Protocols (bench/bench_decode.cu:935-985): ISO = one launch after an L2
flushing write, CUDA events around the launch alone (reps x iso_samples
samples); B2B = `batch` launches back to back, time / batch per rep; PDL = the
same with programmatic dependent launch.  The batches are captured once in a
CUDA graph and replayed, so host launch cost is not timed.  Every launch
reads its weights cold: a point rotates over max(5, ceil(max(1 GiB, 4 x L2) /
weight bytes)) device copies.  p50/p30 use the reference's percentile rule
(bench/bench_decode.cu:582-603).

bandwidth_gbps = (N*K + M*K + 2*M*N) / p50 (bench/bench_decode.cu:1069-1072);
pct_of_spec_peak = bandwidth / 8000 GB/s (B200 HBM3e nominal; the reference
divides by the H20's 4000).  rel_l2 compares one launch's bf16 output with an
fp32 product of the dequantised operands computed by torch on the GPU (TF32
off; the reference uses a cuBLASLt SGEMM, bench/bench_decode.cu:2343-2378);
pass = finite and rel_l2 <= 2e-3.

Synthetic inputs follow the reference's recipe (bench/bench_decode.cu:404-470):
N(0,1)/sqrt(K) values, weights quantised per 128x128 block and activations
per 1x128 block with scale = max(amax, 1e-4)/448; the draws come from torch's
seeded generator on the GPU, not from std::mt19937_64.
"""

from __future__ import annotations

import fcntl
import json
import math
import os
import sys
import time
from dataclasses import dataclass, field
from datetime import datetime, timezone
from typing import Dict, List, Optional, Sequence, Tuple

from . import m_tile_for

KERNEL_BACKEND = "sm100a_tcgen05"
SPEC_PEAK_GBPS = 8000.0
REL_L2_THRESHOLD = 2e-3
BIG_K = 16384
WARMUP_LAUNCHES = 10
DEFAULT_SEED = 20260913
K_BLOCK = 128
FP8_MAX = 448.0
QUANT_EPS = 1.0e-4

STEP_NAMES = ("baseline", "pdl", "blockk", "prepack", "tile_stage", "splitk", "b200", "b200_indep")
STEP_B200 = 6
STEP_B200_INDEP = 7
PROTOCOLS = ("ISO", "B2B", "PDL")

CSV_HEADER = ("model,N,K,M,m_tile,step,step_name,protocol,latency_us_p50,latency_us_p30,"
              "bandwidth_gbps,pct_of_spec_peak,clocks_sm_mhz,rel_l2,pass,config")
DETAIL_HEADER = (CSV_HEADER + ",latency_us_min,latency_us_mean,samples,reps,iso_samples,b2b_batch,"
                 "pdl_batch,variant_kind,tune_index,rank,is_best,padded_n,weight_sets,"
                 "weight_set_bytes,smem_bytes,num_ctas,num_threads,launch_mechanism,rel_l2_launcher")
ABLATION_HEADER = CSV_HEADER + ",splitk_on"
PLACEMENT_HEADER = CSV_HEADER + ",pdl_trigger"
FACTOR_HEADER = CSV_HEADER + ",splitk_factor"
TUNE_BEST_HEADER = ("model,N,K,M,m_tile,step,step_name,rank,is_best,rank_protocol,"
                    "latency_us_p50,latency_us_p30,bandwidth_gbps,pct_of_spec_peak,"
                    "clocks_sm_mhz,rel_l2,pass,config,smem_bytes,num_ctas,weight_sets")

NAN = float("nan")


# ---------------------------------------------------------------------------
# Model table
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class ModelShape:
    id: str
    display: str
    layer: str
    hidden: int
    N: int
    K: int


def builtin_models() -> List[ModelShape]:
    """The reference's fallback table (bench/bench_decode.cu:325-332)."""
    return [
        ModelShape("kimi_k3", "Kimi-K3", "o_proj", 7168, 7168, 12288),
        ModelShape("qwen36", "Qwen3.6-35B-A3B", "o_weight", 2048, 2048, 4096),
        ModelShape("glm52", "GLM-5.2", "wo", 6144, 6144, 16384),
        ModelShape("deepseek_v4_pro", "DeepSeek-V4-Pro", "wo_b", 7168, 7168, 16384),
        ModelShape("minimax_m3", "MiniMax-M3", "w_o", 6144, 6144, 8192),
    ]


def load_models(path: Optional[str]) -> Tuple[List[ModelShape], str]:
    """Models from a models.json ({"models": [{"id", "display", "hidden",
    "gemm": {"layer", "N", "K"}}]}, the reference's models/models.json
    schema), or the builtin table when `path` is None or unreadable."""
    if not path:
        return builtin_models(), "builtin table"
    try:
        with open(path) as f:
            doc = json.load(f)
        out = []
        for m in doc["models"]:
            g = m["gemm"]
            out.append(ModelShape(str(m["id"]), str(m.get("display", m["id"])), str(g.get("layer", "")),
                                  int(m.get("hidden", g["N"])), int(g["N"]), int(g["K"])))
        if not out:
            raise ValueError("no models")
        return out, path
    except (OSError, ValueError, KeyError, TypeError) as e:
        return builtin_models(), f"FALLBACK (builtin table): cannot read {path}: {e}"


def select_models(all_models: Sequence[ModelShape], wanted: Sequence[str]) -> Tuple[List[ModelShape], List[str]]:
    if not wanted:
        return list(all_models), []
    by_id = {m.id: m for m in all_models}
    return [by_id[w] for w in wanted if w in by_id], [w for w in wanted if w not in by_id]


# ---------------------------------------------------------------------------
# Options (bench/bench_decode.cu:98-312)
# ---------------------------------------------------------------------------

def parse_int_ranges(text: str, lo: int, hi: int) -> List[int]:
    """"all", "a-b" and comma lists, clipped to [lo, hi], sorted, unique
    (bench/bench_decode.cu:193-221)."""
    if text in ("", "all"):
        return list(range(lo, hi + 1))
    out = set()
    for item in text.split(","):
        if not item:
            continue
        if item == "all":
            out.update(range(lo, hi + 1))
            continue
        dash = item.find("-")
        if dash < 0:
            v = _atoi(item)
            if lo <= v <= hi:
                out.add(v)
        else:
            a, b = _atoi(item[:dash]), _atoi(item[dash + 1:])
            out.update(v for v in range(min(a, b), max(a, b) + 1) if lo <= v <= hi)
    return sorted(out)


def _atoi(s: str) -> int:
    """C atoi: leading integer, 0 when there is none."""
    s = s.strip()
    n = 0
    sign = 1
    i = 0
    if i < len(s) and s[i] in "+-":
        sign = -1 if s[i] == "-" else 1
        i += 1
    digits = 0
    while i < len(s) and s[i].isdigit():
        n = n * 10 + int(s[i])
        i += 1
        digits += 1
    return sign * n if digits else 0


def parse_csv_strings(text: str) -> List[str]:
    if text in ("", "all"):
        return []
    return [t for t in text.split(",") if t and t != "all"]


@dataclass
class Options:
    models: List[str] = field(default_factory=list)
    steps: List[int] = field(default_factory=list)
    ms: List[int] = field(default_factory=list)
    tune: bool = False
    tune_only: bool = False
    reps: int = 3
    iso_samples: int = 0
    b2b_batch: int = 0
    out_dir: str = ""
    models_json: str = ""
    seed: int = DEFAULT_SEED
    demo: bool = False
    no_correctness: bool = False
    check_launcher: bool = False
    list_only: bool = False
    verbose: bool = False
    weight_cache_gb: float = 8.0
    force_api_launch: bool = False
    allow_shared: bool = False
    l2_flush_mb: int = 256
    protocols: List[str] = field(default_factory=list)
    splitk_ablation: bool = False
    pdl_placement: bool = False
    ablation_out: str = ""
    splitk_factor_sweep: bool = False
    splitk_factors: List[int] = field(default_factory=list)
    factor_out: str = ""
    tune_out: str = ""
    purge_only: str = ""
    resume: bool = False
    resume_path: str = ""
    no_resume: bool = False


USAGE = """usage: python -m decode_opt_b200.bench_decode [options]
  --models all|id,...        model ids (default all; see --list)
  --models-json PATH         model table in the models.json schema
  --steps all|0-7            ladder steps (0..5 the reference's, 6 and 7 the B200 schedule)
  --ms all|1,2,4,...         batch sizes in [1, 128] (default 1,2,4,8,16,32,64,128)
  --protocols ISO,B2B,PDL    protocols to time (default all three)
  --reps R                   repetitions (default 3)
  --iso-samples S            ISO samples per rep (default 30; 20 when K >= 16384)
  --b2b-batch B              launches per B2B/PDL batch (default 90; 50 when K >= 16384)
  --out DIR                  output directory (default ./results)
  --seed S                   input seed (default 20260913)
  --tune / --tune-only       also (only) sweep the B200 tune grid; --tune-out PATH
  --splitk-ablation          step 5 with split-K on and off (ablation_splitk.csv)
  --pdl-placement            steps 4 and 6 with each PDL trigger placement
  --ablation-out PATH        CSV of either ablation (default in --out)
  --splitk-factor-sweep      step 5 geometry with S in --splitk-factors (default 1,2,4,8)
  --factor-out PATH          CSV of the factor sweep
  --resume [CSV]             append to CSV (default: newest bench_*.csv in --out), skipping
                             rows already measured; incomplete groups are dropped first
  --resume-from CSV, --no-resume
  --purge-only CSV           drop incomplete groups from CSV and exit
  --no-correctness           skip the fp32 reference check
  --check-launcher           also check the output of the map-encoding launch entry
  --force-api-launch         time the map-encoding launch entry instead of launch_with_maps
  --weight-cache-gb G        device budget of cold weight copies (default 8)
  --l2-flush-mb MB           L2 flush size of ISO (default 256)
  --allow-shared             run although other compute processes use the GPU
  --demo                     steps 0,1; M 1,8; 1 rep; first model
  --list                     print models and step configurations, then exit
  --verbose
"""


def parse_args(argv: Sequence[str]) -> Options:
    """The reference's parser (bench/bench_decode.cu:233-312): same flags and
    defaults; unknown flags exit with status 2."""
    o = Options()
    argv = list(argv)
    i = 0

    def need() -> str:
        nonlocal i
        if i + 1 >= len(argv):
            sys.stderr.write(f"[bench] {argv[i]} needs a value\n")
            raise SystemExit(2)
        i += 1
        return argv[i]

    while i < len(argv):
        a = argv[i]
        if a == "--models":
            o.models = parse_csv_strings(need())
        elif a == "--steps":
            o.steps = parse_int_ranges(need(), 0, 7)
        elif a == "--ms":
            o.ms = parse_int_ranges(need(), 1, 128)
        elif a == "--tune":
            o.tune = True
        elif a == "--tune-only":
            o.tune = o.tune_only = True
        elif a == "--reps":
            o.reps = max(1, _atoi(need()))
        elif a == "--iso-samples":
            o.iso_samples = max(1, _atoi(need()))
        elif a == "--b2b-batch":
            o.b2b_batch = max(1, _atoi(need()))
        elif a == "--out":
            o.out_dir = need()
        elif a == "--models-json":
            o.models_json = need()
        elif a == "--seed":
            o.seed = int(need())
        elif a == "--demo":
            o.demo = True
        elif a == "--no-correctness":
            o.no_correctness = True
        elif a == "--check-launcher":
            o.check_launcher = True
        elif a == "--list":
            o.list_only = True
        elif a == "--verbose":
            o.verbose = True
        elif a == "--weight-cache-gb":
            o.weight_cache_gb = float(need())
        elif a == "--force-api-launch":
            o.force_api_launch = True
        elif a == "--allow-shared":
            o.allow_shared = True
        elif a == "--protocols":
            o.protocols = [p.upper() for p in need().split(",") if p]
        elif a == "--splitk-ablation":
            o.splitk_ablation = True
        elif a == "--pdl-placement":
            o.pdl_placement = True
        elif a == "--ablation-out":
            o.ablation_out = need()
        elif a == "--splitk-factor-sweep":
            o.splitk_factor_sweep = True
        elif a == "--splitk-factors":
            o.splitk_factors = [f for f in parse_int_ranges(need(), 1, 8) if f in (1, 2, 4, 8)]
        elif a == "--factor-out":
            o.factor_out = need()
        elif a == "--sem-rotate":
            need()   # accepted for compatibility: the sm_100a kernel's workspace writes wait for the prior grid
        elif a == "--tune-out":
            o.tune_out = need()
            o.tune = True
        elif a == "--purge-only":
            o.purge_only = need()
        elif a == "--resume":
            o.resume = True
            if i + 1 < len(argv) and not argv[i + 1].startswith("--"):
                i += 1
                o.resume_path = argv[i]
        elif a == "--resume-from":
            o.resume = True
            o.resume_path = need()
        elif a == "--no-resume":
            o.no_resume = True
            o.resume = False
        elif a == "--l2-flush-mb":
            o.l2_flush_mb = max(1, _atoi(need()))
        elif a in ("-h", "--help"):
            sys.stdout.write(USAGE)
            raise SystemExit(0)
        else:
            sys.stderr.write(f"[bench] unknown argument: {a}\n{USAGE}")
            raise SystemExit(2)
        i += 1
    if o.no_resume:
        o.resume = False
    if o.splitk_factor_sweep and not o.splitk_factors:
        o.splitk_factors = [1, 2, 4, 8]
    bad = [p for p in o.protocols if p not in PROTOCOLS]
    if bad:
        sys.stderr.write(f"[bench] unknown protocol(s): {','.join(bad)}\n")
        raise SystemExit(2)
    if not o.steps:
        o.steps = list(range(0, 8))
    if not o.ms:
        o.ms = [1, 2, 4, 8, 16, 32, 64, 128]
    if o.demo:
        o.steps, o.ms, o.reps, o.iso_samples, o.b2b_batch = [0, 1], [1, 8], 1, 10, 30
        o.models = o.models[:1]
    if not o.out_dir:
        o.out_dir = "results"
    return o


def wanted_protocols(o: Options) -> List[str]:
    return [p for p in PROTOCOLS if not o.protocols or p in o.protocols]


@dataclass(frozen=True)
class TimingPlan:
    reps: int
    iso_samples: int
    batch: int


def plan_for(k: int, o: Options) -> TimingPlan:
    """bench/bench_decode.cu:564-571: fewer samples for K >= 16384."""
    big = k >= BIG_K
    return TimingPlan(o.reps, o.iso_samples or (20 if big else 30), o.b2b_batch or (50 if big else 90))


# ---------------------------------------------------------------------------
# Step ladder (bench/configs.cuh)
# ---------------------------------------------------------------------------

CANDIDATE_BM = (32, 40, 48, 56, 64)
TARGET_TILES = 128


def choose_bm(n: int) -> int:
    """bench/configs.cuh:211-226: no padding first, then a tile count closest
    to 128, then the larger BM (first candidate wins a tie)."""
    def score(bm: int) -> int:
        tiles = -(-n // bm)
        return (tiles * bm - n) * 1000000 + abs(tiles - TARGET_TILES) * 1000 - bm
    best = CANDIDATE_BM[0]
    for bm in CANDIDATE_BM[1:]:
        if score(bm) < score(best):
            best = bm
    return best


def splitk_worth_it(n: int, bm: int, sms: int) -> bool:
    """bench/configs.cuh:398-406 with this GPU's SM count: doubling the CTA
    count must still fit one wave."""
    tiles = -(-n // bm)
    return tiles < sms and 2 * tiles >= sms


@dataclass(frozen=True)
class StepVariant:
    """One measured configuration: a ladder step's reference KernelConfig
    (steps 0..5) or the B200 schedule (step 6)."""
    step: int
    m_tile: int
    kernel_config: object = None        # decode_opt_b200.KernelConfig for steps 0..5
    b200: Optional[dict] = None         # B200Config fields for step 6 / tune
    label: str = ""                     # ablation value (splitk_on / pdl_trigger / factor)
    kind: str = "canonical"
    tune_index: int = -1

    @property
    def step_name(self) -> str:
        if self.kind == "tune":
            return "b200_tune"
        return STEP_NAMES[self.step]


def canonical_kernel_config(step: int, m_tile: int, n: int, k: int, m: int, sms: int, splitk: Optional[int] = None):
    """The reference's canonical configuration of `step` (bench/configs.cuh:255-288
    and :242-252): M_TILE=8 uses BM=64 / WG=4 / REG=112 / STG=2 / SUBS=1 at S0-S3
    (SUBS=2 from S2) and the shape's BM / WG=2 / REG=80 / STG=3 / SUBS=2 from
    S4; M_TILE >= 16 uses the shape's BM / WG=2 / TILES=2 / STG=2 with REG 112
    (M_TILE 16) or 168 and SUBS 2 (1 at M_TILE 128).  PREPACK from S3, PDL from
    S1, 2-way split-K at S5 where `splitk_worth_it` and M >= 8 (`splitk`
    overrides the factor).  The per-shape H20 tune winners
    (bench/configs.cuh:330-352) are not applied."""
    from . import KernelConfig
    if m_tile == 8:
        if step <= 3:
            bm, wg, regs, stg, tiles, subs = 64, 4, 112, 2, 1, (2 if step >= 2 else 1)
        else:
            bm, wg, regs, stg, tiles, subs = choose_bm(n), 2, 80, 3, 1, 2
    else:
        bm, wg, stg, tiles = choose_bm(n), 2, 2, 2
        regs = 112 if m_tile == 16 else 168
        subs = 1 if m_tile >= 128 else 2
    if splitk is None:
        splitk = 2 if (step >= 5 and m >= 8 and splitk_worth_it(n, bm, sms)) else 1
    wpt = wg // tiles
    if splitk > 1 and k % (K_BLOCK * subs * wpt * splitk) != 0:
        splitk = 1
    return KernelConfig(m_tile, bm, wg, regs, stg, tiles, subs, step >= 3, step >= 1, False, splitk > 1,
                        SPLITK_FACTOR=splitk)


def config_string(kc) -> str:
    """The reference's config column (bench/configs.cuh:638-660): ';'-joined
    key=value pairs, never a comma."""
    return (f"M_TILE={kc.M_TILE};BM={kc.OUTPUT_ROWS_PER_CTA};WG={kc.NUM_MATH_WG};REG={kc.MATH_REGS};"
            f"STG={kc.STAGES_PER_WG};TILES={kc.TILES_PER_CTA};SUBS={kc.SUBS_PER_STAGE};"
            f"PREPACK={int(kc.PREPACK)};PDL={int(kc.PDL)};EPI={int(kc.EPI_OVERLAP)};"
            f"SPLITK={int(kc.kSplitKCta)};SK={kc.kSplitKFactor};PR={kc.PROD_REGS};"
            f"SPW={int(kc.SINGLE_PRODUCER_WARP)};PLA={int(kc.PRELOAD_ACT)};SISM={int(kc.kScaleInSmem)}")


LAYOUT_NAMES = {0: "raw", 1: "packed", 2: "swizzled"}


def b200_config_string(b: dict) -> str:
    grid = {0: "tiles", -1: "streamk", -2: "cluster"}.get(b["grid_ctas"], str(b["grid_ctas"]))
    s = (f"B200;M_TILE={b['m_tile']};BN={b['block_n']};SUBS={b['subs']};STAGES={b['stages']};"
         f"LAYOUT={LAYOUT_NAMES[b['layout']]};GRID={grid};PDL={int(b['pdl'])};SK={b['split_k']}")
    if b.get("flags", 0) & 4:
        s += ";ACT_EARLY=1"
    return s


def b200_step_config(m: int, n: int, k: int, independent: bool = False) -> dict:
    """Steps 6 and 7: the library's default schedule with the swizzled layout."""
    from . import LAYOUT_PACKED_SWIZZLED, default_config
    return dict(default_config(m, n, k, layout=LAYOUT_PACKED_SWIZZLED, pdl=True,
                               independent_inputs=independent).__dict__)


TUNE_BLOCK_N = (64, 128, 192, 256)
TUNE_SUBS = (1, 2, 4)
TUNE_STAGES = (2, 3, 4)
TUNE_GRIDS = (0, -1, -2)


def tune_grid(m: int) -> List[dict]:
    """The B200 tune grid: BN x SUBS x ring depth x schedule (reference tiles,
    stream-K, or cluster split-K with the library's split), swizzled layout,
    PDL trigger on.  It replaces the reference's
    SM90 grid (bench/configs.cuh:466-486), whose WG/REG/TILES knobs do not
    exist on the sm_100a kernel."""
    from . import LAYOUT_PACKED_SWIZZLED
    out = []
    for bn in TUNE_BLOCK_N:
        for subs in TUNE_SUBS:
            for st in TUNE_STAGES:
                for grid in TUNE_GRIDS:
                    out.append(dict(m_tile=m_tile_for(m), block_n=bn, subs=subs, stages=st,
                                    layout=LAYOUT_PACKED_SWIZZLED, pdl=True, split_k=1, grid_ctas=grid,
                                    epi_warps=0, flags=0, timeout_ns=0))
    return out


# ---------------------------------------------------------------------------
# CSV (bench/bench_decode.cu:1117-1300)
# ---------------------------------------------------------------------------

def csv_field(s: str) -> str:
    if not any(c in s for c in ',"\n'):
        return s
    return '"' + s.replace('"', '""') + '"'


def _finite(v) -> bool:
    return isinstance(v, (int, float)) and math.isfinite(v)


def f4(v) -> str:
    return f"{v:.4f}" if _finite(v) else "nan"


def f3(v) -> str:
    return f"{v:.3f}" if _finite(v) else "nan"


def f6(v) -> str:
    return f"{v:.6f}" if _finite(v) else "nan"


def fe6(v) -> str:
    return f"{v:.6e}" if _finite(v) else "nan"


def percentile(sorted_vals: Sequence[float], q: float) -> float:
    """bench/bench_decode.cu:582-589: the ceil(q*n)-th smallest (1-based,
    clamped to [1, n])."""
    if not sorted_vals:
        return NAN
    lo = math.ceil(q * len(sorted_vals))
    lo = min(max(lo, 1), len(sorted_vals))
    return sorted_vals[lo - 1]


@dataclass
class TimingStats:
    p50_us: float = NAN
    p30_us: float = NAN
    min_us: float = NAN
    mean_us: float = NAN
    n: int = 0


def summarize(samples: Sequence[float]) -> TimingStats:
    if not samples:
        return TimingStats()
    s = sorted(samples)
    return TimingStats(percentile(s, 0.5), percentile(s, 0.3), s[0], sum(s) / len(s), len(s))


def modeled_bytes(n: int, k: int, m: int) -> float:
    return float(n) * k + float(m) * k + 2.0 * m * n


@dataclass
class CsvRow:
    model: str = ""
    N: int = 0
    K: int = 0
    M: int = 0
    m_tile: int = 0
    step: int = -1
    step_name: str = ""
    protocol: str = ""
    p50: float = NAN
    p30: float = NAN
    bw: float = NAN
    pct: float = NAN
    clocks_mhz: int = -1
    rel_l2: float = NAN
    passed: str = "na"
    config: str = ""
    min_us: float = NAN
    mean_us: float = NAN
    samples: int = 0
    reps: int = 0
    iso_samples: int = 0
    b2b_batch: int = 0
    pdl_batch: int = 0
    kind: str = "canonical"
    tune_index: int = -1
    rank: int = -1
    is_best: bool = False
    padded_n: int = 0
    weight_sets: int = 0
    weight_set_bytes: int = 0
    smem_bytes: int = 0
    num_ctas: int = 0
    num_threads: int = 0
    mechanism: str = ""
    rel_l2_launcher: float = NAN

    def fill_stats(self, protocol: str, st: TimingStats) -> None:
        """bench/bench_decode.cu:1685-1700."""
        self.protocol = protocol
        self.p50, self.p30, self.min_us, self.mean_us, self.samples = st.p50_us, st.p30_us, st.min_us, \
            st.mean_us, st.n
        if _finite(st.p50_us) and st.p50_us > 0:
            self.bw = modeled_bytes(self.N, self.K, self.M) / (st.p50_us * 1e-6) / 1e9
            self.pct = self.bw / SPEC_PEAK_GBPS


def row_main(r: CsvRow) -> str:
    return ",".join([csv_field(r.model), str(r.N), str(r.K), str(r.M), str(r.m_tile), str(r.step),
                     csv_field(r.step_name), r.protocol, f4(r.p50), f4(r.p30), f3(r.bw), f6(r.pct),
                     str(r.clocks_mhz), fe6(r.rel_l2), csv_field(r.passed), csv_field(r.config)])


def row_detail(r: CsvRow) -> str:
    return ",".join([row_main(r), f4(r.min_us), f4(r.mean_us), str(r.samples), str(r.reps), str(r.iso_samples),
                     str(r.b2b_batch), str(r.pdl_batch), csv_field(r.kind), str(r.tune_index), str(r.rank),
                     "1" if r.is_best else "0", str(r.padded_n), str(r.weight_sets), str(r.weight_set_bytes),
                     str(r.smem_bytes), str(r.num_ctas), str(r.num_threads), csv_field(r.mechanism),
                     fe6(r.rel_l2_launcher)])


def row_tune_best(r: CsvRow, rank_protocol: str) -> str:
    return ",".join([csv_field(r.model), str(r.N), str(r.K), str(r.M), str(r.m_tile), str(r.step),
                     csv_field(r.step_name), str(r.rank), "1" if r.is_best else "0", rank_protocol, f4(r.p50),
                     f4(r.p30), f3(r.bw), f6(r.pct), str(r.clocks_mhz), fe6(r.rel_l2), csv_field(r.passed),
                     csv_field(r.config), str(r.smem_bytes), str(r.num_ctas), str(r.weight_sets)])


def split_csv_line(line: str) -> List[str]:
    """RFC-4180 fields of one line; CR/LF stripped (bench/bench_decode.cu:1271-1300)."""
    line = line.rstrip("\r\n")
    out, cur, quoted, i = [], [], False, 0
    while i < len(line):
        c = line[i]
        if quoted:
            if c == '"':
                if i + 1 < len(line) and line[i + 1] == '"':
                    cur.append('"')
                    i += 1
                else:
                    quoted = False
            else:
                cur.append(c)
        elif c == '"':
            quoted = True
        elif c == ",":
            out.append("".join(cur))
            cur = []
        else:
            cur.append(c)
        i += 1
    out.append("".join(cur))
    return out


class CsvWriter:
    """Header on a new file, or append to an existing one; every row flushed."""

    def __init__(self, path: str, header: str, append: bool = False):
        self.path = path
        self.rows = 0
        exists = append and os.path.exists(path) and os.path.getsize(path) > 0
        if exists:
            with open(path) as f:
                self.rows = max(0, sum(1 for ln in f if ln.strip()) - 1)
        self._f = open(path, "a" if exists else "w")
        if not exists:
            self._f.write(header + "\n")
            self._f.flush()

    def write(self, line: str) -> None:
        self._f.write(line + "\n")
        self._f.flush()
        self.rows += 1

    def close(self) -> None:
        self._f.close()


class DoneSet:
    """Rows already measured (bench/bench_decode.cu:1302-1369): keyed by
    (kind, model, N, K, M, m_tile, step, protocol, config); rows whose p50 is
    not a number do not count."""

    NEED = ("model", "N", "K", "M", "m_tile", "step", "protocol", "latency_us_p50")

    def __init__(self):
        self.keys = set()
        self.rows = 0

    @staticmethod
    def key(is_tune: bool, r: CsvRow) -> tuple:
        return ("T" if is_tune else "C", r.model, r.N, r.K, r.M, r.m_tile, r.step, r.protocol, r.config)

    def has(self, is_tune: bool, r: CsvRow) -> bool:
        return self.key(is_tune, r) in self.keys

    def add(self, is_tune: bool, r: CsvRow) -> None:
        self.keys.add(self.key(is_tune, r))

    def load(self, path: str, is_tune: bool) -> bool:
        try:
            with open(path) as f:
                lines = f.read().splitlines()
        except OSError:
            return False
        if not lines:
            return False
        hdr = split_csv_line(lines[0])
        col = {h: i for i, h in enumerate(hdr)}
        if any(c not in col for c in self.NEED):
            return False
        for ln in lines[1:]:
            if not ln.strip():
                continue
            f = split_csv_line(ln)
            if len(f) < len(hdr):
                continue
            lat = f[col["latency_us_p50"]]
            if lat in ("", "nan", "NaN"):
                continue
            r = CsvRow(model=f[col["model"]], N=_atoi(f[col["N"]]), K=_atoi(f[col["K"]]), M=_atoi(f[col["M"]]),
                       m_tile=_atoi(f[col["m_tile"]]), step=_atoi(f[col["step"]]), protocol=f[col["protocol"]],
                       config=f[col["config"]] if "config" in col else "")
            self.add(is_tune, r)
            self.rows += 1
        return True


def purge_incomplete_groups(path: str, protocols: Sequence[str]) -> Tuple[int, int, int]:
    """Drop every group (model, N, K, M, m_tile, step, config) that lacks a
    valid-latency row for one of `protocols` (bench/bench_decode.cu:1371-1476);
    the file is rewritten through a temporary and a rename.  Returns (kept,
    dropped rows, dropped groups)."""
    need = set(protocols) or set(PROTOCOLS)
    try:
        with open(path) as f:
            lines = f.read().splitlines()
    except OSError:
        return 0, 0, 0
    if not lines:
        return 0, 0, 0
    hdr = split_csv_line(lines[0])
    col = {h: i for i, h in enumerate(hdr)}
    gcols = [c for c in ("model", "N", "K", "M", "m_tile", "step", "config") if c in col]
    if "protocol" not in col or "latency_us_p50" not in col:
        return len(lines) - 1, 0, 0
    rows = [(ln, split_csv_line(ln)) for ln in lines[1:] if ln.strip()]
    have: Dict[tuple, set] = {}
    for _, f in rows:
        if len(f) < len(hdr):
            continue
        g = tuple(f[col[c]] for c in gcols)
        if f[col["latency_us_p50"]] not in ("", "nan", "NaN"):
            have.setdefault(g, set()).add(f[col["protocol"]])
    keep, dropped, bad_groups = [], 0, set()
    for ln, f in rows:
        g = tuple(f[col[c]] for c in gcols) if len(f) >= len(hdr) else None
        if g is not None and need <= have.get(g, set()):
            keep.append(ln)
        else:
            dropped += 1
            bad_groups.add(g)
    if dropped:
        tmp = path + ".tmp"
        with open(tmp, "w") as f:
            f.write(lines[0] + "\n")
            for ln in keep:
                f.write(ln + "\n")
        os.replace(tmp, path)
    return len(keep), dropped, len(bad_groups)


def newest_csv(directory: str, prefix: str) -> Optional[str]:
    """Newest `<prefix><UTC stamp>.csv` in `directory` (sidecars excluded)."""
    try:
        names = [n for n in os.listdir(directory)
                 if n.startswith(prefix) and n.endswith(".csv") and not n.endswith("_detail.csv")
                 and not n.startswith(prefix + "best")]
    except OSError:
        return None
    return os.path.join(directory, max(names)) if names else None


def json_backend_of(csv_path: str) -> Optional[str]:
    try:
        with open(os.path.splitext(csv_path)[0] + ".json") as f:
            return json.load(f).get("kernel_backend")
    except (OSError, ValueError):
        return None


class CsvLock:
    """An exclusive advisory lock on `<csv>.lock`, so two runs never append
    to one file (bench/bench_decode.cu:1478-1489)."""

    def __init__(self, csv_path: str):
        self.path = csv_path + ".lock"
        self._f = None

    def acquire(self) -> bool:
        self._f = open(self.path, "w")
        try:
            fcntl.flock(self._f, fcntl.LOCK_EX | fcntl.LOCK_NB)
        except OSError:
            self._f.close()
            self._f = None
            return False
        return True

    def release(self) -> None:
        if self._f is not None:
            fcntl.flock(self._f, fcntl.LOCK_UN)
            self._f.close()
            self._f = None
            try:
                os.unlink(self.path)
            except OSError:
                pass


def utc_stamp() -> str:
    return datetime.now(timezone.utc).strftime("%Y%m%dT%H%M%SZ")


def detail_path_of(csv_path: str) -> str:
    return os.path.splitext(csv_path)[0] + "_detail.csv"


# ---------------------------------------------------------------------------
# Device side
# ---------------------------------------------------------------------------

def block_quantize(x, rows_per_block: int):
    """[R, K] fp32 -> (e4m3 bits uint8 [R, K], fp32 scales [ceil(R/rpb), K/128]):
    scale = max(amax, 1e-4)/448 per rows_per_block x 128 block, q = e4m3(clamp(
    v/scale, +-448)) (bench/bench_decode.cu:397-470)."""
    import torch
    r, k = x.shape
    kb = k // K_BLOCK
    rb = -(-r // rows_per_block)
    pad = rb * rows_per_block - r
    xp = torch.nn.functional.pad(x, (0, 0, 0, pad)) if pad else x
    blocks = xp.view(rb, rows_per_block, kb, K_BLOCK)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.clamp(amax, min=QUANT_EPS) / FP8_MAX
    q = torch.clamp(blocks / scale[:, None, :, None], -FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn)
    q = q.view(torch.uint8).reshape(rb * rows_per_block, k)[:r].contiguous()
    return q, scale.contiguous()


def dequantize(q, scales, rows_per_block: int):
    import torch
    r, k = q.shape
    s = scales.repeat_interleave(rows_per_block, dim=0)[:r].repeat_interleave(K_BLOCK, dim=1)
    return q.view(torch.float8_e4m3fn).float() * s


class ModelData:
    """One model's weights on the device: e4m3 [n_ker, K] (N padded to 128 rows,
    bench/bench_decode.cu:404-407), 128x128 scales with one spare row, and the
    fp32 dequantised copy the reference products use."""

    def __init__(self, shape: ModelShape, seed: int, dev, with_reference: bool):
        import torch
        self.shape = shape
        self.n_log, self.k = shape.N, shape.K
        self.n_ker = -(-shape.N // 128) * 128
        g = torch.Generator(device=dev).manual_seed(seed)
        w = torch.randn((self.n_ker, self.k), generator=g, device=dev) * (1.0 / math.sqrt(self.k))
        if self.n_ker > self.n_log:
            w[self.n_log:] = 0
        self.q, s = block_quantize(w, 128)
        del w
        self.scales = torch.cat([s, torch.zeros((1, s.shape[1]), device=dev)]).contiguous()
        self.deq = dequantize(self.q, s, 128) if with_reference else None


class ActData:
    def __init__(self, m: int, k: int, seed: int, dev):
        import torch
        g = torch.Generator(device=dev).manual_seed(seed)
        a = torch.randn((m, k), generator=g, device=dev) * (1.0 / math.sqrt(k))
        self.q, self.scales = block_quantize(a, 1)
        self.m = m


class WeightCache:
    """Cold-rotation copies of one model's weights per (layout, block_n),
    least-recently-used evicted over `budget` bytes (bench/bench_decode.cu:803-859)."""

    def __init__(self, budget_bytes: int, l2_bytes: int):
        self.budget = budget_bytes
        self.l2 = l2_bytes
        self.groups: Dict[tuple, list] = {}
        self.order: List[tuple] = []

    def sets_for(self, set_bytes: int) -> int:
        return max(5, math.ceil(max(1 << 30, 4 * self.l2) / set_bytes))

    def get(self, md: ModelData, layout: int, block_n: int):
        import torch
        import decode_opt_b200 as dg
        key = (md.shape.id, layout, block_n if layout != dg.LAYOUT_RAW else 0)
        if key in self.groups:
            self.order.remove(key)
            self.order.append(key)
            return self.groups[key]
        base = md.q if layout == dg.LAYOUT_RAW else dg.prepack_weight(md.q, block_n, layout)
        n = self.sets_for(base.numel())
        need = n * base.numel()
        while self.order and self._bytes() + need > self.budget:
            self.groups.pop(self.order.pop(0))
            torch.cuda.empty_cache()
        sets = [base] + [base.clone() for _ in range(n - 1)]
        self.groups[key] = sets
        self.order.append(key)
        return sets

    def _bytes(self) -> int:
        return sum(len(v) * v[0].numel() for v in self.groups.values())

    def drop_model(self, model_id: str) -> None:
        for key in [k for k in self.order if k[0] == model_id]:
            self.order.remove(key)
            self.groups.pop(key)


@dataclass
class PointResult:
    stats: Dict[str, TimingStats] = field(default_factory=dict)
    clocks: Dict[str, int] = field(default_factory=dict)
    rel_l2: float = NAN
    passed: str = "na"
    rel_l2_launcher: float = NAN
    padded_n: int = 0
    weight_sets: int = 0
    set_bytes: int = 0
    smem: int = 0
    ctas: int = 0
    threads: int = 0
    mechanism: str = ""
    skip: str = ""
    rows: list = field(default_factory=list)


class Session:
    """Device state of one run: stream, L2 flush buffer, clock sampler,
    weight cache."""

    def __init__(self, o: Options):
        import torch
        import decode_opt_b200 as dg
        from .clocks import ClockSampler
        self.o = o
        self.dg = dg
        self.torch = torch
        self.dev = torch.device("cuda", torch.cuda.current_device())
        props = torch.cuda.get_device_properties(self.dev)
        self.props = props
        self.sms = props.multi_processor_count
        self.stream = torch.cuda.Stream(device=self.dev)
        self.flush_buf = torch.empty(o.l2_flush_mb << 20, dtype=torch.uint8, device=self.dev)
        self.clock = ClockSampler(self.dev.index or 0)
        self.clock.start()
        self.cache = WeightCache(int(o.weight_cache_gb * (1 << 30)), props.L2_cache_size)
        torch.backends.cuda.matmul.allow_tf32 = False

    def close(self):
        self.clock.stop()

    # ---- one configuration ------------------------------------------------
    def measure(self, md: ModelData, ad: ActData, ref, b200, protocols: Sequence[str], plan: TimingPlan,
                with_corr: bool, emit) -> PointResult:
        """Set up, check and time one configuration.  `b200` is a
        B200Config; `emit(protocol, stats, result)` is called after each
        protocol so a killed run keeps what it measured."""
        torch, dg = self.torch, self.dg
        res = PointResult()
        m, n, k = ad.m, md.n_ker, md.k
        lp = b200.plan(m, n, k)
        if lp.error:
            res.skip = lp.error
            return res
        res.padded_n, res.smem, res.ctas, res.threads = lp.padded_n, lp.smem_bytes, lp.num_ctas, lp.block[0]
        res.mechanism = "launch" if self.o.force_api_launch else "launch_with_maps"
        sets = self.cache.get(md, b200.layout, b200.packed_rows)
        res.weight_sets, res.set_bytes = len(sets), sets[0].numel()
        out = torch.empty((m, n), dtype=torch.bfloat16, device=self.dev)
        ws = torch.zeros(max(lp.ws_floats, 1), dtype=torch.float32, device=self.dev)
        sem = torch.zeros(max(lp.sem_ints, 1), dtype=torch.int32, device=self.dev)
        status = torch.zeros(1, dtype=torch.int32, device=self.dev)
        probs = [dg.Problem(m, n, k, ad.q, w, md.scales, ad.scales, out, ws, sem, status) for w in sets]
        wmaps = [dg.make_weight_tma(b200, p) for p in probs]
        amap = dg.make_activation_tma(b200, probs[0])
        # inputs, prepacked copies and zeroed buffers come from the current
        # stream; the launches below go to self.stream
        torch.cuda.synchronize(self.dev)
        s = self.stream
        api = self.o.force_api_launch

        def launch(i: int, pdl_attr: bool) -> None:
            j = i % len(sets)
            if api:
                cfg = b200 if b200.pdl == pdl_attr else type(b200)(**{**b200.__dict__, "pdl": pdl_attr})
                rc = dg.launch(cfg, probs[j], s)
            else:
                rc = dg.launch_with_maps(b200, probs[j], wmaps[j], amap, s, pdl_attr=pdl_attr)
            if rc != 0:
                raise RuntimeError(f"launch failed: cudaError {rc}")

        with torch.cuda.stream(s):
            for i in range(WARMUP_LAUNCHES):
                launch(i, False)
        s.synchronize()
        self._check_status(status, sem)
        if with_corr and ref is not None:
            res.rel_l2, ok = self._check(out, ref, lambda: launch(0, False))
            res.passed = "1" if ok else "0"
            if self.o.check_launcher:
                res.rel_l2_launcher, _ = self._check(
                    out, ref, lambda: self._api_launch(b200, probs[0], s))
        for proto in protocols:
            t0 = time.perf_counter()
            if proto == "ISO":
                st = self._time_iso(launch, plan)
            else:
                st = self._time_batch(launch, plan, proto == "PDL")
            t1 = time.perf_counter()
            self._check_status(status, sem)
            res.stats[proto] = st
            mhz = self.clock.median_between(t0, t1)
            res.clocks[proto] = int(round(mhz)) if mhz is not None else -1
            emit(proto, st, res)
        return res

    def _api_launch(self, b200, p, s):
        rc = self.dg.launch(b200, p, s)
        if rc != 0:
            raise RuntimeError(f"launch failed: cudaError {rc}")

    def _check(self, out, ref, run) -> Tuple[float, bool]:
        torch = self.torch
        with torch.cuda.stream(self.stream):
            out.zero_()
            run()
        self.stream.synchronize()
        got = out[:, :ref.shape[1]].float()
        finite = bool(torch.isfinite(got).all()) and bool(torch.isfinite(ref).all())
        err = float(torch.linalg.vector_norm((got - ref).double()))
        energy = max(float(torch.linalg.vector_norm(ref.double())) ** 2, 1e-30)
        rel = err / math.sqrt(energy)
        return rel, finite and rel <= REL_L2_THRESHOLD and got.numel() > 0

    def _check_status(self, status, sem) -> None:
        st = int(status.item())
        if st != 0:
            status.zero_()
            sem.zero_()
            raise RuntimeError(f"kernel status {self.dg.status_string(st)}")

    def _time_iso(self, launch, plan: TimingPlan) -> TimingStats:
        """One launch after an L2-flushing write; the flush stays queued ahead
        of the start event, so host submission is not timed."""
        torch, s = self.torch, self.stream
        samples = []
        idx = 0
        for _ in range(plan.reps):
            for _ in range(plan.iso_samples):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(s):
                    self.dg.flush_l2(self.flush_buf, s)
                    e0.record(s)
                    launch(idx, False)
                    e1.record(s)
                e1.synchronize()
                samples.append(e0.elapsed_time(e1) * 1e3)
                idx += 1
        return summarize(samples)

    def _time_batch(self, launch, plan: TimingPlan, pdl_attr: bool) -> TimingStats:
        """`batch` launches captured in one CUDA graph; per rep one replay
        timed by events, microseconds per launch."""
        torch, s = self.torch, self.stream
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for i in range(plan.batch):
                    launch(i, pdl_attr)
            graph.replay()
        s.synchronize()
        per = []
        for _ in range(plan.reps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(s):
                e0.record(s)
                graph.replay()
                e1.record(s)
            e1.synchronize()
            per.append(e0.elapsed_time(e1) * 1e3 / plan.batch)
        del graph
        return summarize(per)


# ---------------------------------------------------------------------------
# Driver
# ---------------------------------------------------------------------------

def canonical_variants(step: int, m: int, n: int, k: int, sms: int) -> StepVariant:
    mt = m_tile_for(m)
    if step in (STEP_B200, STEP_B200_INDEP):
        return StepVariant(step, mt, b200=b200_step_config(m, n, k, independent=step == STEP_B200_INDEP))
    return StepVariant(step, mt, kernel_config=canonical_kernel_config(step, mt, n, k, m, sms))


def resolve(v: StepVariant, m: int, n: int, k: int):
    """(B200Config to launch, config column)."""
    import decode_opt_b200 as dg
    if v.kernel_config is not None:
        kc = v.kernel_config
        b = kc._fitted(m, n, k)
        return b, f"{config_string(kc)};STAGES_SM100={b.stages}"
    b = dg.B200Config(**v.b200)
    return b, b200_config_string(v.b200)


def print_list(o: Options, models: Sequence[ModelShape], note: str, sms: int = 148) -> None:
    print(f"models ({len(models)}, from {note}):")
    for m in models:
        print(f"  {m.id:<18s} N={m.N:<6d} K={m.K:<6d} hidden={m.hidden:<5d} bm={choose_bm(m.N):<3d} "
              f"layer={m.layer}")
    print(f"steps: {', '.join(f'S{i} {n}' for i, n in enumerate(STEP_NAMES))}")
    for m in models[:1]:
        for mt in (8, 16, 32, 64, 128):
            print(f"  {m.id} M_TILE={mt}:")
            for step in range(6):
                kc = canonical_kernel_config(step, mt, m.N, m.K, mt, sms)
                print(f"    S{step} {STEP_NAMES[step]:<11s} {config_string(kc)}")
    print(f"tune grid: BN {TUNE_BLOCK_N} x SUBS {TUNE_SUBS} x STAGES {TUNE_STAGES} x GRID tiles/streamk/cluster = "
          f"{len(TUNE_BLOCK_N) * len(TUNE_SUBS) * len(TUNE_STAGES) * len(TUNE_GRIDS)} configurations")


class Run:
    """Writers, resume state and counters of one invocation."""

    def __init__(self, o: Options):
        self.o = o
        self.protocols = wanted_protocols(o)
        self.skipped: List[dict] = []
        self.best: Dict[tuple, dict] = {}
        self.rows_written = 0
        self.rows_resumed = 0
        self.points_resumed = 0
        self.tune_best_rows = 0
        self.done = DoneSet()
        self.append = False
        self.resume_note = "disabled"
        self.lock = None
        os.makedirs(o.out_dir, exist_ok=True)
        ts = utc_stamp()
        self.csv_path = os.path.join(o.out_dir, f"bench_{ts}.csv")
        if o.resume:
            self._resume()
        self.detail_path = detail_path_of(self.csv_path)
        self.json_path = os.path.splitext(self.csv_path)[0] + ".json"
        if self.lock is None:
            self.lock = CsvLock(self.csv_path)
            if not self.lock.acquire():
                raise SystemExit(f"[bench_decode] {self.csv_path} is being written by another process")
        self.csv = CsvWriter(self.csv_path, CSV_HEADER, self.append)
        self.detail = CsvWriter(self.detail_path, DETAIL_HEADER, self.append)
        self.extra: Dict[str, CsvWriter] = {}
        self.tune_path = ""
        if o.tune:
            self.tune_path = o.tune_out or os.path.join(o.out_dir, f"tune_{ts}.csv")
            tune_append = o.resume and os.path.exists(self.tune_path)
            if tune_append:
                purge_incomplete_groups(self.tune_path, self.protocols)
                purge_incomplete_groups(detail_path_of(self.tune_path), self.protocols)
                self.done.load(self.tune_path, True)
            self.tune_csv = CsvWriter(self.tune_path, CSV_HEADER, tune_append)
            self.tune_detail = CsvWriter(detail_path_of(self.tune_path), DETAIL_HEADER, tune_append)
            self.tune_best_path = os.path.splitext(self.tune_path)[0] + "_best.csv"
            self.tune_best = CsvWriter(self.tune_best_path, TUNE_BEST_HEADER, False)

    def _resume(self) -> None:
        o = self.o
        src = o.resume_path or newest_csv(o.out_dir, "bench_")
        if not src or not os.path.exists(src):
            self.resume_note = f"requested, but there is no bench_*.csv in {o.out_dir}"
            return
        backend = json_backend_of(src)
        if backend is not None and backend != KERNEL_BACKEND:
            self.resume_note = f"refused: {src} was written by kernel_backend={backend}"
            print(f"[bench_decode] resume {self.resume_note}", file=sys.stderr)
            return
        lock = CsvLock(src)
        if not lock.acquire():
            self.resume_note = f"refused: {src} is being written by another process"
            print(f"[bench_decode] resume {self.resume_note}", file=sys.stderr)
            return
        kept, dropped, groups = purge_incomplete_groups(src, self.protocols)
        purge_incomplete_groups(detail_path_of(src), self.protocols)
        if not self.done.load(src, False):
            lock.release()
            self.resume_note = f"cannot parse {src}"
            return
        self.lock = lock
        self.csv_path = src
        self.append = True
        self.resume_note = f"appending to {src} ({kept} rows kept, {dropped} rows of {groups} incomplete groups dropped)"

    def writer(self, kind: str, path_opt: str, default_name: str, header: str) -> CsvWriter:
        if kind not in self.extra:
            path = path_opt or os.path.join(self.o.out_dir, default_name)
            self.extra[kind] = CsvWriter(path, header, self.o.resume and os.path.exists(path))
        return self.extra[kind]

    def close(self) -> None:
        self.csv.close()
        self.detail.close()
        for w in self.extra.values():
            w.close()
        if self.o.tune:
            self.tune_csv.close()
            self.tune_detail.close()
            self.tune_best.close()
        if self.lock is not None:
            self.lock.release()


def base_row(shape: ModelShape, m: int, v: StepVariant, config: str, plan: TimingPlan) -> CsvRow:
    return CsvRow(model=shape.id, N=shape.N, K=shape.K, M=m, m_tile=v.m_tile, step=v.step,
                  step_name=v.step_name, config=config, reps=plan.reps, iso_samples=plan.iso_samples,
                  b2b_batch=plan.batch, pdl_batch=plan.batch, kind=v.kind, tune_index=v.tune_index)


def run_point(run: Run, sess: Session, md: ModelData, ad: ActData, ref, v: StepVariant, plan: TimingPlan,
              is_tune: bool, sink=None, suffix: Optional[str] = None) -> Optional[PointResult]:
    """Measure one variant and write its rows (main + detail, or `sink` with
    the extra column `suffix`).  Rows already in the resume set are skipped."""
    shape = md.shape
    b200, cfg_str = resolve(v, ad.m, md.n_ker, md.k)
    proto = []
    for p in run.protocols:
        probe = base_row(shape, ad.m, v, cfg_str, plan)
        probe.protocol = p
        if sink is None and run.done.has(is_tune, probe):
            run.rows_resumed += 1
            continue
        proto.append(p)
    if not proto:
        run.points_resumed += 1
        return None
    rows: List[CsvRow] = []

    def emit(p: str, st: TimingStats, res: PointResult) -> None:
        r = base_row(shape, ad.m, v, cfg_str, plan)
        r.fill_stats(p, st)
        r.rel_l2, r.passed, r.rel_l2_launcher = res.rel_l2, res.passed, res.rel_l2_launcher
        r.clocks_mhz = res.clocks.get(p, -1)
        r.padded_n, r.weight_sets, r.weight_set_bytes = res.padded_n, res.weight_sets, res.set_bytes
        r.smem_bytes, r.num_ctas, r.num_threads, r.mechanism = res.smem, res.ctas, res.threads, res.mechanism
        rows.append(r)
        if sink is not None:
            sink.write(f"{row_main(r)},{csv_field(suffix or '')}")
        elif is_tune:
            run.tune_csv.write(row_main(r))
            run.tune_detail.write(row_detail(r))
        else:
            run.csv.write(row_main(r))
            run.detail.write(row_detail(r))
        run.rows_written += 1
        if run.o.verbose or not is_tune:
            print(f"[bench_decode] {shape.id:<16s} M={ad.m:<3d} S{v.step} {v.step_name:<12s} {p:<3s} "
                  f"p50={f4(r.p50)} us  {f3(r.bw)} GB/s  rel_l2={fe6(r.rel_l2)} pass={r.passed}"
                  + (f"  [{suffix}]" if suffix else ""), flush=True)

    try:
        res = sess.measure(md, ad, ref, b200, proto, plan, not run.o.no_correctness, emit)
    except RuntimeError as e:
        run.skipped.append({"model": shape.id, "step": v.step, "M": ad.m, "m_tile": v.m_tile,
                            "config": cfg_str, "reason": str(e)})
        print(f"[bench_decode] skip {shape.id} M={ad.m} S{v.step} {cfg_str}: {e}", file=sys.stderr)
        return None
    if res.skip:
        run.skipped.append({"model": shape.id, "step": v.step, "M": ad.m, "m_tile": v.m_tile,
                            "config": cfg_str, "reason": res.skip})
        return None
    res.rows = rows
    if not is_tune and sink is None:
        for r in rows:
            key = (shape.id, ad.m, r.protocol)
            if _finite(r.bw) and r.passed != "0" and r.bw > run.best.get(key, {}).get("bandwidth_gbps", -1.0):
                run.best[key] = {"model": shape.id, "M": ad.m, "protocol": r.protocol, "step": r.step,
                                 "step_name": r.step_name, "latency_us_p50": r.p50, "bandwidth_gbps": r.bw,
                                 "pct_of_spec_peak": r.pct, "config": r.config}
    return res


def run_tune(run: Run, sess: Session, md: ModelData, ad: ActData, ref, plan: TimingPlan) -> None:
    rank_protocol = "PDL" if "PDL" in run.protocols else ("B2B" if "B2B" in run.protocols else "ISO")
    ranked = []
    for idx, cfg in enumerate(tune_grid(ad.m)):
        v = StepVariant(STEP_B200, m_tile_for(ad.m), b200=cfg, kind="tune", tune_index=idx)
        res = run_point(run, sess, md, ad, ref, v, plan, True)
        if res is None:
            continue
        for r in res.rows:
            if r.protocol == rank_protocol and r.passed != "0" and _finite(r.p50):
                ranked.append(r)
    ranked.sort(key=lambda r: r.p50)
    for i, r in enumerate(ranked):
        r.rank = i + 1
        r.is_best = i == 0
        run.tune_best.write(row_tune_best(r, rank_protocol))
        run.tune_best_rows += 1
    if ranked:
        b = ranked[0]
        print(f"[bench_decode] tune best {md.shape.id} M={ad.m}: {f4(b.p50)} us {f3(b.bw)} GB/s {b.config}",
              flush=True)


def env_info(sess) -> dict:
    import torch
    p = sess.props
    info = {"device_name": p.name, "sm_count": p.multi_processor_count, "l2_bytes": p.L2_cache_size,
            "mem_total_bytes": p.total_memory, "torch": torch.__version__, "cuda": torch.version.cuda,
            "cuda_visible_devices": os.environ.get("CUDA_VISIBLE_DEVICES", ""),
            "clock_sm_max_mhz": sess.clock.max_mhz}
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(sess.dev.index or 0)
        procs = pynvml.nvmlDeviceGetComputeRunningProcesses(h)
        others = [int(x.pid) for x in procs if int(x.pid) != os.getpid()]
        info["driver"] = pynvml.nvmlSystemGetDriverVersion()
        info["other_compute_pids"] = others
        info["exclusive_verdict"] = "exclusive" if not others else "shared-or-namespaced"
    except Exception as e:  # noqa: BLE001 - NVML missing
        info["exclusive_verdict"] = f"unknown ({type(e).__name__})"
    return info


def write_summary(run: Run, sess: Session, models, model_note: str, started: float) -> None:
    o = run.o
    doc = {
        "kernel_backend": KERNEL_BACKEND,
        "tool": "decode_opt_b200.bench_decode",
        "started_utc": datetime.fromtimestamp(started, timezone.utc).isoformat(),
        "elapsed_s": time.time() - started,
        "env": env_info(sess),
        "models": [m.__dict__ for m in models],
        "models_source": model_note,
        "options": {k: v for k, v in o.__dict__.items()},
        "protocols": run.protocols,
        "timing": {"warmup_launches": WARMUP_LAUNCHES, "big_k_auto_scale": f"K>={BIG_K}: iso 20, batch 50",
                   "batch_launch": "one CUDA graph per protocol and point, replayed per rep",
                   "iso": f"{o.l2_flush_mb} MB L2-flushing write queued before the start event",
                   "percentiles": "ceil(q*n)-th smallest"},
        "spec_peak_gbps": SPEC_PEAK_GBPS,
        "correctness": {"reference": "fp32 torch matmul of the dequantised operands (TF32 off)",
                        "threshold_rel_l2": REL_L2_THRESHOLD},
        "csv_columns": CSV_HEADER,
        "detail_sidecar_columns": DETAIL_HEADER,
        "outputs": {"csv": run.csv_path, "detail_csv": run.detail_path, "summary": run.json_path,
                    "tune_csv": run.tune_path, "extra": {k: w.path for k, w in run.extra.items()}},
        "rows_written": run.rows_written,
        "rows_resumed": run.rows_resumed,
        "points_resumed": run.points_resumed,
        "resume": run.resume_note,
        "best": sorted(run.best.values(), key=lambda b: (b["model"], b["M"], b["protocol"])),
        "skipped": run.skipped,
    }
    with open(run.json_path, "w") as f:
        json.dump(doc, f, indent=2, default=str)


def main(argv: Optional[Sequence[str]] = None) -> int:
    o = parse_args(sys.argv[1:] if argv is None else argv)
    all_models, note = load_models(o.models_json or None)
    models, missing = select_models(all_models, o.models)
    for w in missing:
        print(f"[bench_decode] WARNING: model {w} is not in the table; skipped", file=sys.stderr)
    if o.demo:
        models = models[:1]
    if not models:
        print("[bench_decode] no models to run", file=sys.stderr)
        return 2
    if o.purge_only:
        kept, dropped, groups = purge_incomplete_groups(o.purge_only, wanted_protocols(o))
        print(f"[bench_decode] purge {o.purge_only}: kept {kept}, dropped {dropped} rows of {groups} groups")
        return 0
    if o.list_only:
        print_list(o, models, note)
        return 0
    import torch
    if not torch.cuda.is_available():
        print("[bench_decode] no CUDA device", file=sys.stderr)
        return 2
    started = time.time()
    sess = Session(o)
    run = Run(o)
    if o.resume:
        print(f"[bench_decode] resume: {run.resume_note} ({run.done.rows} rows measured)")
    env = env_info(sess)
    if env.get("other_compute_pids") and not o.allow_shared:
        print(f"[bench_decode] WARNING: other compute processes on the GPU: {env['other_compute_pids']} "
              "(numbers may be disturbed; pass --allow-shared to silence)", file=sys.stderr)
    print(f"[bench_decode] {env['device_name']} SMs={sess.sms} -> {run.csv_path}", flush=True)
    try:
        for mi, shape in enumerate(models):
            plan = plan_for(shape.K, o)
            md = ModelData(shape, o.seed + 1000003 * (mi + 1), sess.dev, not o.no_correctness)
            for m in o.ms:
                ad = ActData(m, shape.K, o.seed + 7 * m + 13 * mi, sess.dev)
                ref = None
                if not o.no_correctness:
                    deq_a = dequantize(ad.q, ad.scales, 1)
                    ref = (deq_a @ md.deq.t())[:, :shape.N].contiguous()
                    del deq_a
                if not o.tune_only:
                    for step in o.steps:
                        v = canonical_variants(step, m, md.n_ker, shape.K, sess.sms)
                        run_point(run, sess, md, ad, ref, v, plan, False)
                        extra_runs(run, sess, md, ad, ref, v, plan)
                if o.tune:
                    run_tune(run, sess, md, ad, ref, plan)
                del ref
            sess.cache.drop_model(shape.id)
            del md
            torch.cuda.empty_cache()
    finally:
        write_summary(run, sess, models, note, started)
        run.close()
        sess.close()
    print(f"[bench_decode] wrote {run.rows_written} rows to {run.csv_path} (+ {run.detail_path}, {run.json_path});"
          f" {len(run.skipped)} skipped")
    return 0


def extra_runs(run: Run, sess: Session, md: ModelData, ad: ActData, ref, v: StepVariant, plan: TimingPlan):
    """The ablations attached to a ladder step (bench/bench_decode.cu:2380-2560)."""
    import decode_opt_b200 as dg
    o = run.o
    mt = v.m_tile
    n, k, m = md.n_ker, md.k, ad.m
    if o.splitk_ablation and v.step == 5:
        w = run.writer("splitk_ablation", o.ablation_out, "ablation_splitk.csv", ABLATION_HEADER)
        for on in (False, True):
            kc = canonical_kernel_config(5, mt, n, k, m, sess.sms, splitk=2 if on else 1)
            label = "1" if kc.kSplitKCta else "0"
            if on and not kc.kSplitKCta:
                run.skipped.append({"model": md.shape.id, "step": 5, "M": m, "m_tile": mt,
                                    "reason": "split-K ablation: K not divisible for S=2"})
                continue
            run_point(run, sess, md, ad, ref, StepVariant(5, mt, kernel_config=kc, kind="ablation"), plan, False,
                      sink=w, suffix=label)
    if o.splitk_factor_sweep and v.step == 5:
        w = run.writer("splitk_factor", o.factor_out, "splitk_factor_sweep.csv", FACTOR_HEADER)
        for f in o.splitk_factors:
            kc = canonical_kernel_config(5, mt, n, k, m, sess.sms, splitk=f)
            if kc.kSplitKFactor != f:
                run.skipped.append({"model": md.shape.id, "step": 5, "M": m, "m_tile": mt,
                                    "reason": f"split-K factor {f}: K not divisible"})
                continue
            run_point(run, sess, md, ad, ref, StepVariant(5, mt, kernel_config=kc, kind="factor"), plan, False,
                      sink=w, suffix=str(f))
    if o.pdl_placement and v.step in (4, STEP_B200):
        w = run.writer("pdl_placement", o.ablation_out, "ablation_pdl_placement.csv", PLACEMENT_HEADER)
        b, _ = resolve(v, m, n, k)
        base = dict(b.__dict__)
        variants = (("producer", dict(base, pdl=True, flags=base["flags"] & ~dg.FLAG_INDEPENDENT_INPUTS)),
                    ("producer_act_early", dict(base, pdl=True, flags=base["flags"] | dg.FLAG_INDEPENDENT_INPUTS)),
                    ("grid_end", dict(base, pdl=False, flags=base["flags"] & ~dg.FLAG_INDEPENDENT_INPUTS)))
        for label, cfg in variants:
            run_point(run, sess, md, ad, ref, StepVariant(v.step, mt, b200=cfg, kind="placement"), plan, False,
                      sink=w, suffix=label)


if __name__ == "__main__":
    raise SystemExit(main())
