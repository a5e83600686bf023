#!/usr/bin/env python
"""Cold-weight FP8 decode GEMM benchmark (the BASELINE metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--m M]

Workload: Y[M x N] = X[M x K] . W[N x K]^T with N = 7168,
K = 16384, M = 1 by default; W and X are FP8 E4M3 from seeded N(0,1) draws,
each quantised with one per-tensor fp32 scale (amax -> 448); BF16 output,
fp32 accumulation.  Weights rotate over >= max(1 GiB, 4 x L2) of distinct
device copies, so every launch reads its weights cold from HBM (the inputs
are larger than L2; no flush needed).  A step is one GEMM; K steps are timed
with CUDA events on the launching stream, replayed from a CUDA graph, and
with programmatic dependent launch between consecutive GEMMs.

Multi-GPU (launched with torch.distributed.run, one rank per GPU): the path
partitions by weight rows with no exchange inside the GEMM, so the headline
is weak scaling: every rank streams its own N x K shard of one
tensor-parallel layer of g*N rows, value = all ranks' bytes / the max-over-
ranks time.  Beside it: the same step with the NCCL all-gather of the BF16
output slices, and the strong-scaling layer (the single N x K matrix
N-sharded g ways, with and without the gather).

Metric: algorithmic bytes (N*K + M*K + 2*M*N) per GEMM / time, GB/s, and
us per GEMM.  `e2e` repeats the measurement through the public API with
every step's activation and scales copied in from pinned host memory and its
output copied back, inside the timed region: a serving loop with
--e2e-depth requests in flight (one stream each, captured in CUDA graphs;
on N GPUs the fused GEMMs stay on one stream in groups of --e2e-group that
chain under PDL, and the copies overlap them), and beside it one request at
a time on one stream.

`--impl reference` times the reference's own CPU implementation of the path
(the host scalar GEMM of kernels/smoke_test.cu, compiled from the reference
source into oracle/_ref; the oracle restatement when that build is absent)
on all host cores, on bounded samples of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "cold-weight HBM GB/s & % of peak per B200 at M=1..128; µs per GEMM"
# Where the one JSON line goes (the process's stdout; see main()).
JSON_OUT = sys.stdout
SPEC_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--n", type=int, default=7168)
    ap.add_argument("--k", type=int, default=16384)
    ap.add_argument("--layout", choices=["raw", "packed", "swizzled"], default="swizzled")
    ap.add_argument("--no-pdl", action="store_true")
    ap.add_argument("--pdl-mode", choices=["independent", "dependent"], default="independent",
                    help="independent: consecutive GEMMs do not produce each other's inputs (the "
                         "reference's back-to-back PDL protocol); dependent: every launch waits for "
                         "the previous grid before reading its activation (a layer chain). Both are "
                         "timed; this picks the headline.")
    ap.add_argument("--schedule", choices=["cluster", "stream_k"], default="cluster",
                    help="default_config's schedule: cluster split-K (default) or stream-K over one CTA per SM")
    ap.add_argument("--batch-class", choices=["auto", "default", "swap_ab"], default="auto",
                    help="kernel class for M <= 16 on the cluster schedule: auto (default_config's measured "
                         "choice), the default class (batch on the MMA's M side, padded to 64) or swap-AB "
                         "(weights on the M side, batch padded to 16 on N)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--e2e-depth", type=int, default=8,
                    help="e2e loop on 1 GPU: requests in flight, one stream each (1: no pipelined loop); "
                         "the independent schedule's 28-CTA GEMMs need about five in flight to fill the GPU")
    ap.add_argument("--e2e-group", type=int, default=16,
                    help="e2e loop on N GPUs: fused GEMMs per group that chain under PDL, the group's "
                         "first waiting on the copy streams (1: no pipelined loop)")
    ap.add_argument("--e2e-schedule", choices=["independent", "dependent"], default="independent",
                    help="schedule of the e2e loop's GEMMs (they do not feed each other)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="CPU work the rank-0 cpu_baseline sample is sized to")
    ap.add_argument("--ref-seconds", type=float, default=60.0,
                    help="--impl reference: CPU time its warm-up and timed steps are sized to")
    ap.add_argument("--graph-chunk", type=int, default=500, help="launches per captured CUDA graph")
    ap.add_argument("--no-sweep", action="store_true", help="skip the M = 1..128 sweep")
    ap.add_argument("--no-cublas", action="store_true", help="skip the cuBLASLt FP8 baseline")
    ap.add_argument("--no-chain", action="store_true", help="skip the 61-layer dependent chain")
    ap.add_argument("--gather-protocol", choices=["flags", "lines"], default="lines",
                    help="fused-gather protocol of the N-GPU e2e serving loop (dg_launch_gather with epoch "
                         "flags, or dg_launch_gather_lines with tagged lines)")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic(workload_key):
    """DRAM bytes per launch from the committed ncu summary (profiles/)."""
    path = os.path.join(ROOT, "profiles", "ncu_traffic.txt")
    try:
        with open(path) as f:
            return json.load(f).get(workload_key)
    except (OSError, ValueError):
        return None


def quantize_pertensor(x, fp8):
    """Per-tensor scale s = amax/448, q = clamp(x/s) -> e4m3 (round to nearest even)."""
    import torch
    amax = x.abs().max().clamp_min(1e-4)
    s = (amax / 448.0).float()
    q = (x / s).clamp(-448.0, 448.0).to(fp8).view(torch.uint8)
    return q, s


# ---------------------------------------------------------------------------
# reference arm: the reference's CPU path on all host cores
# ---------------------------------------------------------------------------

def cpu_gemm_fn():
    """(callable, kind): the reference's own compute_reference when it was
    built here (oracle/_ref), else the oracle restatement."""
    import ctypes
    import numpy as np
    import oracle
    ref = oracle.load_ref()
    if ref is not None:
        kind = "reference"

        def run(a, as_, w, ws, n_rows):
            m, k = a.shape
            out = np.zeros((m, n_rows), np.float32)
            ref.ref_compute_reference(m, n_rows, k, a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                                      as_.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                      w.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
                                      ws.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                      out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
            return out
    else:
        kind = "port"

        def run(a, as_, w, ws, n_rows):
            return oracle.compute_reference(a, as_, w, ws, n=n_rows)
    return run, kind


def cpu_parallel_gemm(run, a, as_, w, ws, threads):
    """Rows of W split over threads in 128-row blocks (scale groups stay
    whole); each block is an independent call of the single-threaded
    reference GEMM, so the result equals the one-thread result."""
    import numpy as np
    n = w.shape[0]
    blocks = max(1, (n + 127) // 128)
    per = (blocks + threads - 1) // threads
    parts = [None] * threads
    kb = a.shape[1] // 128

    def work(t):
        b0, b1 = t * per, min(blocks, (t + 1) * per)
        if b0 >= b1:
            return
        r0, r1 = b0 * 128, min(n, b1 * 128)
        parts[t] = (r0, run(a, as_, np.ascontiguousarray(w[r0:r1]),
                            np.ascontiguousarray(ws[b0:b1].reshape(-1, kb)), r1 - r0))

    pool = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    for th in pool:
        th.start()
    for th in pool:
        th.join()
    out = np.zeros((a.shape[0], n), np.float32)
    for part in parts:
        if part is not None:
            out[:, part[0]:part[0] + part[1].shape[1]] = part[1]
    return out


def cublaslt_driver(n, k, ms, dev):
    """Runs decode_opt_b200/dg_cublaslt_fp8 (block-scaled and per-tensor) on
    `dev`: {"block": [per-M dicts], "tensor": [...]}, or {"unavailable": why}."""
    import subprocess
    exe = os.path.join(os.path.dirname(os.path.abspath(__file__)), "decode_opt_b200", "dg_cublaslt_fp8")
    if not os.path.exists(exe):
        return {"unavailable": "dg_cublaslt_fp8 not built"}
    # The child's device 0 is this process's `dev`.
    idx = dev.index or 0
    visible = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES=visible[idx] if idx < len(visible) and visible[idx] else str(idx))
    out = {}
    for mode in ("block", "tensor"):
        try:
            proc = subprocess.run([exe, "--n", str(n), "--k", str(k), "--ms", ",".join(map(str, ms)),
                                   "--mode", mode, "--iters", "200"], capture_output=True, text=True,
                                  timeout=600, env=env)
            rows = [json.loads(ln) for ln in proc.stdout.splitlines() if ln.startswith("{")]
            out[mode] = rows if proc.returncode == 0 else [{"unavailable": proc.stderr[-300:]}]
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            out[mode] = [{"unavailable": f"{type(exc).__name__}: {exc}"[:200]}]
    return out


def host_inputs(n, k, m, seed=20260913):
    """Per-tensor-scaled N(0,1) e4m3 inputs on the host (torch CPU generator)."""
    import numpy as np
    import torch
    g = torch.Generator().manual_seed(seed)
    w = torch.randn((n, k), generator=g)
    qw, sw = quantize_pertensor(w, torch.float8_e4m3fn)
    del w
    x = torch.randn((m, k), generator=g)
    qx, sx = quantize_pertensor(x, torch.float8_e4m3fn)
    kb = k // 128
    ws = np.full(((n + 127) // 128, kb), float(sw), np.float32)
    as_ = np.full((m, kb), float(sx), np.float32)
    return qw.numpy(), ws, qx.numpy(), as_


def reference_arm(args, rank, world):
    if rank != 0:
        return
    import numpy as np
    run, kind = cpu_gemm_fn()
    threads = os.cpu_count() or 1
    n, k, m = args.n, args.k, args.m
    w, ws, a, as_ = host_inputs(n, k, m)
    # Size each step's sample so the warm-up and timed steps take about
    # --ref-seconds (a minute by default).
    rows_probe = min(n, 1024)
    t0 = time.perf_counter()
    cpu_parallel_gemm(run, a, as_, w[:rows_probe], ws[: (rows_probe + 127) // 128], threads)
    per_row = (time.perf_counter() - t0) / rows_probe
    budget = args.ref_seconds / max(args.steps + args.warmup, 1)
    rows = int(max(128, min(n, budget / max(per_row, 1e-12))) // 128 * 128)
    w_s, ws_s = w[:rows], ws[: rows // 128]
    for _ in range(args.warmup):
        cpu_parallel_gemm(run, a, as_, w_s, ws_s, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_parallel_gemm(run, a, as_, w_s, ws_s, threads)
    dt = (time.perf_counter() - t0) / max(args.steps, 1)
    byt = rows * k + m * k + 2 * m * rows
    gbs = byt / dt / 1e9
    sample = (f"{rows} of {n} weight rows per step (x {k} K, M={m}), {threads} threads, "
              f"reference compute_reference per 128-row block")
    line = {
        "impl": "reference", "metric": METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp8e4m3-in/f32-acc/bf16-out", "data": "synthetic",
        "config": {"workload": f"C2 decode GEMM N={n} K={k} M={m} (CPU sample)", "M": m, "N": n, "K": k},
        "cpu_baseline": {"value": gbs, "unit": "GB/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), file=JSON_OUT, flush=True)


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

class Rotation:
    """One weight shard of n x k e4m3 in `layout`, rotated over enough
    distinct device copies (>= max(1 GiB, 4 x L2)) that every launch reads
    its weights cold from HBM, plus the problems and tensor maps for one
    batch size."""

    def __init__(self, qw, layout, block_n, dev):
        import torch
        import decode_opt_b200 as dg
        self.n, self.k = qw.shape
        base = qw if layout == dg.LAYOUT_RAW else dg.prepack_weight(qw, block_n, layout)
        self.set_bytes = base.numel()
        l2 = torch.cuda.get_device_properties(dev).L2_cache_size
        self.l2 = l2
        self.nsets = max(5, math.ceil(max(1 << 30, 4 * l2) / self.set_bytes))
        self.sets = [base] + [base.clone() for _ in range(self.nsets - 1)]


class GemmSetup:
    """Problems, maps and buffers for one (rotation, M, config)."""

    def __init__(self, rot, cfg, m, qx, wscale, ascale, dev, host_out=None):
        """host_out: a pinned host [m, n] bf16 tensor the kernel writes its
        output into directly (zero-copy, dg.host_device_pointer)."""
        import torch
        import decode_opt_b200 as dg
        self.cfg = cfg
        self.m = m
        self.plan = cfg.plan(m, rot.n, rot.k)
        if self.plan.error:
            raise SystemExit(self.plan.error)
        if host_out is None:
            self.out = torch.empty((m, rot.n), dtype=torch.bfloat16, device=dev)
            out_arg = self.out
        else:
            self.out = host_out
            out_arg = dg.host_device_pointer(host_out)
        self.ws = torch.zeros(max(self.plan.ws_floats, 1), dtype=torch.float32, device=dev)
        self.sem = torch.zeros(max(self.plan.sem_ints, 1), dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.probs = [dg.Problem(m, rot.n, rot.k, qx, w, wscale, ascale, out_arg, self.ws, self.sem, self.status)
                      for w in rot.sets]
        self.wmaps = [dg.make_weight_tma(cfg, p) for p in self.probs]
        self.amap = dg.make_activation_tma(cfg, self.probs[0])
        self.nsets = rot.nsets

    def launch(self, i, stream):
        import decode_opt_b200 as dg
        rc = dg.launch_with_maps(self.cfg, self.probs[i % self.nsets], self.wmaps[i % self.nsets], self.amap,
                                 stream, pdl_attr=self.cfg.pdl)
        if rc != 0:
            raise RuntimeError(f"launch failed: cudaError {rc}")

    def check_status(self):
        import decode_opt_b200 as dg
        st = int(self.status.item())
        if st != 0:
            raise RuntimeError(f"kernel status {dg.status_string(st)}")


def b200_arm(args, rank, world, local_rank):
    import numpy as np
    import torch
    import torch.distributed as dist
    import decode_opt_b200 as dg

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    n, k, m = args.n, args.k, args.m
    layout = {"raw": dg.LAYOUT_RAW, "packed": dg.LAYOUT_PACKED, "swizzled": dg.LAYOUT_PACKED_SWIZZLED}[args.layout]
    pdl = not args.no_pdl
    independent = args.pdl_mode == "independent"

    def default_config(*a, **kw):
        if args.batch_class == "swap_ab" and a[0] <= 16 and args.schedule == "cluster":
            kw.setdefault("swap_ab", True)
        elif args.batch_class == "default":
            kw.setdefault("swap_ab", False)
        return dg.default_config(*a, schedule=args.schedule, **kw)

    stream = torch.cuda.Stream(device=dev)
    pg = dist.group.WORLD if world > 1 else None

    def device_max(t):
        if world > 1:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            return float(tt.item())
        return t

    def capture(fn, count):
        """CUDA graphs of `count` calls of fn(i) on `stream` (chunks of graph_chunk)."""
        graphs = []
        left = count
        base = 0
        with torch.cuda.stream(stream):
            while left > 0:
                chunk = min(left, args.graph_chunk)
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for i in range(chunk):
                        fn(base + i)
                graphs.append(gr)
                left -= chunk
                base += chunk
        return graphs

    def timed(graphs, warm=True):
        """Seconds for one replay of all graphs: barrier + synchronize on both
        sides, CUDA events on the launching stream, max over ranks."""
        if warm:
            with torch.cuda.stream(stream):
                graphs[0].replay()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for gr in graphs:
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        t = device_max(e0.elapsed_time(e1) / 1e3)
        if world > 1:
            dist.barrier()
        return t

    # ---- synthetic inputs: per-tensor-scaled N(0,1) e4m3 --------------------
    # Weak scaling: every rank holds a full n x k shard of one tensor-parallel
    # layer of world*n rows (rank r: rows [r*n, (r+1)*n)); the activation is
    # shared.  Seeds make every rank's shard distinct and reproducible.
    g = torch.Generator(device=dev).manual_seed(20260913 + 7919 * rank)
    w_full = torch.randn((n, k), device=dev, generator=g)
    qw, sw = quantize_pertensor(w_full, torch.float8_e4m3fn)
    del w_full
    gx = torch.Generator(device=dev).manual_seed(20260913)
    x = torch.randn((128, k), device=dev, generator=gx)
    kb = k // 128
    wscale = torch.full(((n + 127) // 128, kb), float(sw), device=dev)

    def act(mm):
        q, s = quantize_pertensor(x[:mm], torch.float8_e4m3fn)
        return q.contiguous(), torch.full((mm, kb), float(s), device=dev), float(s)

    qx, ascale, sx = act(m)
    rotations = {}

    def rotation(block_n):
        """Cold copies of this rank's weights in the layout `block_n` needs."""
        key = 0 if layout == dg.LAYOUT_RAW else block_n
        if key not in rotations:
            rotations[key] = Rotation(qw, layout, block_n, dev)
        return rotations[key]

    def lines_ready(setup, mm, nn, rot_fn, qx_m, ws_m, as_m, indep):
        """A setup the tagged-lines gather accepts: `setup` itself where its
        plan splits every tile over at least two CTAs (the gather stores from
        the cluster reduction), else one on default_config(gather_lines=True)."""
        if setup.plan.cluster >= 2:
            return setup
        cfg_l = default_config(mm, nn, k, layout=layout, pdl=pdl, independent_inputs=indep, gather_lines=True)
        return GemmSetup(rot_fn(cfg_l.block_n), cfg_l, mm, qx_m, ws_m, as_m, dev)

    # The headline mode's schedule and the other PDL mode's, each with its own
    # weight copies (packed for its tile width) and tensor maps.
    cfg = default_config(m, n, k, layout=layout, pdl=pdl, independent_inputs=independent)
    cfg_other = default_config(m, n, k, layout=layout, pdl=pdl, independent_inputs=not independent)
    rot = rotation(cfg.block_n)
    gs = GemmSetup(rot, cfg, m, qx, wscale, ascale, dev)
    gs_other = GemmSetup(rotation(cfg_other.block_n), cfg_other, m, qx, wscale, ascale, dev)
    gs_dep = gs_other if independent else gs      # inputs produced by the preceding operation
    gathered = torch.empty((world * m, n), dtype=torch.bfloat16, device=dev)

    def gemm_step(i):
        gs.launch(i, stream)

    def tp_step(i):
        # An NCCL collective between GEMMs serialises them: the dependent
        # (latency) schedule is the best one for this baseline.
        gs_dep.launch(i, stream)
        dist.all_gather_into_tensor(gathered, gs_dep.out, group=pg)

    K = args.steps
    # Fused-gather sections alternate two buffer sets per launch; an even
    # launch count keeps the alternation across graph replays (a replay
    # restarting on the set the previous one ended on would hand a peer a set
    # this rank may still be reading).
    K2 = K + K % 2
    # ---- warm-up: eager launches, then every graph once (in timed()) ------------
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            gs.launch(i, stream)
            if world > 1:
                dist.all_gather_into_tensor(gathered, gs.out, group=pg)
    torch.cuda.synchronize(dev)
    gs.check_status()

    graphs = capture(gemm_step, K)
    from decode_opt_b200.clocks import ClockSampler
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.05)
    with torch.cuda.stream(stream):
        graphs[0].replay()
    torch.cuda.synchronize(dev)
    clocks.mark()
    t_gemm = timed(graphs, warm=False)
    clocks.mark()
    clocks.stop()
    del graphs
    gs.check_status()
    with torch.cuda.stream(stream):
        for i in range(3):
            gs_other.launch(i, stream)
    torch.cuda.synchronize(dev)
    gs_other.check_status()
    graphs = capture(lambda i: gs_other.launch(i, stream), K)
    t_other = timed(graphs)
    del graphs
    gs_other.check_status()

    byt_gpu = n * k + m * k + 2 * m * n             # one rank's GEMM per step
    byt_job = world * byt_gpu
    us_gemm = t_gemm / K * 1e6
    value = byt_job / (t_gemm / K) / 1e9
    peak, peak_kind = measured_peaks()
    achieved = byt_gpu / (t_gemm / K) / 1e9
    workload_key = f"N{n}_K{k}_M{m}_{args.layout}" + ("_swap_ab" if cfg.flags & dg.FLAG_SWAP_AB else "")

    # ---- multi-GPU: with the NCCL gather, and the strong-scaling layer ---------
    tp = None
    fused = None
    if world > 1:
        from decode_opt_b200 import tp as dg_tp
        graphs = capture(tp_step, K)
        t_tp = timed(graphs)
        del graphs
        # The all-gather fused into the GEMM: every rank stores its slices into
        # all ranks' gathered buffers over NVLink (two buffer sets alternate).
        # Both protocols run on one setup that the tagged-lines gather accepts
        # (at least two CTAs per tile), so their outputs can be compared.
        gs_g = lines_ready(gs, m, n, rotation, qx, wscale, ascale, independent)
        fused = dg_tp.FusedGather(m, n, device=dev)
        fdesc = [fused.descriptor(0), fused.descriptor(1)]

        def fused_step(i, setup=gs_g):
            rc = dg.launch_gather(setup.cfg, setup.probs[i % setup.nsets], fdesc[i % 2],
                                  setup.wmaps[i % setup.nsets], setup.amap, stream, pdl_attr=setup.cfg.pdl)
            if rc != 0:
                raise RuntimeError(f"fused launch failed: cudaError {rc}")
        def fused_steps(i):
            fused_step(i)
            if i == K2 - 1:      # the last launch's gather completes inside the timed region
                fused.wait((K2 - 1) % 2, stream=stream, status=gs_g.status)
        graphs = capture(fused_steps, K2)
        t_fused = timed(graphs)
        del graphs
        gs_g.check_status()
        # The same with the gather in tagged lines (no flags, no fences).
        fused_l = dg_tp.FusedGather(m, n, device=dev, protocol="lines")
        ldesc = [fused_l.descriptor(0), fused_l.descriptor(1)]

        def lines_steps(i):
            rc = dg.launch_gather(gs_g.cfg, gs_g.probs[i % gs_g.nsets], ldesc[i % 2], gs_g.wmaps[i % gs_g.nsets],
                                  gs_g.amap, stream, pdl_attr=gs_g.cfg.pdl)
            if rc != 0:
                raise RuntimeError(f"fused launch (lines) failed: cudaError {rc}")
        graphs = capture(lines_steps, K2)
        t_fused_l = timed(graphs)
        del graphs
        gs_g.check_status()
        # Both protocols gathered the same product of the same inputs.
        lines_match = bool(torch.equal(fused_l.output((K2 - 1) % 2, m).view(torch.int16),
                                       fused.output((K2 - 1) % 2, m).view(torch.int16)))
        fused_l.close()
        # Strong scaling: the one n x k layer N-sharded over
        # the ranks, each streaming n/world rows, then the gather -- at the
        # headline M and at config 5's M = 1, 8, 64.
        n_s = n // world
        strong = None
        if n % world == 0 and n_s % 128 == 0:
            q_s = qw[:n_s].contiguous()
            ws_s = wscale[: n_s // 128].contiguous()
            rot_cache = {}

            def rot_for(block_n):
                key = 0 if layout == dg.LAYOUT_RAW else block_n
                if key not in rot_cache:
                    rot_cache[key] = Rotation(q_s, layout, block_n, dev)
                return rot_cache[key]

            def strong_for(mm, qx_m, ascale_m):
                cfg_s = default_config(mm, n_s, k, layout=layout, pdl=pdl, independent_inputs=independent)
                gs_s = GemmSetup(rot_for(cfg_s.block_n), cfg_s, mm, qx_m, ws_s, ascale_m, dev)
                gathered_s = torch.empty((world * mm, n_s), dtype=torch.bfloat16, device=dev)
                graphs = capture(lambda i: gs_s.launch(i, stream), K)
                t_s = timed(graphs)
                del graphs
                cfg_sd = default_config(mm, n_s, k, layout=layout, pdl=pdl, independent_inputs=False)
                gs_sd = gs_s if cfg_sd == cfg_s else GemmSetup(rot_for(cfg_sd.block_n), cfg_sd, mm, qx_m, ws_s,
                                                               ascale_m, dev)
                with torch.cuda.stream(stream):
                    for i in range(3):
                        gs_sd.launch(i, stream)
                torch.cuda.synchronize(dev)

                def strong_tp(i):
                    gs_sd.launch(i, stream)
                    dist.all_gather_into_tensor(gathered_s, gs_sd.out, group=pg)
                graphs = capture(strong_tp, K)
                t_s_tp = timed(graphs)
                del graphs
                gs_sg = lines_ready(gs_s, mm, n_s, rot_for, qx_m, ws_s, ascale_m, independent)
                fused_s = dg_tp.FusedGather(mm, n_s, device=dev)
                fdesc_s = [fused_s.descriptor(0), fused_s.descriptor(1)]

                def strong_fused(i):
                    rc = dg.launch_gather(gs_sg.cfg, gs_sg.probs[i % gs_sg.nsets], fdesc_s[i % 2],
                                          gs_sg.wmaps[i % gs_sg.nsets], gs_sg.amap, stream, pdl_attr=gs_sg.cfg.pdl)
                    if rc != 0:
                        raise RuntimeError(f"fused launch failed: cudaError {rc}")

                def strong_fused_steps(i):
                    strong_fused(i)
                    if i == K2 - 1:
                        fused_s.wait((K2 - 1) % 2, stream=stream, status=gs_sg.status)
                graphs = capture(strong_fused_steps, K2)
                t_s_fused = timed(graphs)
                del graphs
                fused_sl = dg_tp.FusedGather(mm, n_s, device=dev, protocol="lines")
                ldesc_s = [fused_sl.descriptor(0), fused_sl.descriptor(1)]

                def strong_lines(i):
                    rc = dg.launch_gather(gs_sg.cfg, gs_sg.probs[i % gs_sg.nsets], ldesc_s[i % 2],
                                          gs_sg.wmaps[i % gs_sg.nsets], gs_sg.amap, stream, pdl_attr=gs_sg.cfg.pdl)
                    if rc != 0:
                        raise RuntimeError(f"fused launch (lines) failed: cudaError {rc}")
                graphs = capture(strong_lines, K2)
                t_s_lines = timed(graphs)
                del graphs
                same_s = bool(torch.equal(fused_sl.output((K2 - 1) % 2, mm).view(torch.int16),
                                          fused_s.output((K2 - 1) % 2, mm).view(torch.int16)))
                fused_sl.close()
                fused_s.close()
                gs_s.check_status()
                gs_sg.check_status()
                byt_layer = n * k + mm * k + 2 * mm * n
                return {"M": mm, "N_layer": n, "rows_per_gpu": n_s,
                        "gemm_only": {"us_per_gemm": t_s / K * 1e6, "GBps_job": byt_layer / (t_s / K) / 1e9},
                        "with_gather": {"us_per_step": t_s_tp / K * 1e6,
                                        "GBps_job": byt_layer / (t_s_tp / K) / 1e9},
                        "with_fused_gather": {"us_per_step": t_s_fused / K2 * 1e6,
                                              "GBps_job": byt_layer / (t_s_fused / K2) / 1e9},
                        "with_fused_gather_lines": {"us_per_step": t_s_lines / K2 * 1e6,
                                                    "GBps_job": byt_layer / (t_s_lines / K2) / 1e9,
                                                    "output_equals_flags_protocol": same_s}}

            strong = strong_for(m, qx, ascale)
            strong["m_sweep"] = []
            for mm in (1, 8, 64):
                if mm == m:
                    strong["m_sweep"].append({kk: vv for kk, vv in strong.items() if kk != "m_sweep"})
                    continue
                q_m, s_m, _ = act(mm)
                strong["m_sweep"].append(strong_for(mm, q_m, s_m))
            del rot_cache
        tp = {"with_gather": {"us_per_step": t_tp / K * 1e6, "GBps_job": byt_job / (t_tp / K) / 1e9,
                              "collective": "NCCL all_gather_into_tensor of the bf16 [M, N/g] slices"},
              "with_fused_gather": {"us_per_step": t_fused / K2 * 1e6, "GBps_job": byt_job / (t_fused / K2) / 1e9,
                                    "collective": "none: the GEMM stores its slices into every rank's "
                                                  "gathered [M, g*N] buffer over NVLink (dg_launch_gather)"},
              "with_fused_gather_lines": {"us_per_step": t_fused_l / K2 * 1e6,
                                          "GBps_job": byt_job / (t_fused_l / K2) / 1e9,
                                          "output_equals_flags_protocol": lines_match,
                                          "collective": "none: the GEMM stores its slices as tagged 16-byte lines "
                                                        "{2 bf16, epoch} x 2 into every rank's line buffer over "
                                                        "NVLink; each rank unpacks its own "
                                                        "(dg_launch_gather_lines)"},
              "strong_scaling": strong}

    # ---- end to end through the public API with host buffers ----------------
    e2e = None
    if not args.no_e2e:
        # The step's inputs -- activation [m, k] e4m3 and its scales [m, k/128]
        # fp32 -- travel as one pinned buffer in one host-to-device copy into
        # one device buffer that the GEMM reads in place.
        in_bytes = m * k + m * kb * 4
        hin = torch.empty(in_bytes, dtype=torch.uint8).pin_memory()
        hin[: m * k].copy_(qx.view(torch.uint8).reshape(-1).cpu())
        hin[m * k:].copy_(ascale.reshape(-1).cpu().view(torch.uint8))
        dev_in = torch.empty(in_bytes, dtype=torch.uint8, device=dev)
        act_in = dev_in[: m * k].view(m, k)
        sc_in = dev_in[m * k:].view(torch.float32).view(m, kb)
        gs_e2e = GemmSetup(rotation(gs_dep.cfg.block_n), gs_dep.cfg, m, act_in, wscale, sc_in, dev)
        if world > 1 and args.gather_protocol == "lines":
            gs_e2e = lines_ready(gs_e2e, m, n, rotation, act_in, wscale, sc_in, False)
        hy = torch.empty((m, world * n), dtype=torch.bfloat16).pin_memory()

        fused_e = None
        if world > 1:
            fused_e = dg_tp.FusedGather(m, n, device=dev, protocol=args.gather_protocol)
            edesc = [fused_e.descriptor(0), fused_e.descriptor(1)]

        def e2e_step(i):
            dev_in.copy_(hin, non_blocking=True)
            if world > 1:
                rc = dg.launch_gather(gs_e2e.cfg, gs_e2e.probs[i % gs_e2e.nsets], edesc[i % 2],
                                      gs_e2e.wmaps[i % gs_e2e.nsets], gs_e2e.amap, stream, pdl_attr=gs_e2e.cfg.pdl)
                if rc != 0:
                    raise RuntimeError(f"fused launch failed: cudaError {rc}")
                fused_e.wait(i % 2, stream=stream, status=gs_e2e.status)
                hy.copy_(fused_e.output(i % 2, m), non_blocking=True)
            else:
                gs_e2e.launch(i, stream)
                hy.copy_(gs_e2e.out, non_blocking=True)

        def timed_serial(steps, step_fn=e2e_step):
            """One request at a time on one stream (H2D, GEMM -- with the fused
            gather on N GPUs -- D2H), captured in CUDA graphs."""
            with torch.cuda.stream(stream):
                for i in range(4):
                    step_fn(i)
            torch.cuda.synchronize(dev)
            graphs = capture(lambda i: step_fn(i + 4), steps)
            t = timed(graphs)
            del graphs
            return t

        # Zero-copy output (one GPU): the GEMM writes its bf16 result straight
        # into pinned host memory over PCIe (dg.host_device_pointer), so the
        # step is the H2D copy and the launch; the result's bytes still cross
        # PCIe every step, as kernel stores instead of a copy node.
        hy_zc = torch.empty((m, n), dtype=torch.bfloat16).pin_memory() if world == 1 else None
        gs_zc = (GemmSetup(rotation(gs_dep.cfg.block_n), gs_dep.cfg, m, act_in, wscale, sc_in, dev, host_out=hy_zc)
                 if world == 1 else None)

        def e2e_step_zc(i):
            dev_in.copy_(hin, non_blocking=True)
            gs_zc.launch(i, stream)

        # The same with the input copied by a kernel (dg.copy_from_host) under
        # programmatic dependent launch instead of a copy node: it waits for
        # the previous request's GEMM before writing the input, so requests
        # still run one at a time, but each GEMM launches and prefetches its
        # weights while the previous one runs.
        hy_zk = torch.empty((m, n), dtype=torch.bfloat16).pin_memory() if world == 1 else None
        gs_zk = (GemmSetup(rotation(gs_dep.cfg.block_n), gs_dep.cfg, m, act_in, wscale, sc_in, dev, host_out=hy_zk)
                 if world == 1 else None)
        hin_dev = dg.host_device_pointer(hin) if world == 1 else None

        def e2e_step_zk(i):
            dg.copy_from_host(dev_in, hin, stream, pdl_attr=True, src_device=hin_dev)
            gs_zk.launch(i, stream)

        pipe = None
        if world == 1:
            # A serving loop keeps `depth` requests in flight: request i runs
            # on stream i % depth with that slot's own device input, output and
            # pinned host output -- its H2D copy, GEMM and D2H copy in stream
            # order -- so one request's copies overlap the others' GEMMs.  The
            # GEMMs do not feed each other: the independent-inputs schedule.
            depth = max(1, args.e2e_depth)
            cfg_p = default_config(m, n, k, layout=layout, pdl=pdl,
                                      independent_inputs=args.e2e_schedule == "independent")

            def run_pipe(zero_copy):
                slots = []
                for _ in range(depth):
                    d_in = torch.empty(in_bytes, dtype=torch.uint8, device=dev)
                    h_out = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
                    g_p = GemmSetup(rotation(cfg_p.block_n), cfg_p, m, d_in[: m * k].view(m, k), wscale,
                                    d_in[m * k:].view(torch.float32).view(m, kb), dev,
                                    host_out=h_out if zero_copy else None)
                    slots.append((d_in, g_p, h_out, torch.cuda.Stream(device=dev)))

                def pipe_step(i):
                    d_in, g_p, h_out, st = slots[i % depth]
                    with torch.cuda.stream(st):
                        d_in.copy_(hin, non_blocking=True)
                        g_p.launch(i, st)
                        if not zero_copy:
                            h_out.copy_(g_p.out, non_blocking=True)

                for i in range(3 * depth):
                    pipe_step(i)
                torch.cuda.synchronize(dev)
                # The loop is captured in CUDA graphs (graph_chunk requests each,
                # forked to the slot streams and joined back), as a decode server
                # replays its step: the copy nodes still move every request's
                # bytes over PCIe at replay time, but no Python runs per request.
                graphs = []
                with torch.cuda.stream(stream):
                    for base in range(0, K, args.graph_chunk):
                        gr = torch.cuda.CUDAGraph()
                        with torch.cuda.graph(gr, stream=stream):
                            for _, _, _, st in slots:
                                st.wait_stream(stream)
                            for i in range(base, min(K, base + args.graph_chunk)):
                                pipe_step(i)
                            for _, _, _, st in slots:
                                stream.wait_stream(st)
                        graphs.append(gr)
                t_pipe = timed(graphs)
                del graphs
                return {"t": t_pipe, "depth": depth, "cfg": cfg_p, "zero_copy": zero_copy,
                        "plan": slots[0][1].plan, "outs": [sl[2] for sl in slots], "setups": [sl[1] for sl in slots]}

            pipe_copy = run_pipe(False)
            pipe_zc = run_pipe(True)
            pipe = pipe_zc if pipe_zc["t"] < pipe_copy["t"] else pipe_copy
        elif args.e2e_group > 1:
            # Requests pipelined on N GPUs, in groups of `grp`
            # (decode_opt_b200.tp.serving_schedule: which operation waits on
            # which).  A fused launch waits for its peers' launches, so every
            # rank issues the fused GEMMs on ONE stream in the same order (two
            # of them in flight on one GPU from different streams could wait on
            # each other across GPUs); the H2D copies and the D2H copy after
            # every GEMM run on two copy streams beside them.  Only a group's
            # first GEMM waits on the copy streams: a captured GEMM node with
            # cross-stream edges loses its programmatic edge, and the other
            # GEMMs of the group keep theirs, so they overlap under PDL.
            # 2*grp input slots and gathered buffer sets rotate.  Each graph
            # forks and joins the copy streams, so events never cross a graph
            # boundary.
            grp = args.e2e_group
            nset = 2 * grp
            depth = nset
            cfg_p = default_config(m, n, k, layout=layout, pdl=pdl,
                                   independent_inputs=args.e2e_schedule == "independent",
                                   gather_lines=args.gather_protocol == "lines")
            fused_p = dg_tp.FusedGather(m, n, buffers=nset, device=dev, protocol=args.gather_protocol)
            pdesc = [fused_p.descriptor(j) for j in range(nset)]
            slots = []
            for _ in range(nset):
                d_in = torch.empty(in_bytes, dtype=torch.uint8, device=dev)
                slots.append((d_in, GemmSetup(rotation(cfg_p.block_n), cfg_p, m, d_in[: m * k].view(m, k),
                                              wscale, d_in[m * k:].view(torch.float32).view(m, kb), dev)))
            h_outs = [torch.empty((m, world * n), dtype=torch.bfloat16).pin_memory() for _ in range(nset)]
            h2d_st = torch.cuda.Stream(device=dev)
            d2h_st = torch.cuda.Stream(device=dev)
            ring = 2 * nset + 2
            op_stream = {"h2d": h2d_st, "gemm": stream, "d2h": d2h_st}
            op_done = {kind: [torch.cuda.Event() for _ in range(ring)] for kind in op_stream}

            def run_op(kind, j, waits):
                st = op_stream[kind]
                for w_kind, w_j in waits:
                    st.wait_event(op_done[w_kind][w_j % ring])
                if kind == "h2d":
                    with torch.cuda.stream(st):
                        slots[j % nset][0].copy_(hin, non_blocking=True)
                elif kind == "gemm":
                    g_p = slots[j % nset][1]
                    rc = dg.launch_gather(g_p.cfg, g_p.probs[j % g_p.nsets], pdesc[j % nset],
                                          g_p.wmaps[j % g_p.nsets], g_p.amap, stream, pdl_attr=g_p.cfg.pdl)
                    if rc != 0:
                        raise RuntimeError(f"fused launch failed: cudaError {rc}")
                    # No dg_gather_wait node: a fused grid completes only after
                    # its last CTA saw every peer's epoch for this launch (each
                    # peer publishes after a system-scope fence over its slice
                    # stores), so the copy that follows reads the whole output.
                else:
                    with torch.cuda.stream(st):
                        h_outs[j % nset].copy_(fused_p.output(j % nset, m), non_blocking=True)
                op_done[kind][j % ring].record(st)

            def mg_chunk(base, count):
                h2d_st.wait_stream(stream)
                d2h_st.wait_stream(stream)
                for op in dg_tp.serving_schedule(base, count, grp):
                    run_op(*op)
                stream.wait_stream(h2d_st)
                stream.wait_stream(d2h_st)

            with torch.cuda.stream(stream):
                mg_chunk(0, 3 * nset)
            torch.cuda.synchronize(dev)
            chunk = max(grp, args.graph_chunk - args.graph_chunk % grp)
            graphs = []
            with torch.cuda.stream(stream):
                for base in range(0, K, chunk):
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=stream):
                        mg_chunk(base, min(K, base + chunk) - base)
                    graphs.append(gr)
            t_pipe = timed(graphs)
            del graphs
            pipe = {"t": t_pipe, "depth": depth, "cfg": cfg_p, "plan": slots[0][1].plan,
                    "outs": h_outs, "setups": [sl[1] for sl in slots], "fused": fused_p}

        K_ser = K2 if world > 1 else K          # two gather sets alternate on N GPUs
        te_serial = timed_serial(K_ser) * K / K_ser
        te_serial_zc = timed_serial(K, e2e_step_zc) if world == 1 else None
        te_serial_zk = timed_serial(K, e2e_step_zk) if world == 1 else None
        gs.check_status()
        gs_e2e.check_status()
        # Output checks.  The serial path runs the dependent schedule and the
        # pipelined one the e2e schedule (other K splits, so other fp32
        # summation orders): each is checked bit for bit against a plain
        # device launch of its own configuration (N = 1) or against the other
        # requests of its own path (N > 1: every request computes the same
        # gathered product), and the two paths against each other within the
        # reference's rel_l2 gate.
        e2e_check = {}
        if world == 1:
            gs_dep.out.zero_()
            with torch.cuda.stream(stream):
                gs_dep.launch(0, stream)
            torch.cuda.synchronize(dev)
            want_s = gs_dep.out.cpu().view(torch.int16)
            e2e_check["serial_bit_exact"] = bool(torch.equal(hy.view(torch.int16), want_s))
            gs_zc.check_status()
            e2e_check["serial_zero_copy_bit_exact"] = bool(torch.equal(hy_zc.view(torch.int16), want_s))
            gs_zk.check_status()
            e2e_check["serial_copy_kernel_bit_exact"] = bool(torch.equal(hy_zk.view(torch.int16), want_s))
            if pipe is not None:
                g0 = pipe_copy["setups"][0]
                g0.out.zero_()
                with torch.cuda.stream(stream):
                    g0.launch(0, stream)
                torch.cuda.synchronize(dev)
                want_p = g0.out.cpu().view(torch.int16)
                for g_p in pipe_copy["setups"] + pipe_zc["setups"]:
                    g_p.check_status()
                e2e_check["pipelined_bit_exact"] = all(bool(torch.equal(h.view(torch.int16), want_p))
                                                       for h in pipe_copy["outs"] + pipe_zc["outs"])
        elif pipe is not None:
            for g_p in pipe["setups"]:
                g_p.check_status()
            first = pipe["outs"][0].view(torch.int16)
            e2e_check["pipelined_bit_exact"] = all(bool(torch.equal(h.view(torch.int16), first))
                                                   for h in pipe["outs"])
            pipe["fused"].close()
        if pipe is not None:
            a_ = hy.float()
            b_ = pipe["outs"][0].float()
            rel = float((a_ - b_).norm() / max(float(a_.norm()), 1e-30))
            e2e_check["serial_vs_pipelined"] = {"rel_l2": rel, "differing_elements": int((a_ != b_).sum())}
        e2e_ok = bool(all(v for kk, v in e2e_check.items() if isinstance(v, bool)) and
                      e2e_check.get("serial_vs_pipelined", {"rel_l2": 0.0})["rel_l2"] <= 2e-3)
        e2e_check["ok"] = e2e_ok
        te = pipe["t"] if pipe is not None else te_serial
        sched = pipe["plan"] if pipe is not None else gs_e2e.plan
        e2e = {"value": byt_job / (te / K) / 1e9, "unit": "GB/s",
               "output_check": e2e_check,
               "h2d_bytes_per_step": int(hin.numel()),
               "d2h_bytes_per_step": int(hy.numel() * 2),
               "us_per_step": te / K * 1e6,
               "requests_in_flight": pipe["depth"] if pipe is not None else 1,
               "serial": {"us_per_step": te_serial / K * 1e6,
                          "zero_copy_us_per_step": te_serial_zc / K * 1e6 if te_serial_zc is not None else None,
                          "copy_kernel_us_per_step": te_serial_zk / K * 1e6 if te_serial_zk is not None else None,
                          "note": "one request at a time on one stream, dependent schedule, CUDA graphs"
                                  + ("; zero_copy: the kernel writes the bf16 result into pinned host memory, "
                                     "no D2H copy node; copy_kernel: zero-copy output and the input copied by "
                                     "dg.copy_from_host under PDL instead of a copy node"
                                     if te_serial_zc is not None else "")},
               "output_to_host": ("zero-copy: the GEMM stores the bf16 result straight into pinned host "
                                  "memory over PCIe (dg.host_device_pointer), no D2H copy node; the result's "
                                  "bytes still cross PCIe every step"
                                  if pipe is not None and pipe.get("zero_copy") else "a D2H copy every step"),
               "variants_us_per_step": ({"d2h_copy": pipe_copy["t"] / K * 1e6, "zero_copy": pipe_zc["t"] / K * 1e6}
                                        if world == 1 and pipe is not None else None),
               "schedule": {"block_n": (pipe["cfg"] if pipe is not None else gs_e2e.cfg).block_n,
                            "grid": list(sched.grid), "cluster": sched.cluster,
                            "pdl_mode": args.e2e_schedule if pipe is not None else "dependent",
                            "gather_protocol": args.gather_protocol if world > 1 and pipe is not None else None},
               "path": "one pinned H2D copy of activation + scales, "
                       + ("dg.launch_gather (GEMM with the fused NVLink all-gather), D2H of the gathered "
                          "bf16 [M, g*N] output" if world > 1 else
                          "dg.launch_with_maps, the bf16 output to pinned host memory "
                          + ("written by the kernel (zero-copy)" if pipe is not None and pipe.get("zero_copy")
                             else "by a D2H copy"))
                       + ", every step" + ("" if pipe is None else
                                           f"; {pipe['depth']} requests in flight on as many streams" if world == 1 else
                                           "; pipelined: the fused GEMMs on one stream in the same order on every "
                                           f"rank in groups of {pipe['depth'] // 2} (PDL inside a group), H2D and "
                                           "D2H copies on two copy streams beside them "
                                           f"({pipe['depth']} input slots and gathered buffer sets)")}

    if fused is not None:
        torch.cuda.synchronize(dev)
        fused.close()
    if e2e is not None and world > 1 and fused_e is not None:
        fused_e.close()

    # ---- M sweep (M in 1..128), one GPU, headline mode ----
    sweep = None
    if not args.no_sweep and world == 1:
        sweep = []
        steps_s = min(K, 1000)
        for mm in (1, 2, 4, 8, 16, 32, 64, 128):
            qx_m, as_m, _ = act(mm)
            cfg_m = default_config(mm, n, k, layout=layout, pdl=pdl, independent_inputs=independent)
            gs_m = GemmSetup(rotation(cfg_m.block_n), cfg_m, mm, qx_m, wscale, as_m, dev)
            graphs = capture(lambda i: gs_m.launch(i, stream), steps_s)
            t_m = timed(graphs)
            del graphs
            gs_m.check_status()
            b_m = n * k + mm * k + 2 * mm * n
            gbs = b_m / (t_m / steps_s) / 1e9
            sweep.append({"M": mm, "us_per_gemm": t_m / steps_s * 1e6, "GBps": gbs, "frac_of_peak": gbs / peak,
                          "block": gs_m.plan.block[0], "mma_m": gs_m.plan.mma_m})
            del gs_m

    # ---- 61-layer decode chain with a true data dependency:
    # layers alternate N x K = 7168 x 16384 ("down", the C2 shape) and
    # 16384 x 7168 ("up"); every layer is a GEMM launched with PDL in the
    # dependent mode (its activation is read only after the previous grid
    # completes, its weights are prefetched before) whose bf16 output is
    # quantised into the next layer's e4m3 activation and 1x128 block scales.
    # Two variants, the faster one the headline: "fused" quantises in the
    # GEMM's cluster reduction (dg.launch_quantized, one kernel per layer,
    # 256-row tiles); "separate" runs the GPU quantiser as its own PDL launch
    # after the GEMM (two kernels per layer, the default tiles).  Each layer
    # has its own weight copy (7.2 GB, cold).
    chain = None
    chain_last = {}
    if not args.no_chain and world == 1:
        layers = 61
        passes = max(3, min(20, K // 500))
        dn = (n, k)
        up = (k, n)
        shapes = [dn if li % 2 == 0 else up for li in range(layers)]
        bytes_layer = sum(nn * kk + m * kk + 2 * m * nn for (nn, kk) in shapes) / layers
        raw = {}
        for (nn, kk) in (dn, up):
            gw = torch.Generator(device=dev).manual_seed(1000 + nn)
            wq, ws_ = quantize_pertensor(torch.randn((nn, kk), device=dev, generator=gw), torch.float8_e4m3fn)
            # Weight scales carry 1/sqrt(K), as a trained layer's output keeps the
            # size of its input: 61 unnormalised N(0,1) layers would grow by
            # ~sqrt(K) each and overflow bf16 within ~20 layers.
            raw[(nn, kk)] = (wq, torch.full(((nn + 127) // 128, kk // 128), float(ws_) / math.sqrt(kk), device=dev))
        q0, s0 = dg.quantize_activation(torch.randn((m, k), device=dev, generator=gx).bfloat16())
        chain = {"layers": layers, "passes_timed": passes, "shapes": "alternating 7168x16384 / 16384x7168"}
        for variant in ("separate", "fused"):
            base = {}
            for sh in (dn, up):
                cfg_l = default_config(m, *sh, layout=layout, pdl=pdl, independent_inputs=False)
                fq = variant == "fused"
                if fq:
                    cfg_l = default_config(m, *sh, layout=layout, pdl=pdl, independent_inputs=False,
                                           quantized_output=True)
                wq = raw[sh][0]
                base[sh] = (wq if layout == dg.LAYOUT_RAW else dg.prepack_weight(wq, cfg_l.block_n, layout), cfg_l,
                            fq)
            weights = [base[sh][0].clone() for sh in shapes]
            act_in = {w_: torch.zeros((m, w_), dtype=torch.uint8, device=dev) for w_ in (k, n)}
            act_sc = {w_: torch.zeros((m, w_ // 128), device=dev) for w_ in (k, n)}
            outs = {w_: torch.empty((m, w_), dtype=torch.bfloat16, device=dev) for w_ in (n, k)}
            act_in[k].copy_(q0)
            act_sc[k].copy_(s0)
            plans = {sh: base[sh][1].plan(m, *sh) for sh in (dn, up)}
            ws_c = torch.zeros(max(max(pl.ws_floats for pl in plans.values()), 1), device=dev)
            sem_c = torch.zeros(max(max(pl.sem_ints for pl in plans.values()), 1), dtype=torch.int32, device=dev)
            st_c = torch.zeros(1, dtype=torch.int32, device=dev)
            steps_c = []
            for li, (nn, kk) in enumerate(shapes):
                cfg_l = base[(nn, kk)][1]
                pr = dg.Problem(m, nn, kk, act_in[kk], weights[li], raw[(nn, kk)][1], act_sc[kk], outs[nn], ws_c,
                                sem_c, st_c)
                steps_c.append((cfg_l, pr, dg.make_weight_tma(cfg_l, pr), dg.make_activation_tma(cfg_l, pr), nn,
                                base[(nn, kk)][2]))

            def chain_step(i, steps_c=steps_c, act_in=act_in, act_sc=act_sc, outs=outs):
                cfg_l, pr, wm_, am_, nn, fused_q = steps_c[i % layers]
                if fused_q:
                    rc = dg.launch_quantized(cfg_l, pr, wm_, am_, act_in[nn], act_sc[nn], stream, pdl_attr=cfg_l.pdl)
                else:
                    rc = dg.launch_with_maps(cfg_l, pr, wm_, am_, stream, pdl_attr=cfg_l.pdl)
                if rc != 0:
                    raise RuntimeError(f"chain launch failed: cudaError {rc}")
                if not fused_q:
                    dg.quantize_activation(outs[nn], out=act_in[nn], scales=act_sc[nn], stream=stream, pdl_attr=True)
            graphs = capture(chain_step, layers * passes)
            t_chain = timed(graphs)
            del graphs
            if int(st_c.item()) != 0:
                raise RuntimeError(f"chain status {dg.status_string(int(st_c.item()))}")
            per_layer = t_chain / (layers * passes)
            # The last layer's input activation and scales, its bf16 output and the
            # quantiser's bytes of that output are still in their buffers: the
            # CPU leg below checks them against the oracle.
            ln, lk = shapes[(layers * passes - 1) % layers]
            chain_last[variant] = {"shape": (ln, lk), "act": act_in[lk].clone(), "act_scales": act_sc[lk].clone(),
                                   "out": outs[ln].clone(), "q": act_in[ln].clone(), "q_scales": act_sc[ln].clone(),
                                   "w": raw[(ln, lk)][0], "w_scales": raw[(ln, lk)][1]}
            chain[variant] = {
                "us_per_layer": per_layer * 1e6, "GBps": bytes_layer / per_layer / 1e9,
                "frac_of_peak": bytes_layer / per_layer / 1e9 / peak,
                "block_n": {f"{sh[0]}x{sh[1]}": base[sh][1].block_n for sh in (dn, up)},
                "quantisation": {f"{sh[0]}x{sh[1]}": "fused" if base[sh][2] else "separate" for sh in (dn, up)}}
            del weights, steps_c, base
        # headline: the fastest variant (all three are checked against the oracle)
        best = min(("separate", "fused"), key=lambda v: chain[v]["us_per_layer"])
        chain.update({key: chain[best][key] for key in ("us_per_layer", "GBps", "frac_of_peak")})
        chain["variant"] = best
        chain["per_layer"] = ("GEMM launched with PDL in the dependent mode (weights before griddepcontrol.wait, "
                              "activation after); its bf16 output quantised into the next layer's e4m3 activation "
                              "and 1x128 scales either in the GEMM's cluster reduction (fused, dg.launch_quantized: "
                              "one kernel, 256-row tiles) or by the GPU quantiser as a second PDL launch (separate)")

    # ---- the 61-layer decode chain on N GPUs (tensor parallel, strong scaling):
    # the same layers as chain_61, each full matrix N-sharded over the ranks;
    # every layer is the fused GEMM + gather in tagged lines
    # (dg_launch_gather_lines, dependent mode, PDL) followed by the GPU
    # quantiser of the gathered [M, N] output into the next layer's activation
    # on every rank.  Each shape has its own gather (two line-buffer sets
    # alternating per use), every rank makes the same launches in the same
    # order.  Rank 0 checks the last layer's gathered output against the
    # oracle in the CPU leg below.
    chain_tp = None
    chain_tp_last = {}
    if not args.no_chain and world > 1 and n % (world * 128) == 0 and k % (world * 128) == 0:
        from decode_opt_b200 import tp as dg_tp
        layers = 61
        passes = max(3, min(20, K // 500))
        # A gather's two sets must alternate on every use, also across graph
        # replays: an even number of passes and graphs of whole pairs of
        # passes give every gather an even number of uses per graph (each
        # graph starts on set 0 and ends on set 1).
        passes_t = passes + passes % 2
        dn = (n, k)
        up = (k, n)
        shapes = [dn if li % 2 == 0 else up for li in range(layers)]
        bytes_layer_t = sum(nn * kk + m * kk + 2 * m * nn for (nn, kk) in shapes) / layers
        full = {}
        for (nn, kk) in (dn, up):
            gw = torch.Generator(device=dev).manual_seed(1000 + nn)      # the same full matrix on every rank
            wq, ws_ = quantize_pertensor(torch.randn((nn, kk), device=dev, generator=gw), torch.float8_e4m3fn)
            full[(nn, kk)] = (wq, torch.full(((nn + 127) // 128, kk // 128), float(ws_) / math.sqrt(kk), device=dev))
        q0, s0 = dg.quantize_activation(torch.randn((m, k), device=dev, generator=gx).bfloat16())
        chain_tp = {"layers": layers, "passes_timed": passes_t, "gpus": world,
                    "shapes": "alternating 7168x16384 / 16384x7168, each N-sharded over the GPUs"}
        for variant in ("separate", "fused"):
            fused_q = variant == "fused"
            act_in = {w_: torch.zeros((m, w_), dtype=torch.uint8, device=dev) for w_ in (k, n)}
            act_sc = {w_: torch.zeros((m, w_ // 128), device=dev) for w_ in (k, n)}
            act_in[k].copy_(q0)
            act_sc[k].copy_(s0)
            base = {}
            for (nn, kk) in (dn, up):
                wq, sc_full = full[(nn, kk)]
                n_loc = nn // world
                lo = rank * n_loc
                cfg_l = default_config(m, n_loc, kk, layout=layout, pdl=pdl, independent_inputs=False,
                                       gather_lines=True)
                w_loc = wq[lo:lo + n_loc].contiguous()
                fg = dg_tp.FusedGather(m, n_loc, device=dev, protocol="lines")
                desc = [fg.descriptor(j, act_in[nn], act_sc[nn]) if fused_q else fg.descriptor(j) for j in (0, 1)]
                base[(nn, kk)] = {"w": w_loc if layout == dg.LAYOUT_RAW else dg.prepack_weight(w_loc, cfg_l.block_n,
                                                                                               layout),
                                  "sc": sc_full[lo // 128:(lo + n_loc) // 128].contiguous(), "cfg": cfg_l,
                                  "fg": fg, "desc": desc, "n_loc": n_loc}
            weights = [base[sh]["w"].clone() for sh in shapes]
            st_t = torch.zeros(1, dtype=torch.int32, device=dev)
            steps_t = []
            for li, (nn, kk) in enumerate(shapes):
                b = base[(nn, kk)]
                pr = dg.Problem(m, b["n_loc"], kk, act_in[kk], weights[li], b["sc"], act_sc[kk], None, None, None,
                                st_t)
                steps_t.append((b, pr, dg.make_weight_tma(b["cfg"], pr), dg.make_activation_tma(b["cfg"], pr), nn))
            uses = {dn: 0, up: 0}
            last_set = {}

            def chain_tp_step(i, steps_t=steps_t, uses=uses, last_set=last_set, fused_q=fused_q, act_in=act_in,
                              act_sc=act_sc):
                b, pr, wm_, am_, nn = steps_t[i % layers]
                sh = shapes[i % layers]
                j = uses[sh] % 2          # this gather's buffer set: alternates per use
                uses[sh] += 1
                last_set[sh] = j
                rc = dg.launch_gather(b["cfg"], pr, b["desc"][j], wm_, am_, stream, pdl_attr=b["cfg"].pdl)
                if rc != 0:
                    raise RuntimeError(f"tensor-parallel chain launch failed: cudaError {rc}")
                if not fused_q:
                    dg.quantize_activation(b["fg"].output(j, m), out=act_in[nn], scales=act_sc[nn], stream=stream,
                                           pdl_attr=True)
            graphs = []
            with torch.cuda.stream(stream):
                for base_i in range(0, layers * passes_t, 8 * layers):
                    gr = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(gr, stream=stream):
                        for i in range(base_i, min(layers * passes_t, base_i + 8 * layers)):
                            chain_tp_step(i)
                    graphs.append(gr)
            assert all(u % 2 == 0 for u in uses.values())
            t_ct = timed(graphs)
            del graphs
            if int(st_t.item()) != 0:
                raise RuntimeError(f"tensor-parallel chain status {dg.status_string(int(st_t.item()))}")
            per_layer_t = t_ct / (layers * passes_t)
            ln, lk = shapes[(layers * passes_t - 1) % layers]
            if rank == 0:
                bl = base[(ln, lk)]
                chain_tp_last[variant] = {"shape": (ln, lk), "act": act_in[lk].clone(),
                                          "act_scales": act_sc[lk].clone(),
                                          "out": bl["fg"].output(last_set[(ln, lk)], m).clone(),
                                          "q": act_in[ln].clone(), "q_scales": act_sc[ln].clone(),
                                          "w": full[(ln, lk)][0], "w_scales": full[(ln, lk)][1]}
            chain_tp[variant] = {
                "us_per_layer": per_layer_t * 1e6, "GBps_job": bytes_layer_t / per_layer_t / 1e9,
                "kernels_per_layer": 1 if fused_q else 2,
                "per_layer": ("GEMM of this rank's N/g rows with the all-gather fused in tagged lines "
                              "(dg_launch_gather_lines, dependent mode, PDL) whose unpack also writes the next "
                              "layer's e4m3 activation and 1x128 scales, on every rank") if fused_q else
                             ("the same GEMM + gather, then the GPU quantiser of the gathered [M, N] output "
                              "(PDL), on every rank")}
            torch.cuda.synchronize(dev)
            for sh in (dn, up):
                base[sh]["fg"].close()
            del weights, steps_t, base
        best_t = min(("separate", "fused"), key=lambda v: chain_tp[v]["us_per_layer"])
        chain_tp.update({"us_per_layer": chain_tp[best_t]["us_per_layer"],
                         "GBps_job": chain_tp[best_t]["GBps_job"], "variant": best_t})
        del full

    # ---- cuBLASLt FP8 (torch._scaled_mm) on the same cold weights: a reported
    # library baseline with per-tensor scales (no 128-block scales), M padded
    # to 16 rows.
    cublas = None
    if rank == 0 and world == 1 and not args.no_cublas:
        try:
            m16 = max(16, (m + 15) // 16 * 16)
            a16 = torch.zeros((m16, k), dtype=torch.float8_e4m3fn, device=dev)
            a16[:m] = qx.view(torch.float8_e4m3fn)
            raw_sets = [qw.view(torch.float8_e4m3fn)] + [qw.view(torch.float8_e4m3fn).clone()
                                                         for _ in range(rot.nsets - 1)]
            sa = torch.tensor(sx, device=dev)
            sb = torch.tensor(float(sw), device=dev)

            def cub(i):
                torch._scaled_mm(a16, raw_sets[i % len(raw_sets)].t(), scale_a=sa, scale_b=sb,
                                 out_dtype=torch.bfloat16)
            # Eager calls first: cuBLASLt picks its algorithm and workspace
            # outside the graph capture.
            with torch.cuda.stream(stream):
                for i in range(3):
                    cub(i)
            torch.cuda.synchronize(dev)
            graphs = capture(cub, K)
            t_c = timed(graphs)
            del graphs
            cublas = {"us_per_gemm": t_c / K * 1e6, "GBps": byt_gpu / (t_c / K) / 1e9,
                      "call": f"torch._scaled_mm e4m3 [{m16}x{k}] x [{k}x{n}] per-tensor scales, bf16 out"}
            # The same GEMM with this problem's block scales: 1x128 on the
            # activation, 128x128 on the weights (cuBLASLt VEC128 / BLK128x128).
            sa_blk = torch.full((m16, kb), sx, device=dev)
            sb_blk = wscale.t()                     # (K/128, N/128) view
            blk = None
            for name, sa_v, sb_v in (("row-major scales", sa_blk.contiguous(), sb_blk.contiguous()),
                                     ("outer-dim-major scales", sa_blk.t().contiguous().t(), sb_blk)):
                try:
                    torch._scaled_mm(a16, raw_sets[0].t(), scale_a=sa_v, scale_b=sb_v, out_dtype=torch.bfloat16)
                    torch.cuda.synchronize(dev)
                    blk = (name, sa_v, sb_v)
                    break
                except Exception as exc:  # noqa: BLE001 - try the next scale layout
                    last_err = f"{type(exc).__name__}: {exc}"[:200]
            if blk is None:
                cublas["blockwise_torch"] = {"unavailable": last_err}
            else:
                def cub_blk(i):
                    torch._scaled_mm(a16, raw_sets[i % len(raw_sets)].t(), scale_a=blk[1], scale_b=blk[2],
                                     out_dtype=torch.bfloat16)
                with torch.cuda.stream(stream):
                    for i in range(3):
                        cub_blk(i)
                torch.cuda.synchronize(dev)
                graphs = capture(cub_blk, K)
                t_b = timed(graphs)
                del graphs
                cublas["blockwise_torch"] = {"us_per_gemm": t_b / K * 1e6, "GBps": byt_gpu / (t_b / K) / 1e9,
                                             "call": f"torch._scaled_mm e4m3 1x128 activation / 128x128 weight "
                                                     f"block scales ({blk[0]}), M padded to {m16}"}
            del raw_sets
        except Exception as exc:  # noqa: BLE001 - reported, not fatal
            cublas = {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}
        # The CUDA toolkit's cuBLASLt (whose header declares the 128-block
        # scale modes torch's bundled build refuses) in its own process: the
        # reference's scale layout (CUBLASLT_MATMUL_MATRIX_SCALE_BLK128x128_32F
        # on the weights, VEC128_32F on the activation) and per-tensor, each
        # checked against an fp32 reference before it is timed, at the
        # reference's baseline batch sizes (results/baseline_cublaslt.csv).
        cublas["toolkit_cublaslt"] = cublaslt_driver(n, k, sorted({1, 8, 64, 128, m}), dev)
        blk_rows = [r for r in cublas["toolkit_cublaslt"].get("block", []) if r.get("M") == m]
        if blk_rows and "us_per_gemm" in blk_rows[0]:
            cublas["blockwise"] = {"us_per_gemm": blk_rows[0]["us_per_gemm"], "GBps": blk_rows[0]["GBps"],
                                   "call": f"cuBLASLt {blk_rows[0]['cublaslt']} e4m3 BLK128x128 weight / VEC128 "
                                           f"activation scales, M={m}, bf16 out"}
        elif blk_rows:
            cublas["blockwise"] = {"unavailable": blk_rows[0].get("unavailable", "no result")}

    # ---- CPU baseline on rank 0 (N = 1 only), also the parity check -----------
    cpu = None
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        run, kind = cpu_gemm_fn()
        w_h = qw.view(torch.uint8).cpu().numpy()
        a_h = qx.view(torch.uint8).cpu().numpy()
        ws_h = wscale.cpu().numpy()
        as_h = ascale.cpu().numpy()
        # parity of the benchmarked launch: one launch on set 0 against the
        # reference GEMM on the same bytes
        gs.out.zero_()
        gs_other.out.zero_()
        with torch.cuda.stream(stream):
            gs.launch(0, stream)
            gs_other.launch(0, stream)
        torch.cuda.synchronize(dev)
        got = gs.out.float().cpu().numpy()
        got_other = gs_other.out.float().cpu().numpy()
        threads = 1
        t0 = time.perf_counter()
        want = None
        reps = 0
        while True:
            want_i = cpu_parallel_gemm(run, a_h, as_h, w_h, ws_h, threads)
            reps += 1
            if want is None:
                want = want_i
            if time.perf_counter() - t0 >= args.cpu_seconds:
                break
        dt = (time.perf_counter() - t0) / reps
        cpu_bytes = n * k + m * k + 2 * m * n
        cpu = {"value": cpu_bytes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": kind,
               "sample": f"{reps} full GEMM(s) N={n} K={k} M={m}, single thread, "
                         f"{dt * 1e3:.1f} ms per GEMM"}
        ok, worst = oracle.elementwise_ok(got, want)
        ok_o, worst_o = oracle.elementwise_ok(got_other, want)
        parity = {"rel_l2": oracle.rel_l2(got, want), "max_rel_err_floored": worst, "ok": bool(ok),
                  "other_pdl_mode": {"rel_l2": oracle.rel_l2(got_other, want), "max_rel_err_floored": worst_o,
                                     "ok": bool(ok_o)}}
        for variant, cl in chain_last.items():
            # The timed chain's last layer: its GEMM against the oracle on the
            # bytes it read, and its quantisation bit for bit.
            got_c = cl["out"].float().cpu().numpy()
            want_c = oracle.compute_reference(cl["act"].cpu().numpy(), cl["act_scales"].cpu().numpy(),
                                              cl["w"].view(torch.uint8).cpu().numpy(),
                                              cl["w_scales"].cpu().numpy(), threads=os.cpu_count() or 1)
            ok_c, worst_c = oracle.elementwise_ok(got_c, want_c)
            rl2_c = oracle.rel_l2(got_c, want_c)
            want_q, want_s = oracle.quantize_rows(got_c)
            q_ok = bool(np.array_equal(cl["q"].cpu().numpy(), want_q) and
                        np.array_equal(cl["q_scales"].cpu().numpy(), want_s))
            chain[variant]["parity"] = {"layer": f"last ({cl['shape'][0]}x{cl['shape'][1]})", "rel_l2": rl2_c,
                                        "max_rel_err_floored": worst_c, "quantisation_bit_exact": q_ok,
                                        "ok": bool(ok_c and rl2_c <= oracle.REL_L2_GATE and q_ok)}
        if chain is not None and "parity" in chain.get(chain.get("variant", ""), {}):
            chain["parity"] = chain[chain["variant"]]["parity"]

    if rank == 0 and chain_tp_last and not args.no_cpu_baseline:
        # The tensor-parallel chain's last layer, each variant: its gathered
        # output against the oracle on the full matrix and the bytes it read,
        # and its quantisation bit for bit.
        import oracle
        for variant, cl in chain_tp_last.items():
            got_t = cl["out"].float().cpu().numpy()
            want_t = oracle.compute_reference(cl["act"].cpu().numpy(), cl["act_scales"].cpu().numpy(),
                                              cl["w"].view(torch.uint8).cpu().numpy(), cl["w_scales"].cpu().numpy(),
                                              threads=os.cpu_count() or 1)
            ok_t, worst_t = oracle.elementwise_ok(got_t, want_t)
            rl2_t = oracle.rel_l2(got_t, want_t)
            want_qt, want_st = oracle.quantize_rows(got_t)
            q_ok_t = bool(np.array_equal(cl["q"].cpu().numpy(), want_qt) and
                          np.array_equal(cl["q_scales"].cpu().numpy(), want_st))
            chain_tp[variant]["parity"] = {"layer": f"last ({cl['shape'][0]}x{cl['shape'][1]}, gathered)",
                                           "rel_l2": rl2_t, "max_rel_err_floored": worst_t,
                                           "quantisation_bit_exact": q_ok_t,
                                           "ok": bool(ok_t and rl2_t <= oracle.REL_L2_GATE and q_ok_t)}
        chain_tp["parity"] = chain_tp[chain_tp["variant"]].get("parity")

    if world > 1:
        dist.barrier()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": K,
        "warmup": args.warmup,
        "ms_per_step": us_gemm / 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8e4m3-in/f32-acc/bf16-out",
        "data": "synthetic",
        "config": {
            "workload": f"C2 decode GEMM N={n} K={k} M={m}, cold weights"
                        + (f"; x{world} GPUs, each a {n}-row shard of an N={world * n} tensor-parallel layer"
                           if world > 1 else ""),
            "M": m, "N": n, "K": k, "layout": args.layout, "block_n": cfg.block_n, "subs": cfg.subs,
            "stages": gs.plan.stages, "grid": list(gs.plan.grid), "threads_per_cta": gs.plan.block[0],
            "batch_class": ("swap_ab" if cfg.flags & dg.FLAG_SWAP_AB else "default"),
            "mma": f"{gs.plan.mma_m}x{gs.plan.n_mma}x32",
            "pdl": cfg.pdl, "pdl_mode": args.pdl_mode, "rotation_sets": rot.nsets,
            "working_set_bytes": rot.nsets * rot.set_bytes, "l2_bytes": rot.l2,
            "cold": "inputs larger than L2 (rotated weight copies), no flush",
            "timing": "CUDA events around CUDA-graph replays of K launches, max over ranks",
        },
        "us_per_gemm": us_gemm,
        "pdl_mode": args.pdl_mode,
        "other_pdl_mode": {"mode": "dependent" if independent else "independent",
                           "us_per_gemm": t_other / K * 1e6, "GBps_per_gpu": byt_gpu / (t_other / K) / 1e9,
                           "block_n": cfg_other.block_n, "grid": list(gs_other.plan.grid),
                           "cluster": gs_other.plan.cluster},
        "schedule": {"kind": "cluster split-K" if cfg.grid_ctas == dg.GRID_CLUSTER else "stream-K",
                     "cluster": gs.plan.cluster, "ctas": gs.plan.num_ctas,
                     "pdl_modes": "independent: the reference's B2B+PDL protocol (the same GEMM repeated; the "
                                  "reference kernel never waits on the grid dependency), activations read before "
                                  "griddepcontrol.wait, writes after; consecutive GEMMs stream side by side on "
                                  "disjoint SMs, so us_per_gemm is the steady-state period (throughput), not one "
                                  "GEMM's latency. dependent: every GEMM reads its activation only after the "
                                  "previous grid completed (a layer chain): latency-bound"},
        "pct_of_spec_8TBs": achieved / SPEC_HBM_GBS,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "traffic": ncu_traffic(workload_key), "algorithmic_bytes_per_launch": byt_gpu},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "gpu_launches": K,
        "clocks": clocks.summary(),
        "parity": parity,
        "m_sweep": sweep,
        "cublaslt_fp8": cublas,
        "tensor_parallel": tp,
        # BASELINE config 5 as strong scaling: the one N x K layer split over
        # the ranks (also inside tensor_parallel), at the headline M and at
        # M = 1, 8, 64.
        "strong_scaling": tp.get("strong_scaling") if tp else None,
        "chain_61": chain,
        "chain_61_tp": chain_tp,
    }
    print(json.dumps(line), file=JSON_OUT, flush=True)


def main():
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("run N>1 under torch.distributed.run (one rank per GPU)")
    if world > 1:
        # stdout carries exactly one JSON line: keep the real stdout for it and
        # point file descriptor 1 at stderr, so that whatever libraries print
        # there (NCCL's version banner, for one) goes to stderr.
        global JSON_OUT
        sys.stdout.flush()
        JSON_OUT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)
        import datetime
        import torch.distributed as dist
        backend = "nccl" if args.impl == "b200" else "gloo"
        if backend == "nccl":
            import torch
            torch.cuda.set_device(local_rank)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=120))
    try:
        if args.impl == "reference":
            reference_arm(args, rank, world)
        else:
            b200_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
