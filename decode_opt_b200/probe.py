"""Measurement probes behind the kernel's design choices, through the C ABI.

    python -m decode_opt_b200.probe [--json PATH] [--quick] [--skip-mma]

The rebuild of the reference's ``tools/peak_bw_probe.cu`` for sm_100a, plus the
tensor-core cost probe:

* ``hbm``: achievable HBM read bandwidth -- the denominator of "% of
  achievable bandwidth".  A read stream through a shared-memory ring with
  ``cp.async.bulk`` (``dg_probe_bulk_stream``: one issuing thread and one
  consuming thread per CTA) swept over op bytes x CTAs (1, 2, 4 per SM) x
  ring stages, as the reference sweeps op bytes x CTAs x stages
  (tools/peak_bw_probe.cu:71-75), and the naive control, 16-byte
  ``ld.global.nc`` with four loads in flight per thread over 1..8 blocks of
  512 threads per SM (``dg_probe_naive_read``, the reference's
  naive_read_nc).  Cold data: eight rotating 512 MiB buffers (4 GiB >> the
  126 MB L2), every launch reads a different one, timed with CUDA events
  around single launches (median of 7) and as an 8-launch batch.  The decode
  GEMM's own volume, 117 MB launches back to back in a CUDA graph, is
  reported beside it.
* ``l2_selftest``: the honesty gate (reference :190-211).  The same probes
  re-reading one 32 MiB buffer that stays in L2 must report far more than
  any HBM figure -- proof that the harness tells L2 hits from DRAM reads.
* ``mma``: tcgen05.mma kind::f8f6f4 cost per instruction (``dg_probe_mma``):
  1, 2 or 4 warps issue concurrently, each over 1, 2 or 4 independent TMEM
  accumulators, for the GEMM's shapes (M 64/128 x N 16..256) -- one issuing
  thread's per-instruction cost against the tensor pipe's throughput.

``--json PATH`` writes everything as one JSON document in the spirit of the
reference's results/peak_bw.json (spec, best measured figure and its
configuration, every configuration, the self-test, the method).
"""

from __future__ import annotations

import argparse
import json
import statistics

from . import _lib

SPEC_GBPS = 8000.0                       # B200 HBM3e (DGX figure)
GEMM_N, GEMM_K = 7168, 16384             # the C2 weight matrix: 117,440,512 bytes per launch
SWEEP_BYTES = 512 << 20                  # per launch
SWEEP_SETS = 8                           # 4 GiB of cold buffers
L2_SELFTEST_BYTES = 32 << 20
SMEM_PER_CTA = 227 * 1024


# ------------------------------------------------------------------- MMA ---
def mma_cost(mma_m: int, mma_n: int, iters: int = 4096, accumulators: int = 1, issuers: int = 1, ctas: int = 1):
    """(issue, completion) cycles per MMA (all issuers together), mean over CTAs."""
    import torch
    out = torch.full((2 * ctas,), -1, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().dg_probe_mma(mma_m, mma_n, iters, accumulators, issuers, ctas, out.data_ptr(),
                                 status.data_ptr(), torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"dg_probe_mma({mma_m}, {mma_n}) failed: cudaError {rc}")
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError(f"dg_probe_mma status {int(status.item()):#x}")
    v = out.view(ctas, 2).double().mean(0).tolist()
    n = (iters // issuers) * issuers
    return v[0] / n, v[1] / n


def mma_table(quick: bool = False):
    rows = []
    shapes = ([(64, n) for n in (16, 64, 256)] + [(128, n) for n in (16, 32, 64, 256)]) if quick else \
        ([(64, n) for n in (16, 32, 64, 128, 256)] + [(128, n) for n in (16, 32, 64, 128, 256)])
    for m, n in shapes:
        for issuers in (1, 2, 4):
            for acc in (1, 2, 4):
                if issuers * acc * n > 512 or (quick and acc == 2):
                    continue
                for ctas in ((1,) if quick else (1, 148)):
                    issue, done = mma_cost(m, n, accumulators=acc, issuers=issuers, ctas=ctas)
                    rows.append({"mma_m": m, "mma_n": n, "issuers": issuers, "accumulators_per_issuer": acc,
                                 "ctas": ctas, "issue_cycles": issue, "complete_cycles": done,
                                 "weight_bytes_per_cycle": n * 32 / done, "mac_per_cycle": m * n * 32 / done})
    return rows


# ------------------------------------------------------------------- HBM ---
def _events_us(fn, count: int) -> float:
    import torch
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    s = torch.cuda.current_stream()
    e0.record(s)
    for i in range(count):
        fn(i, s.cuda_stream)
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / count


def _single_and_batch(fn, rounds: int = 7, warm: int = 3, batch: int = 8):
    """Median single-launch us over `rounds`, and us per launch of a batch."""
    import torch
    for i in range(warm):
        fn(i, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    singles = []
    k = warm
    for _ in range(rounds):
        singles.append(_events_us(lambda i, s: fn(k + i, s), 1))
        k += 1
    batch_us = _events_us(lambda i, s: fn(k + i, s), batch)
    return statistics.median(singles), batch_us, singles


def _graph_us(fn, iters: int) -> float:
    """Mean us per launch over `iters` launches captured in one CUDA graph (best of 5)."""
    import torch
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i, s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(iters):
            fn(i, s.cuda_stream)
    best = None
    for _ in range(5):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(s):
            e0.record(s)
            g.replay()
            e1.record(s)
        torch.cuda.synchronize()
        t = e0.elapsed_time(e1) * 1e3 / iters
        best = t if best is None else min(best, t)
    del g
    return best


def hbm_sweep(quick: bool = False):
    """Returns (configs, naive, gemm_size, l2_selftest) lists of dicts."""
    import torch
    L = _lib.lib()
    sms = L.dg_num_sms()
    nsets = 3 if quick else SWEEP_SETS
    bufs = [torch.empty(SWEEP_BYTES, dtype=torch.uint8, device="cuda") for _ in range(nsets)]
    for i, b in enumerate(bufs):
        b.fill_(i + 1)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    sink = torch.zeros(1, dtype=torch.int64, device="cuda")

    def bulk(op, ctas, stages, nbytes=SWEEP_BYTES, rotate=True):
        def fn(i, s):
            b = bufs[i % nsets] if rotate else bufs[0]
            rc = L.dg_probe_bulk_stream(b.data_ptr(), nbytes - nbytes % op, op, ctas, stages, status.data_ptr(),
                                        sink.data_ptr(), s)
            if rc != 0:
                raise RuntimeError(f"dg_probe_bulk_stream failed: cudaError {rc}")
        return fn

    def naive(bps, nbytes=SWEEP_BYTES, rotate=True):
        def fn(i, s):
            b = bufs[i % nsets] if rotate else bufs[0]
            rc = L.dg_probe_naive_read(b.data_ptr(), nbytes, bps, sink.data_ptr(), s)
            if rc != 0:
                raise RuntimeError(f"dg_probe_naive_read failed: cudaError {rc}")
        return fn

    ops = (32768, 65536) if quick else (16384, 32768, 65536, 98304)
    per_sm = (1, 2) if quick else (1, 2, 4)
    stage_list = (2, 4) if quick else (2, 4, 8)
    configs = []
    for op in ops:
        for k in per_sm:
            for st in stage_list:
                row = {"op_bytes": op, "ctas": sms * k, "ctas_per_sm": k, "stages": st,
                       "smem_bytes": st * op, "launch_bytes": SWEEP_BYTES - SWEEP_BYTES % op}
                if st * op + 256 > SMEM_PER_CTA:
                    row.update(feasible=False, gbps=None, skip_reason="stages * op_bytes exceeds 227 KiB")
                    configs.append(row)
                    continue
                med, batch, rounds = _single_and_batch(bulk(op, sms * k, st))
                row.update(feasible=True, median_us=med, batch_us=batch, round_us=rounds,
                           gbps=row["launch_bytes"] / med / 1e3, batch_gbps=row["launch_bytes"] / batch / 1e3,
                           pct_of_spec=100.0 * row["launch_bytes"] / med / 1e3 / SPEC_GBPS)
                configs.append(row)
    naive_rows = []
    for bps in ((2, 4) if quick else (1, 2, 4, 8)):
        med, batch, rounds = _single_and_batch(naive(bps))
        naive_rows.append({"blocks_per_sm": bps, "threads": 512, "loads_in_flight_per_thread": 4,
                           "launch_bytes": SWEEP_BYTES, "median_us": med, "batch_us": batch, "round_us": rounds,
                           "gbps": SWEEP_BYTES / med / 1e3, "batch_gbps": SWEEP_BYTES / batch / 1e3,
                           "pct_of_spec": 100.0 * SWEEP_BYTES / med / 1e3 / SPEC_GBPS})
    # The decode GEMM's volume: 117 MB launches back to back (CUDA graph).
    gemm_bytes = GEMM_N * GEMM_K
    gemm_rows = []
    for name, fn in (("bulk_stream op=32KiB ctas=1/SM stages=3", bulk(32768, sms, 3, gemm_bytes)),
                     ("bulk_stream op=32KiB ctas=2/SM stages=3", bulk(32768, 2 * sms, 3, gemm_bytes)),
                     ("naive_read 4 blocks/SM", naive(4, gemm_bytes))):
        us = _graph_us(fn, 30 if quick else 90)
        gemm_rows.append({"probe": name, "launch_bytes": gemm_bytes, "b2b_us": us, "b2b_gbps": gemm_bytes / us / 1e3})
    # L2 self-test: one 32 MiB buffer re-read back to back stays in L2.
    l2 = []
    for name, fn in (("naive_read 4 blocks/SM", naive(4, L2_SELFTEST_BYTES, rotate=False)),
                     ("bulk_stream op=16KiB ctas=4/SM stages=2", bulk(16384, 4 * sms, 2, L2_SELFTEST_BYTES,
                                                                         rotate=False))):
        us = _graph_us(fn, 100 if quick else 400)
        l2.append({"probe": name, "bytes": L2_SELFTEST_BYTES, "b2b_us": us, "gbps": L2_SELFTEST_BYTES / us / 1e3})
    if int(status.item()) != 0:
        raise RuntimeError(f"probe status {int(status.item()):#x}")
    del bufs
    torch.cuda.empty_cache()
    return configs, naive_rows, gemm_rows, l2


def run(quick: bool = False, skip_mma: bool = False) -> dict:
    import torch
    configs, naive_rows, gemm_rows, l2 = hbm_sweep(quick)
    measured = [c for c in configs if c.get("feasible")] + naive_rows
    best = max(measured, key=lambda c: c["gbps"])
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    doc = {
        "spec_gbps": SPEC_GBPS,
        "measured_best_gbps": best["gbps"],
        "best": best,
        "l2_selftest_gbps": max(r["gbps"] for r in l2),
        "hbm_best_over_spec": best["gbps"] / SPEC_GBPS,
        "method": ("Cold reads of 512 MiB per launch from eight rotating buffers (4 GiB >> L2), CUDA events "
                   "around single launches (median of 7 after 3 warm-ups) and an 8-launch batch. "
                   "bulk_stream: per CTA one thread issues cp.async.bulk copies of op_bytes into a "
                   "stages-deep shared-memory ring (mbarrier complete_tx), one thread consumes a word of "
                   "every stage and frees it; swept over op bytes x CTAs (1, 2, 4 per SM) x stages, "
                   "combinations whose ring exceeds 227 KiB recorded as skipped. naive: 16-byte "
                   "ld.global.nc.L1::no_allocate, four loads in flight per thread, 512-thread blocks. "
                   "L2 self-test: the same probes re-reading one 32 MiB buffer back to back in a CUDA "
                   "graph must report far more than any HBM figure."),
        "configs": configs,
        "naive": naive_rows,
        "gemm_volume_back_to_back": gemm_rows,
        "l2_selftest": l2,
        "device": {"name": props.name, "sms": props.multi_processor_count, "l2_bytes": props.L2_cache_size},
    }
    if not skip_mma:
        doc["mma"] = mma_table(quick)
    return doc


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--json", metavar="PATH", help="write the results as one JSON document")
    ap.add_argument("--quick", action="store_true", help="a reduced sweep (the GPU test's)")
    ap.add_argument("--skip-mma", action="store_true", help="HBM probes only")
    args = ap.parse_args(argv)
    doc = run(args.quick, args.skip_mma)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(doc, f, indent=1)
    print("HBM read probes: 512 MiB per launch, rotating cold buffers, median of 7 single launches")
    print(f"{'op KiB':>7} {'CTAs':>5} {'/SM':>4} {'stages':>6} {'us':>9} {'GB/s':>8} {'batch GB/s':>11}")
    for c in doc["configs"]:
        if not c["feasible"]:
            print(f"{c['op_bytes'] // 1024:>7} {c['ctas']:>5} {c['ctas_per_sm']:>4} {c['stages']:>6}  skipped")
            continue
        print(f"{c['op_bytes'] // 1024:>7} {c['ctas']:>5} {c['ctas_per_sm']:>4} {c['stages']:>6} "
              f"{c['median_us']:>9.2f} {c['gbps']:>8.0f} {c['batch_gbps']:>11.0f}")
    for r in doc["naive"]:
        print(f"naive ld.global.nc {r['blocks_per_sm']} blocks/SM: {r['median_us']:.2f} us {r['gbps']:.0f} GB/s "
              f"(batch {r['batch_gbps']:.0f})")
    print(f"best: {doc['measured_best_gbps']:.0f} GB/s ({100 * doc['hbm_best_over_spec']:.1f} % of "
          f"{SPEC_GBPS:.0f} spec)")
    for r in doc["gemm_volume_back_to_back"]:
        print(f"117 MB back to back, {r['probe']}: {r['b2b_us']:.2f} us {r['b2b_gbps']:.0f} GB/s")
    for r in doc["l2_selftest"]:
        print(f"L2 self-test ({r['bytes'] >> 20} MiB re-read), {r['probe']}: {r['gbps']:.0f} GB/s")
    if "mma" in doc:
        print("\ntcgen05.mma kind::f8f6f4, K=32: cycles per instruction (all issuers together)")
        print(f"{'M':>4} {'N':>4} {'warps':>5} {'acc/w':>5} {'ctas':>5} {'issue':>8} {'complete':>9} "
              f"{'W B/cyc':>8} {'MAC/cyc':>8}")
        for r in doc["mma"]:
            print(f"{r['mma_m']:>4} {r['mma_n']:>4} {r['issuers']:>5} {r['accumulators_per_issuer']:>5} "
                  f"{r['ctas']:>5} {r['issue_cycles']:>8.1f} {r['complete_cycles']:>9.1f} "
                  f"{r['weight_bytes_per_cycle']:>8.1f} {r['mac_per_cycle']:>8.0f}")


if __name__ == "__main__":
    main()
