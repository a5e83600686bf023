"""Measurement probes behind the kernel's design choices, through the C ABI.

    python -m decode_opt_b200.probe [--json]

* ``mma``: tcgen05.mma kind::f8f6f4 issue and completion cost per shape
  (``dg_probe_mma``): the fixed per-instruction cost that puts the weights on
  the MMA's N side with N = 256.
* ``hbm``: achievable HBM read bandwidth for the decode GEMM's bytes (the
  rebuild of the reference's tools/peak_bw_probe.cu:82-211): the cp.async.bulk
  stream (``dg_probe_bulk_stream``) and 16-byte ld.global.nc reads
  (``dg_probe_naive_read``) over a rotation of cold 117 MB buffers (>= 1 GiB
  in total), one launch alone and back to back in a CUDA graph, plus the L2
  self-test (a 96 MiB buffer re-read) that must read far above HBM speed.
"""

from __future__ import annotations

import argparse
import ctypes
import json

from . import _lib

N, K = 7168, 16384          # the C2 weight matrix: 117,440,512 bytes per launch


def mma_cost(mma_m: int, mma_n: int, iters: int = 4096, accumulators: int = 1, ctas: int = 1):
    """(issue, completion) cycles per MMA, mean over CTAs."""
    import torch
    out = torch.full((2 * ctas,), -1, dtype=torch.int64, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = _lib.lib().dg_probe_mma(mma_m, mma_n, iters, accumulators, ctas, out.data_ptr(), status.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
    if rc != 0:
        raise RuntimeError(f"dg_probe_mma({mma_m}, {mma_n}) failed: cudaError {rc}")
    torch.cuda.synchronize()
    if int(status.item()) != 0:
        raise RuntimeError(f"dg_probe_mma status {int(status.item()):#x}")
    v = out.view(ctas, 2).double().mean(0).tolist()
    return v[0] / iters, v[1] / iters


def mma_table():
    rows = []
    for m in (64, 128):
        for n in (16, 32, 64, 128, 256):
            for acc, ctas in ((1, 1), (2, 1), (1, 148)):
                if acc * n > 512:
                    continue
                issue, done = mma_cost(m, n, accumulators=acc, ctas=ctas)
                rows.append({"mma_m": m, "mma_n": n, "accumulators": acc, "ctas": ctas,
                             "issue_cycles": issue, "complete_cycles": done,
                             "weight_bytes_per_cycle": n * 32 / done, "mac_per_cycle": m * n * 32 / done})
    return rows


def _graph_us(launch, count: int, iters: int) -> float:
    """Mean microseconds per launch: `iters` launches captured in a graph."""
    import torch
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(3):
            launch(i, s.cuda_stream)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(iters):
            launch(i, s.cuda_stream)
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
    return best


def _single_us(launch) -> float:
    import torch
    ts = []
    for i in range(5):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        launch(i, torch.cuda.current_stream().cuda_stream)
        e1.record()
        torch.cuda.synchronize()
        ts.append(e0.elapsed_time(e1) * 1e3)
    return sorted(ts)[len(ts) // 2]


def hbm_table():
    import torch
    L = _lib.lib()
    nbytes = N * K
    nsets = 10
    bufs = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(nsets)]
    for i, b in enumerate(bufs):
        b.fill_(i + 1)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    sink = torch.zeros(1, dtype=torch.int64, device="cuda")
    sms = L.dg_num_sms()
    rows = []

    def bulk(op, stages):
        return lambda i, s: L.dg_probe_bulk_stream(bufs[i % nsets].data_ptr(), nbytes, op, sms, stages,
                                                   status.data_ptr(), sink.data_ptr(), s)

    def naive(bps):
        return lambda i, s: L.dg_probe_naive_read(bufs[i % nsets].data_ptr(), nbytes, bps, sink.data_ptr(), s)

    probes = [(f"bulk_stream op={op // 1024}KiB stages={st}", bulk(op, st))
              for op, st in ((16384, 4), (32768, 2), (32768, 3), (65536, 2), (49152, 2))]
    probes += [(f"naive_read {b} blocks/SM", naive(b)) for b in (2, 4)]
    for name, fn in probes:
        single = _single_us(fn)
        b2b = _graph_us(fn, nsets, 90)
        rows.append({"probe": name, "bytes": nbytes, "single_us": single, "single_GBps": nbytes / single / 1e3,
                     "b2b_us": b2b, "b2b_GBps": nbytes / b2b / 1e3})
    # L2 self-test: a 96 MiB buffer read over and over stays in the 126 MB L2.
    small = 96 << 20
    fn = lambda i, s: L.dg_probe_bulk_stream(bufs[0].data_ptr(), small, 32768, sms, 3, status.data_ptr(),
                                             sink.data_ptr(), s)
    b2b = _graph_us(fn, 1, 200)
    rows.append({"probe": "L2 self-test bulk_stream 96 MiB", "bytes": small, "b2b_us": b2b,
                 "b2b_GBps": small / b2b / 1e3})
    if int(status.item()) != 0:
        raise RuntimeError(f"probe status {int(status.item()):#x}")
    return rows


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--json", action="store_true", help="one JSON object instead of tables")
    args = ap.parse_args(argv)
    mma = mma_table()
    hbm = hbm_table()
    if args.json:
        print(json.dumps({"mma": mma, "hbm": hbm}))
        return
    print("tcgen05.mma kind::f8f6f4, K=32, cycles per instruction (clock64, mean over CTAs)")
    print(f"{'M':>4} {'N':>4} {'acc':>4} {'ctas':>5} {'issue':>8} {'complete':>9} {'W B/cyc':>8} {'MAC/cyc':>8}")
    for r in mma:
        print(f"{r['mma_m']:>4} {r['mma_n']:>4} {r['accumulators']:>4} {r['ctas']:>5} {r['issue_cycles']:>8.1f} "
              f"{r['complete_cycles']:>9.1f} {r['weight_bytes_per_cycle']:>8.1f} {r['mac_per_cycle']:>8.0f}")
    print("\nHBM read probes over 10 rotating 117 MB buffers (cold), CUDA events")
    for r in hbm:
        single = f"single {r['single_us']:.2f} us {r['single_GBps']:.0f} GB/s | " if "single_us" in r else ""
        print(f"{r['probe']:36s} {single}b2b {r['b2b_us']:.2f} us {r['b2b_GBps']:.0f} GB/s")


if __name__ == "__main__":
    main()
