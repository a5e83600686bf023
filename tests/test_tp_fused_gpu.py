"""GPU tests of the GEMM with the tensor-parallel all-gather fused into the
kernel (dg_launch_gather).

* One GPU: the output-copy path with a row stride and a column offset (a
  world of one writing into a wider buffer); columns outside its slice keep
  their sentinel.
* One GPU: the lines protocol (dg_launch_gather_lines) with a world of one,
  and its rejections.
* Two GPUs (skipped on a box with fewer): two ranks as child processes, each
  computing its N-shard and storing into both ranks' gathered buffers over
  NVLink (epoch flags) or both ranks' line buffers (tagged lines); after the
  completion both gathered outputs must match the oracle for the whole N over
  four consecutive launches (alternating buffer sets), with status 0.
* Two GPUs: the serving loop's schedule (decode_opt_b200.tp.serving_schedule)
  run for 24 requests in groups of 4 -- H2D copies, fused GEMMs and D2H
  copies on three streams, input slots and gathered sets reused -- with five
  different activations cycling, so that a reuse hazard would corrupt a
  request; every request's gathered output must match the oracle.
"""

import ctypes
import os
import socket

import numpy as np
import pytest
import torch

import decode_opt_b200 as dg
from decode_opt_b200 import _lib, tp

pytestmark = pytest.mark.gpu


def test_strided_output_at_column_offset():
    import oracle
    from helpers import check_against_oracle
    n, k, m = 1024, 2048, 5
    w, ws = oracle.gen_weight_smoke(n, k, 77)
    a, as_ = oracle.gen_activation_smoke(m, k, 78)
    ref = oracle.compute_reference(a, as_, w, ws, threads=8)
    dev = "cuda"
    cfg = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED)
    plan = cfg.plan(m, n, k)
    wt = dg.prepack_weight(torch.from_numpy(w).to(dev), cfg.block_n, cfg.layout)
    ldo, col = n + 64, 32
    wide = torch.full((m, ldo), -7.0, dtype=torch.bfloat16, device=dev)
    ws_buf = torch.zeros(max(plan.ws_floats, 1), device=dev)
    sem = torch.zeros(max(plan.sem_ints, 1), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    act = torch.from_numpy(a).to(dev)
    p = dg.Problem(m, n, k, act, wt, torch.from_numpy(ws).to(dev), torch.from_numpy(as_).to(dev), None, ws_buf,
                   sem, status)
    g = _lib.DgGather()
    g.world, g.rank, g.ldo = 1, 0, ldo
    g.outputs[0] = wide.data_ptr() + 2 * col
    g.sync = 0
    rc = dg.launch_gather(cfg, p, g, dg.make_weight_tma(cfg, p), dg.make_activation_tma(cfg, p))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = wide.float().cpu().numpy()
    ok, rl2, worst = check_against_oracle(got[:, col:col + n], ref)
    assert ok, (rl2, worst)
    assert np.all(got[:, :col] == -7.0) and np.all(got[:, col + n:] == -7.0)


def test_lines_world_one_and_rejections():
    """dg_launch_gather_lines with a world of one is a plain launch into the
    gathered buffer (row stride ldo); configurations the lines protocol cannot
    serve are refused before any launch: a stream-K plan, N not a multiple of
    4, misaligned line or output pointers, ldo < world * N."""
    import oracle
    from helpers import check_against_oracle
    n, k, m = 1024, 2048, 3
    w, ws = oracle.gen_weight_smoke(n, k, 81)
    a, as_ = oracle.gen_activation_smoke(m, k, 82)
    ref = oracle.compute_reference(a, as_, w, ws, threads=8)
    dev = "cuda"
    cfg = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED)
    assert cfg.plan(m, n, k).cluster >= 2
    wt = dg.prepack_weight(torch.from_numpy(w).to(dev), cfg.block_n, cfg.layout)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    p = dg.Problem(m, n, k, torch.from_numpy(a).to(dev), wt, torch.from_numpy(ws).to(dev),
                   torch.from_numpy(as_).to(dev), None, None, None, status)
    wm, am = dg.make_weight_tma(cfg, p), dg.make_activation_tma(cfg, p)
    ldo = n + 64
    wide = torch.full((m, ldo), -7.0, dtype=torch.bfloat16, device=dev)
    sync = torch.zeros(2, dtype=torch.int32, device=dev)
    g1 = tp.lines_descriptor(1, 0, n, wide.data_ptr(), [0], sync.data_ptr())
    g1.ldo = ldo
    assert dg.launch_gather(cfg, p, g1, wm, am) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    got = wide.float().cpu().numpy()
    ok, rl2, worst = check_against_oracle(got[:, :n], ref)
    assert ok, (rl2, worst)
    assert np.all(got[:, n:] == -7.0)

    # world 2 descriptors over local buffers: every one is refused.
    lines = torch.zeros((2, m, 2 * n // 4, 2), dtype=torch.int64, device=dev)
    out2 = torch.zeros((m, 2 * n), dtype=torch.bfloat16, device=dev)

    def desc(**kw):
        g = tp.lines_descriptor(2, 0, n, out2.data_ptr(), [lines[0].data_ptr(), lines[1].data_ptr()],
                                sync.data_ptr())
        for key, v in kw.items():
            if key == "line1":
                g.lines[1] = v
            else:
                setattr(g, key, v)
        return g
    sk = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, schedule="stream_k")
    skp = dg.Problem(m, n, k, p.activation, dg.prepack_weight(torch.from_numpy(w).to(dev), sk.block_n, sk.layout),
                     p.weight_scales, p.activation_scales, None,
                     torch.zeros(max(sk.plan(m, n, k).ws_floats, 1), device=dev),
                     torch.zeros(max(sk.plan(m, n, k).sem_ints, 1), dtype=torch.int32, device=dev), status)
    assert dg.launch_gather(sk, skp, desc(), dg.make_weight_tma(sk, skp), dg.make_activation_tma(sk, skp)) == \
        dg.CUDA_ERROR_INVALID_VALUE
    assert dg.launch_gather(cfg, p, desc(line1=lines[1].data_ptr() + 8), wm, am) == dg.CUDA_ERROR_INVALID_VALUE
    assert dg.launch_gather(cfg, p, desc(output=out2.data_ptr() + 2), wm, am) == dg.CUDA_ERROR_INVALID_VALUE
    assert dg.launch_gather(cfg, p, desc(ldo=2 * n - 4), wm, am) == dg.CUDA_ERROR_INVALID_VALUE
    assert dg.launch_gather(cfg, p, desc(sync=0), wm, am) == dg.CUDA_ERROR_INVALID_VALUE
    qb = torch.zeros((m, 2 * n), dtype=torch.uint8, device=dev)
    qsb = torch.zeros((m, 2 * n // 128), device=dev)
    g1q = tp.lines_descriptor(1, 0, n, wide.data_ptr(), [0], sync.data_ptr(), qb.data_ptr(), qsb.data_ptr())
    g1q.ldo = ldo
    assert dg.launch_gather(cfg, p, g1q, wm, am) == dg.CUDA_ERROR_INVALID_VALUE        # no quantised world of one
    assert dg.launch_gather(cfg, p, desc(q_out=qb.data_ptr()), wm, am) == dg.CUDA_ERROR_INVALID_VALUE
    assert dg.launch_gather(cfg, p, desc(q_out=qb.data_ptr() + 1, q_scales=qsb.data_ptr()), wm, am) == \
        dg.CUDA_ERROR_INVALID_VALUE
    n6 = n - 2
    p6 = dg.Problem(m, n6, k, p.activation, wt, p.weight_scales, p.activation_scales, None, None, None, status)
    g6 = tp.lines_descriptor(2, 0, n6, out2.data_ptr(), [lines[0].data_ptr(), lines[1].data_ptr()], sync.data_ptr())
    assert dg.launch_gather(cfg, p6, g6, dg.make_weight_tma(cfg, p6), dg.make_activation_tma(cfg, p6)) == \
        dg.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    p8 = dg.Problem(m, n - 4, k, p.activation, wt, p.weight_scales, p.activation_scales, None, None, None, status)
    g8 = tp.lines_descriptor(2, 0, n - 4, out2.data_ptr(), [lines[0].data_ptr(), lines[1].data_ptr()],
                             sync.data_ptr(), qb.data_ptr(), qsb.data_ptr())        # 2 * 1020 % 128 != 0
    assert dg.launch_gather(cfg, p8, g8, dg.make_weight_tma(cfg, p8), dg.make_activation_tma(cfg, p8)) == \
        dg.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
    assert not bool(out2.view(torch.int16).any()) and not bool(lines.any()) and not bool(sync.any())
    assert not bool(qb.any()) and not bool(qsb.any())


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, m, n, k, result_dir, protocol="flags", steps=2, quant=False):
    import torch.distributed as dist
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fg = None
    try:
        dev = torch.device("cuda", rank)
        w, ws = oracle.gen_weight_smoke(n, k, 91)
        n_loc = n // world
        lo, hi = tp.shard_rows(n, world, rank)
        cfg = dg.default_config(m, n_loc, k, layout=dg.LAYOUT_PACKED_SWIZZLED, gather_lines=protocol == "lines")
        plan = cfg.plan(m, n_loc, k)
        wt = dg.prepack_weight(torch.from_numpy(np.ascontiguousarray(w[lo:hi])).to(dev), cfg.block_n, cfg.layout)
        wsc = torch.from_numpy(np.ascontiguousarray(tp.shard_scales(ws, world, rank, n))).to(dev)
        ws_buf = torch.zeros(max(plan.ws_floats, 1), device=dev)
        sem = torch.zeros(max(plan.sem_ints, 1), dtype=torch.int32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        fg = tp.FusedGather(m, n_loc, device=dev, protocol=protocol)
        results, qs_bytes, qs_scales = [], [], []
        for step in range(steps):
            a, as_ = oracle.gen_activation_smoke(m, k, 200 + step)
            act = torch.from_numpy(a).to(dev)
            p = dg.Problem(m, n_loc, k, act, wt, wsc, torch.from_numpy(as_).to(dev), None, ws_buf, sem, status)
            q = torch.full((m, n), 0x55, dtype=torch.uint8, device=dev)
            qs = torch.full((m, n // 128), -1.0, device=dev)
            desc = fg.descriptor(step % 2, q, qs) if quant else fg.descriptor(step % 2)
            dist.barrier()
            rc = dg.launch_gather(cfg, p, desc, dg.make_weight_tma(cfg, p), dg.make_activation_tma(cfg, p))
            assert rc == 0, rc
            fg.wait(step % 2, status=status)
            torch.cuda.synchronize(dev)
            assert int(status.item()) == 0, dg.status_string(int(status.item()))
            results.append(fg.output(step % 2, m).float().cpu().numpy())
            qs_bytes.append(q.cpu().numpy())
            qs_scales.append(qs.cpu().numpy())
        np.save(os.path.join(result_dir, f"rank{rank}.npy"), np.stack(results))
        np.save(os.path.join(result_dir, f"q{rank}.npy"), np.stack(qs_bytes))
        np.save(os.path.join(result_dir, f"qs{rank}.npy"), np.stack(qs_scales))
        dist.barrier()
    finally:
        if fg is not None:
            fg.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("protocol", ["flags", "lines", "lines_quant"])
@pytest.mark.parametrize("m", [1, 8])
def test_two_gpu_fused_gather_matches_oracle(tmp_path, m, protocol):
    """Four consecutive launches (buffer sets 0, 1, 0, 1; under the lines
    protocol epochs 1..4, so a set's stale lines from two launches back must
    not be taken for the current ones).  lines_quant: the unpack also writes
    the gathered output's e4m3 block quantisation, which must equal the
    oracle's quantisation of that output bit for bit."""
    import torch.multiprocessing as mp
    import oracle
    from helpers import check_against_oracle
    n, k, world, steps = 2048, 4096, 2, 4
    quant = protocol == "lines_quant"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, m, n, k, str(tmp_path),
                                                  "lines" if quant else protocol, steps, quant))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.exitcode is None:
            p.kill()
        assert p.exitcode == 0
    w, ws = oracle.gen_weight_smoke(n, k, 91)
    for step in range(steps):
        a, as_ = oracle.gen_activation_smoke(m, k, 200 + step)
        ref = oracle.compute_reference(a, as_, w, ws, threads=8)
        for r in range(world):
            got = np.load(os.path.join(str(tmp_path), f"rank{r}.npy"))[step]
            ok, rl2, worst = check_against_oracle(got, ref)
            assert ok, (r, step, rl2, worst)
            if quant:
                want_q, want_s = oracle.quantize_rows(got)
                assert np.array_equal(np.load(os.path.join(str(tmp_path), f"q{r}.npy"))[step], want_q), (r, step)
                assert np.array_equal(np.load(os.path.join(str(tmp_path), f"qs{r}.npy"))[step], want_s), (r, step)


def _serve_main(rank, world, port, m, n, k, group, count, distinct, result_dir, protocol="flags"):
    """One rank of the N-GPU serving loop (decode_opt_b200.tp.serving_schedule,
    executed as bench.py executes it, eagerly): request j copies activation
    j % distinct in from pinned host memory, runs the fused GEMM into
    gathered set j % (2*group) and copies its output to its own pinned host
    buffer."""
    import torch.distributed as dist
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    fg = None
    try:
        dev = torch.device("cuda", rank)
        w, ws = oracle.gen_weight_smoke(n, k, 91)
        n_loc = n // world
        lo, hi = tp.shard_rows(n, world, rank)
        cfg = dg.default_config(m, n_loc, k, layout=dg.LAYOUT_PACKED_SWIZZLED, independent_inputs=True,
                                gather_lines=protocol == "lines")
        plan = cfg.plan(m, n_loc, k)
        wt = dg.prepack_weight(torch.from_numpy(np.ascontiguousarray(w[lo:hi])).to(dev), cfg.block_n, cfg.layout)
        wsc = torch.from_numpy(np.ascontiguousarray(tp.shard_scales(ws, world, rank, n))).to(dev)
        ws_buf = torch.zeros(max(plan.ws_floats, 1), device=dev)
        sem = torch.zeros(max(plan.sem_ints, 1), dtype=torch.int32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        nset = 2 * group
        fg = tp.FusedGather(m, n_loc, buffers=nset, device=dev, protocol=protocol)
        kb = k // 128
        in_bytes = m * k + m * kb * 4
        hins = []
        for r in range(distinct):
            a, as_ = oracle.gen_activation_smoke(m, k, 300 + r)
            h = torch.empty(in_bytes, dtype=torch.uint8).pin_memory()
            h[: m * k].copy_(torch.from_numpy(a.reshape(-1)))
            h[m * k:].copy_(torch.from_numpy(as_.reshape(-1)).view(torch.uint8))
            hins.append(h)
        slots, probs = [], []
        for _ in range(nset):
            d_in = torch.empty(in_bytes, dtype=torch.uint8, device=dev)
            p = dg.Problem(m, n_loc, k, d_in[: m * k].view(m, k), wt, wsc,
                           d_in[m * k:].view(torch.float32).view(m, kb), None, ws_buf, sem, status)
            slots.append(d_in)
            probs.append((p, dg.make_activation_tma(cfg, p)))
        w_map = dg.make_weight_tma(cfg, probs[0][0])
        descs = [fg.descriptor(i) for i in range(nset)]
        h_outs = [torch.empty((m, world * n_loc), dtype=torch.bfloat16).pin_memory() for _ in range(count)]
        compute = torch.cuda.Stream(device=dev)
        streams = {"h2d": torch.cuda.Stream(device=dev), "gemm": compute, "d2h": torch.cuda.Stream(device=dev)}
        ring = 2 * nset + 2
        done = {kind: [torch.cuda.Event() for _ in range(ring)] for kind in streams}
        dist.barrier()
        for kind, j, waits in tp.serving_schedule(0, count, group):
            st = streams[kind]
            for wk, wj in waits:
                st.wait_event(done[wk][wj % ring])
            with torch.cuda.stream(st):
                if kind == "h2d":
                    slots[j % nset].copy_(hins[j % distinct], non_blocking=True)
                elif kind == "gemm":
                    p, a_map = probs[j % nset]
                    rc = dg.launch_gather(cfg, p, descs[j % nset], w_map, a_map, st, pdl_attr=cfg.pdl)
                    assert rc == 0, rc
                else:
                    h_outs[j].copy_(fg.output(j % nset, m), non_blocking=True)
            done[kind][j % ring].record(st)
        torch.cuda.synchronize(dev)
        assert int(status.item()) == 0, dg.status_string(int(status.item()))
        np.save(os.path.join(result_dir, f"serve{rank}.npy"), np.stack([h.float().numpy() for h in h_outs]))
        dist.barrier()
    finally:
        if fg is not None:
            fg.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("protocol", ["flags", "lines"])
@pytest.mark.parametrize("m", [1, 8])
def test_two_gpu_serving_schedule_matches_oracle(tmp_path, m, protocol):
    import torch.multiprocessing as mp
    import oracle
    from helpers import check_against_oracle
    n, k, world, group, count, distinct = 2048, 4096, 2, 4, 24, 5
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_serve_main, args=(r, world, port, m, n, k, group, count, distinct, str(tmp_path),
                                                   protocol))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.exitcode is None:
            p.kill()
        assert p.exitcode == 0
    w, ws = oracle.gen_weight_smoke(n, k, 91)
    refs = []
    for r in range(distinct):
        a, as_ = oracle.gen_activation_smoke(m, k, 300 + r)
        refs.append(oracle.compute_reference(a, as_, w, ws, threads=8))
    for r in range(world):
        got = np.load(os.path.join(str(tmp_path), f"serve{r}.npy"))
        for j in range(count):
            ok, rl2, worst = check_against_oracle(got[j], refs[j % distinct])
            assert ok, (r, j, rl2, worst)
