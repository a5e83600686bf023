"""Multi-rank host logic of the N-sharded tensor-parallel path, on CPU.

Two `gloo` ranks (world_size 2) shard W by rows exactly as the GPU path does,
compute each slice with the oracle (standing in for the kernel on a machine
without a GPU), all-gather through torch.distributed and must reproduce the
single-rank oracle result bit-for-bit."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from decode_opt_b200 import tp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, m, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import oracle
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, k = 512, 384
        w, ws = oracle.gen_weight_smoke(n, k, 41)
        a, as_ = oracle.gen_activation_smoke(m, k, 42)
        lo, hi = tp.shard_rows(n, world, rank)
        local = oracle.compute_reference(a, as_, np.ascontiguousarray(w[lo:hi]),
                                         np.ascontiguousarray(tp.shard_scales(ws, world, rank, n)))
        full = tp.gather_slices(torch.from_numpy(local))
        if rank == 0:
            np.save(result_path, full.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("m", [1, 3])
def test_two_rank_shard_and_gather_matches_single_rank(tmp_path, m):
    import oracle
    world = 2
    path = str(tmp_path / "full.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, path)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    full = np.load(path)
    n, k = 512, 384
    w, ws = oracle.gen_weight_smoke(n, k, 41)
    a, as_ = oracle.gen_activation_smoke(m, k, 42)
    want = oracle.compute_reference(a, as_, w, ws)
    assert np.array_equal(full.view(np.uint32), want.view(np.uint32))


def test_shard_rows_alignment():
    assert tp.shard_rows(7168, 8, 3) == (2688, 3584)
    assert tp.shard_rows(7168, 1, 0) == (0, 7168)
    with pytest.raises(ValueError):
        tp.shard_rows(7168, 3, 0)          # 7168/3 is not an integer
    with pytest.raises(ValueError):
        tp.shard_rows(2048, 32, 0)         # 64-row shards break 128-row scale groups


def test_assemble_layout():
    g, m, n_loc = 4, 3, 5
    gathered = torch.arange(g * m * n_loc).reshape(g, m, n_loc)
    full = tp.assemble(gathered, m)
    for r in range(g):
        assert torch.equal(full[:, r * n_loc:(r + 1) * n_loc], gathered[r])
    assert tp.assemble(gathered[:, :1], 1).shape == (1, g * n_loc)


def test_gather_descriptor_pointer_table():
    """Rank r of g writes columns [r*n_loc, (r+1)*n_loc) of every rank's
    gathered buffer; the row stride is g*n_loc; flags and sync pass through."""
    world, n_loc = 4, 896
    bases = [0x10000000 * (q + 1) for q in range(world)]
    flags = [0x7000 + 64 * q for q in range(world)]
    for rank in range(world):
        g = tp.gather_descriptor(world, rank, n_loc, bases, flags, 0x9000)
        assert (g.world, g.rank, g.ldo) == (world, rank, world * n_loc)
        for q in range(world):
            assert g.outputs[q] == bases[q] + 2 * rank * n_loc
            assert g.flags[q] == flags[q]
        assert g.sync == 0x9000
    with pytest.raises(ValueError):
        tp.gather_descriptor(9, 0, n_loc, bases * 3, flags * 3, 0)


def test_lines_descriptor_pointer_table():
    """The lines protocol's descriptor: this rank's own gathered buffer at
    column 0, every rank's line buffer base as mapped here (the kernel adds
    the rank's column offset in lines), row stride g*n_loc, sync passed
    through; a world above 8 or a rank outside it is refused."""
    world, n_loc = 8, 896
    lines = [0x20000000 * (q + 1) for q in range(world)]
    for rank in range(world):
        g = tp.lines_descriptor(world, rank, n_loc, 0x5000, lines, 0x9000)
        assert (g.world, g.rank, g.ldo, g.output, g.sync) == (world, rank, world * n_loc, 0x5000, 0x9000)
        assert [g.lines[q] for q in range(world)] == lines
    for bad in ((9, 0), (2, 2), (2, -1)):
        with pytest.raises(ValueError):
            tp.lines_descriptor(bad[0], bad[1], n_loc, 0x5000, lines + lines, 0x9000)
