"""Cluster split-K (grid_ctas = DG_GRID_CLUSTER): the S CTAs of a tile form a
thread-block cluster and reduce through distributed shared memory.  Parity
with the oracle across batch classes, layouts, ragged N and split factors
(portable and non-portable cluster sizes), run-to-run bit determinism, no
workspace, back-to-back launches under programmatic dependent launch, tile
widths that are any multiple of 8, splits finer than a tile's chunks, and the
planner's rejections."""

import numpy as np
import pytest

import oracle
from helpers import DeviceCase, check_against_oracle, smoke_case

dg = pytest.importorskip("decode_opt_b200")
pytestmark = pytest.mark.gpu


def _cfg(m, block_n=256, subs=2, split=1, layout=None, pdl=False, stages=2):
    return dg.B200Config(m_tile=dg.m_tile_for(m), block_n=block_n, subs=subs, stages=stages,
                         layout=dg.LAYOUT_PACKED_SWIZZLED if layout is None else layout, pdl=pdl,
                         split_k=split, grid_ctas=dg.GRID_CLUSTER)


def _check(dc, cfg, ref, runs=2):
    first = None
    for _ in range(runs):
        rc, got, status = dc.run(cfg)
        assert rc == 0 and status == 0, (rc, hex(status))
        if first is None:
            first = got
            ok, rl2, worst = check_against_oracle(got, ref)
            assert ok, (rl2, worst)
        else:
            assert np.array_equal(got.view(np.uint32), first.view(np.uint32)), "not bit-identical"
    assert dc.splitk_ws is None and dc.sem is None     # no workspace in cluster mode
    return first


@pytest.mark.parametrize("m", [1, 3, 8, 16, 17, 32, 40, 64, 65, 100, 128])
def test_batch_classes_auto_split(m):
    n, k = 2048, 4096
    w, ws, a, as_, ref = smoke_case(n, k, 7, m)
    dc = DeviceCase(w, ws, a, as_, n)
    cfg = _cfg(m)
    plan = cfg.plan(m, n, k)
    assert plan.error is None and plan.cluster == 8 and plan.grid == (8, 8, 1)
    assert plan.ws_floats == 0 and plan.sem_ints == 0
    _check(dc, cfg, ref)


@pytest.mark.parametrize("split", [2, 3, 5, 7, 8, 11, 16])
def test_split_factors(split):
    n, k, m = 1536, 5632, 9          # 44 k-blocks: uneven ranges for most S
    w, ws, a, as_, ref = smoke_case(n, k, 11, m)
    dc = DeviceCase(w, ws, a, as_, n)
    cfg = _cfg(m, block_n=128, subs=1, split=split)
    assert cfg.plan(m, n, k).cluster == split
    _check(dc, cfg, ref)


@pytest.mark.parametrize("layout", [0, 1, 2])
@pytest.mark.parametrize("block_n", [64, 96, 128, 256])
def test_layouts_ragged_n(layout, block_n):
    n, k, m = 1000, 2048, 5          # last tile partial; N not a multiple of 8
    w, ws, a, as_, ref = smoke_case(n, k, 13, m)
    dc = DeviceCase(w, ws, a, as_, n)
    cfg = _cfg(m, block_n=block_n, subs=1, split=4, layout=layout, stages=3)
    _check(dc, cfg, ref)


def test_c2_shape_m1_and_m128():
    n, k = 7168, 16384
    for m in (1, 128):
        w, ws = oracle.gen_weight_smoke(n, k, 21)
        a, as_ = oracle.gen_activation_smoke(m, k, 22 + m)
        ref = oracle.compute_reference(a, as_, w, ws, threads=8)
        dc = DeviceCase(w, ws, a, as_, n)
        cfg = _cfg(m)
        plan = cfg.plan(m, n, k)
        assert plan.cluster == 4 and plan.num_ctas == 112     # 28 clusters of 4: one wave
        _check(dc, cfg, ref, runs=2)


def test_back_to_back_pdl_graph():
    """A CUDA graph of back-to-back cluster launches with programmatic
    dependent launch (the benchmark's loop): last output equals one launch."""
    import torch
    n, k, m = 2048, 4096, 4
    w, ws, a, as_, ref = smoke_case(n, k, 17, m)
    dc = DeviceCase(w, ws, a, as_, n)
    cfg = _cfg(m, pdl=True)
    _, single, _ = dc.run(cfg)
    wt = dc.weight_for(cfg)
    p = dg.Problem(m, n, k, dc.a, wt, dc.ws, dc.as_, dc.out, None, None, dc.status)
    wm, am = dg.make_weight_tma(cfg, p), dg.make_activation_tma(cfg, p)
    s = torch.cuda.Stream()
    dc.out.zero_()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(20):
            assert dg.launch_with_maps(cfg, p, wm, am, s, pdl_attr=True) == 0
    with torch.cuda.stream(s):
        g.replay()
        g.replay()
    torch.cuda.synchronize()
    assert int(dc.status.item()) == 0
    got = dc.out.float().cpu().numpy()
    assert np.array_equal(got.view(np.uint32), single.view(np.uint32))


@pytest.mark.parametrize("m,n,k,bn,subs,split", [
    (8, 1000, 2048, 56, 2, 2),     # a tile width that is no multiple of 32 (partial rows padded to 64 floats)
    (5, 1000, 2048, 240, 2, 9),    # 9 CTAs per cluster, 8 chunks per tile: one CTA adds a zero partial
    (64, 700, 1024, 120, 1, 16),   # 16 CTAs (non-portable cluster), 8 chunks: half of them idle
])
def test_any_width_and_splits_finer_than_the_chunks(m, n, k, bn, subs, split):
    w, ws, a, as_, ref = smoke_case(n, k, 61, m)
    dc = DeviceCase(w, ws, a, as_, n)
    _check(dc, _cfg(m, block_n=bn, subs=subs, split=split, stages=0), ref)


def test_planner_rejections():
    assert "split_k must be <= 16" in _cfg(8, split=17).plan(8, 2048, 16384).error
    # M=128 x 256 fp32 = 128 KiB of partial does not fit a 1-stage ring
    assert "partial" in _cfg(128, subs=1, split=2, stages=1).plan(128, 2048, 4096).error
    # S = 1 is the plain tile schedule (no cluster)
    plan = _cfg(8, split=1).plan(8, 65536, 1024)
    assert plan.error is None and plan.cluster == 1
