"""GPU parity of the swap-AB batch class (FLAG_SWAP_AB, M <= 16): the weights
on the tcgen05.mma M side (two 128-row MMAs per tile, issued by two warps),
the batch padded to 16 on the N side.

* Against the oracle (the reference's host GEMM, kernels/smoke_test.cu
  :60-207 restated) on the reference's smoke generators: every M up to 16,
  the three weight layouts, both PDL modes, tile widths 136 / 224 / 256
  (below 256 rows the second 128-row half also reads the rows after the
  tile, whose results are dropped), the cluster split the library picks,
  splits finer than a tile's chunks, and one CTA per tile (no split: the
  direct-store path).  The reference's gate: rel_l2 <= 2e-3 and the
  per-element bound.
* Run-to-run bit-identical (the cluster reduction sums in rank order).
* Against the default M <= 16 class on the same inputs: the same outputs up
  to the accumulation order inside the tensor core (the per-element fold and
  the reduction order are the same).
* The fused quantiser (dg_launch_quantized) on the swap class: bf16 output
  bit-identical to the plain launch and e4m3 bytes/scales bit-identical to
  the standalone quantiser.
* The test hook that makes one bounded wait run out: status 0x51, and the
  next clean launch is correct (both MMA issuers drain and free TMEM).
* Rejections: M > 16, block_n <= 128, a stream-K schedule.
"""

from dataclasses import replace

import numpy as np
import pytest
import torch

import decode_opt_b200 as dg
import oracle
from helpers import DeviceCase, check_against_oracle, smoke_case

pytestmark = pytest.mark.gpu

SEED = 0x5A5A1234


def swap_cfg(m, n, k, layout, independent=False, block_n=None, split_k=None):
    cfg = dg.default_config(m, n, k, layout=layout, pdl=True, independent_inputs=independent, swap_ab=True)
    if block_n is not None:
        cfg = replace(cfg, block_n=block_n)
    if split_k is not None:
        cfg = replace(cfg, split_k=split_k)
    return cfg


CASES = [
    # m, n, k, layout, independent, block_n, split_k
    (1, 7168, 16384, dg.LAYOUT_PACKED_SWIZZLED, False, None, None),
    (1, 7168, 16384, dg.LAYOUT_PACKED_SWIZZLED, True, None, None),
    (1, 2048, 4096, dg.LAYOUT_RAW, False, None, None),
    (2, 2048, 4096, dg.LAYOUT_PACKED, True, None, None),
    (3, 6144, 8192, dg.LAYOUT_PACKED_SWIZZLED, False, 256, None),
    (5, 1000, 4096, dg.LAYOUT_RAW, False, 224, None),
    (7, 2048, 4096, dg.LAYOUT_PACKED_SWIZZLED, True, 136, None),
    (8, 7168, 16384, dg.LAYOUT_RAW, False, None, None),
    (11, 4096, 7168, dg.LAYOUT_PACKED, False, 224, 5),
    (13, 584, 1024, dg.LAYOUT_PACKED_SWIZZLED, False, 256, 8),     # split 8 > 4 chunks: zero partials
    (16, 2048, 4096, dg.LAYOUT_PACKED_SWIZZLED, False, None, None),
    (16, 7168, 16384, dg.LAYOUT_PACKED_SWIZZLED, True, None, None),
    (1, 1792, 16384, dg.LAYOUT_PACKED_SWIZZLED, False, None, None),  # 4-GPU shard: clusters of 16 (non-portable)
    (8, 896, 16384, dg.LAYOUT_PACKED_SWIZZLED, False, 256, None),    # 8-GPU shard: 4 tiles x 16
    (4, 20480, 1024, dg.LAYOUT_RAW, True, 256, None),              # 80 tiles: no split fits, one CTA per tile
    (9, 20480, 1024, dg.LAYOUT_PACKED_SWIZZLED, False, 256, None),
]


@pytest.mark.parametrize("m,n,k,layout,independent,block_n,split_k", CASES)
def test_swap_ab_matches_oracle(m, n, k, layout, independent, block_n, split_k):
    w, ws, a, as_, ref = smoke_case(n, k, SEED, m)
    dc = DeviceCase(w, ws, a, as_, n)
    cfg = swap_cfg(m, n, k, layout, independent, block_n, split_k)
    plan = cfg.plan(m, n, k)
    assert plan.error is None, plan.error
    assert plan.mma_m == 128 and plan.n_mma == 16 and plan.ws_floats == 0
    if n == 20480:
        assert plan.cluster == 1          # the direct-store path
    if n in (896, 1792) and not independent:
        assert plan.cluster == 16         # a non-portable cluster size
    rc, got, status = dc.run(cfg)
    assert rc == 0 and status == 0, (rc, dg.status_string(status))
    ok, rl2, worst = check_against_oracle(got, ref)
    assert ok, (rl2, worst)
    # run-to-run bit-identical
    rc, again, status = dc.run(cfg)
    assert rc == 0 and status == 0
    assert np.array_equal(got.view(np.uint32), again.view(np.uint32))


@pytest.mark.parametrize("m,n,k,independent", [(1, 7168, 16384, False), (4, 2048, 4096, True),
                                               (16, 6144, 8192, False)])
def test_swap_ab_matches_default_class(m, n, k, independent):
    w, ws, a, as_, ref = smoke_case(n, k, SEED, m)
    dc = DeviceCase(w, ws, a, as_, n)
    layout = dg.LAYOUT_PACKED_SWIZZLED
    base = dg.default_config(m, n, k, layout=layout, pdl=True, independent_inputs=independent, swap_ab=False)
    sw = swap_cfg(m, n, k, layout, independent, block_n=base.block_n)
    assert sw.plan(m, n, k).cluster == base.plan(m, n, k).cluster
    rc, want, status = dc.run(base)
    assert rc == 0 and status == 0
    rc, got, status = dc.run(sw)
    assert rc == 0 and status == 0
    # Same fold and reduction order; only the tensor core's accumulation
    # order inside a 128-K block may differ between the two placements.
    assert oracle.rel_l2(got, want) <= 1e-5
    ok, rl2, worst = check_against_oracle(got, ref)
    assert ok, (rl2, worst)


@pytest.mark.parametrize("m,n,k", [(1, 7168, 16384), (16, 2048, 7168), (3, 640, 512)])
def test_swap_ab_quantized_output(m, n, k):
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(77 + m)
    w, ws, _, _, _ = smoke_case(n, k, SEED, 1)
    a, a_sc = dg.quantize_activation(torch.randn((m, k), device=dev, generator=g).bfloat16())
    cfg = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, pdl=True, quantized_output=True,
                            swap_ab=True)
    plan = cfg.plan(m, n, k)
    assert plan.error is None and plan.cluster >= 2 and plan.n_mma == 16
    w_dev = dg.prepack_weight(torch.from_numpy(w).to(dev), cfg.packed_rows, cfg.layout)
    w_sc = torch.from_numpy(ws).to(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    out_ref = torch.full((m, n), 7.0, dtype=torch.bfloat16, device=dev)
    out = torch.full((m, n), -3.0, dtype=torch.bfloat16, device=dev)
    q = torch.full((m, n), 0x55, dtype=torch.uint8, device=dev)
    qs = torch.full((m, n // 128), 9.0, dtype=torch.float32, device=dev)
    p_ref = dg.Problem(m, n, k, a, w_dev, w_sc, a_sc, out_ref, None, None, status)
    wm = dg.make_weight_tma(cfg, p_ref)
    assert dg.launch_with_maps(cfg, p_ref, wm, dg.make_activation_tma(cfg, p_ref)) == 0
    p = dg.Problem(m, n, k, a, w_dev, w_sc, a_sc, out, None, None, status)
    assert dg.launch_quantized(cfg, p, wm, dg.make_activation_tma(cfg, p), q, qs) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0, dg.status_string(int(status.item()))
    assert torch.equal(out.view(torch.int16), out_ref.view(torch.int16))
    want_q, want_s = dg.quantize_activation(out)
    torch.cuda.synchronize()
    assert torch.equal(q, want_q) and torch.equal(qs, want_s)
    want = oracle.compute_reference(a.cpu().numpy(), a_sc.cpu().numpy(), w, ws, threads=8)
    ok, rl2, worst = check_against_oracle(out.float().cpu().numpy(), want)
    assert ok, (rl2, worst)


def test_swap_ab_timeout_then_clean_launch():
    m, n, k = 8, 2048, 4096
    w, ws, a, as_, ref = smoke_case(n, k, SEED, m)
    dc = DeviceCase(w, ws, a, as_, n)
    cfg = swap_cfg(m, n, k, dg.LAYOUT_PACKED_SWIZZLED)
    bad = replace(cfg, flags=cfg.flags | dg.FLAG_INJECT_TIMEOUT, timeout_ns=20_000_000)
    rc, _, status = dc.run(bad)
    assert rc == 0 and status == dg.ERR_INJECTED_TIMEOUT, dg.status_string(status)
    rc, got, status = dc.run(cfg)
    assert rc == 0 and status == 0, dg.status_string(status)
    ok, rl2, worst = check_against_oracle(got, ref)
    assert ok, (rl2, worst)


def test_swap_ab_rejections():
    base = dg.default_config(8, 2048, 4096, layout=dg.LAYOUT_RAW, swap_ab=True)
    assert base.plan(8, 2048, 4096).error is None
    assert "M must be <= 16" in replace(base, m_tile=32).plan(17, 2048, 4096).error
    assert "block_n" in replace(base, block_n=128).plan(8, 2048, 4096).error
    assert "cluster" in replace(base, grid_ctas=-1).plan(8, 2048, 4096).error
    with pytest.raises(ValueError):
        dg.default_config(17, 2048, 4096, swap_ab=True)
    with pytest.raises(ValueError):
        dg.default_config(8, 2048, 4096, schedule="stream_k", swap_ab=True)
