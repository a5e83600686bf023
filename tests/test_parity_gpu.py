"""GPU parity tests: the sm_100a kernel against the oracle, through the C ABI.

The first group replays the reference's own correctness gate
(kernels/smoke_test.cu:542-618): the same 50 (shape, M, KernelConfig) cases,
the same seeds, the same rel_l2 <= 2e-3 gate, plus the per-element bound
|got - want| <= 1e-2 * max(|want|, 1e-2 * rms(want)), the split-K ticket
self-reset check and a second launch.  The 37-case subset of the north star
is A_contract (26) + B_big (7) + the first four C_smalln cases.
"""

import numpy as np
import pytest

import decode_opt_b200 as dg
import oracle
from helpers import DeviceCase, check_against_oracle, smoke_case

pytestmark = pytest.mark.gpu

KC = dg.KernelConfig


def cfg(mt, bm, wg, reg, stg, tiles, subs, pack, pdl, epi, splitk, preg=32, spw=False, pre=False, sis=None,
        skf=0):
    return KC(mt, bm, wg, reg, stg, tiles, subs, pack, pdl, epi, splitk, preg, spw, pre, sis, skf)


# kernels/smoke_test.cu:410-457, the reference's named configurations.
S0_m8 = cfg(8, 64, 4, 112, 2, 1, 1, False, False, False, False)
S1_m8 = cfg(8, 64, 4, 112, 2, 1, 1, False, True, False, False)
S2_m8 = cfg(8, 64, 4, 112, 2, 1, 2, False, True, False, False)
S3_m8 = cfg(8, 64, 4, 112, 2, 1, 2, True, True, False, False)
S4_m8 = cfg(8, 48, 2, 80, 3, 1, 2, True, True, False, False)
S5_m8 = cfg(8, 48, 2, 80, 3, 1, 2, True, True, True, False)
S6_m8 = cfg(8, 48, 2, 80, 3, 1, 2, True, True, True, True)
S4_m8_bm56 = cfg(8, 56, 2, 80, 3, 1, 2, True, True, False, False)
S5_m8_bm56 = cfg(8, 56, 2, 80, 3, 1, 2, True, True, True, False)
S6_m8_bm56 = cfg(8, 56, 2, 80, 3, 1, 2, True, True, True, True)
S5_m8_pad = cfg(8, 48, 2, 80, 3, 1, 2, True, True, True, False)
S0_m8_pad = cfg(8, 48, 4, 112, 2, 1, 1, False, False, False, False)
S6_m8_n2048 = cfg(8, 32, 2, 80, 3, 1, 2, True, True, True, True)
S2_m8_n2048_splitk = cfg(8, 64, 4, 112, 2, 1, 2, False, True, False, True)
S5_m8_n2048 = cfg(8, 32, 2, 80, 3, 1, 2, True, True, True, False)
S6F2_qwen = cfg(8, 32, 2, 80, 3, 1, 2, True, True, True, True, skf=2)
S6F4_qwen = cfg(8, 32, 2, 80, 3, 1, 2, True, True, True, True, skf=4)
S6F8_qwen = cfg(8, 32, 2, 80, 3, 1, 2, True, True, True, True, skf=8)
S6F2_kimi = cfg(8, 56, 2, 80, 3, 1, 2, True, True, True, True, skf=2)
S6F4_kimi = cfg(8, 56, 2, 80, 3, 1, 2, True, True, True, True, skf=4)
S6F8_kimi = cfg(8, 56, 2, 80, 3, 1, 2, True, True, True, True, skf=8)
S5_nosmem_scale = cfg(8, 48, 2, 80, 3, 1, 2, True, True, True, False, sis=False)
S5_preload = cfg(8, 48, 2, 80, 3, 1, 2, True, True, True, False, pre=True)
S5_spw = cfg(8, 48, 2, 80, 3, 1, 2, True, True, True, False, spw=True)
S5_tiles2 = cfg(8, 48, 4, 80, 2, 2, 2, True, True, True, False)
S5_wg1 = cfg(8, 64, 1, 112, 4, 1, 4, True, True, True, False)
S5_m16 = cfg(16, 64, 2, 112, 2, 2, 2, True, True, True, False)
S5_m32 = cfg(32, 64, 2, 168, 2, 2, 2, True, True, True, False, sis=False)
S5_m64 = cfg(64, 48, 2, 168, 2, 2, 2, True, True, True, False, sis=False)
S5_m128 = cfg(128, 48, 2, 168, 2, 2, 1, True, True, True, False, sis=False)
S2_m16_raw = cfg(16, 64, 2, 112, 2, 2, 2, False, True, False, False)
S6_m32 = cfg(32, 48, 2, 168, 2, 2, 2, True, True, True, True, sis=False)
S1_m128_raw = cfg(128, 64, 1, 232, 2, 1, 1, False, True, False, False, sis=False)

A, B, C, D = "A_contract", "B_big", "C_smalln", "D_kimi3"
SMOKE_CASES = [
    # A_contract 6144 x 7168 (kernels/smoke_test.cu:542-570)
    (A, 1, "S0 baseline", S0_m8), (A, 1, "S1 pdl", S1_m8), (A, 1, "S2 blockk", S2_m8),
    (A, 1, "S3 prepack", S3_m8), (A, 1, "S4 tile_stage", S4_m8), (A, 1, "S5 epi_overlap", S5_m8),
    (A, 1, "S6 splitk", S6_m8), (A, 1, "S5 scale_in_reg", S5_nosmem_scale),
    (A, 1, "S5 preload_act", S5_preload), (A, 1, "S5 single_prod_warp", S5_spw),
    (A, 1, "S5 tiles2", S5_tiles2), (A, 1, "S5 wg1_sub4", S5_wg1),
    (A, 8, "S0 baseline", S0_m8), (A, 8, "S1 pdl", S1_m8), (A, 8, "S2 blockk", S2_m8),
    (A, 8, "S3 prepack", S3_m8), (A, 8, "S4 tile_stage", S4_m8), (A, 8, "S5 epi_overlap", S5_m8),
    (A, 8, "S6 splitk", S6_m8), (A, 8, "S5 scale_in_reg", S5_nosmem_scale),
    (A, 16, "M16 S5", S5_m16), (A, 16, "M16 S2 raw", S2_m16_raw), (A, 32, "M32 S5", S5_m32),
    (A, 64, "M64 S5", S5_m64), (A, 128, "M128 S5", S5_m128), (A, 32, "M32 S6 splitk", S6_m32),
    # B_big 7168 x 16384 (:571-584)
    (B, 1, "S0 baseline bm48 pad", S0_m8_pad), (B, 1, "S4 tile_stage bm56", S4_m8_bm56),
    (B, 8, "S5 epi_overlap bm56", S5_m8_bm56), (B, 8, "S5 epi_overlap bm48 pad", S5_m8_pad),
    (B, 1, "S6 splitk bm56", S6_m8_bm56), (B, 32, "M32 S5 bm64", S5_m32),
    (B, 128, "M128 S1 raw wg1", S1_m128_raw),
    # C_smalln 2048 x 4096 (:585-598)
    (C, 1, "S5 epi_overlap bm32", S5_m8_n2048), (C, 1, "S6 splitk bm32", S6_m8_n2048),
    (C, 8, "S6 splitk bm32", S6_m8_n2048), (C, 1, "S2+splitk raw bm64", S2_m8_n2048_splitk),
    (C, 1, "S6 splitk S=2 bm32", S6F2_qwen), (C, 1, "S6 splitk S=4 bm32", S6F4_qwen),
    (C, 1, "S6 splitk S=8 bm32", S6F8_qwen), (C, 8, "S6 splitk S=2 bm32", S6F2_qwen),
    (C, 8, "S6 splitk S=4 bm32", S6F4_qwen), (C, 8, "S6 splitk S=8 bm32", S6F8_qwen),
    # D_kimi3 7168 x 12288 (:599-612)
    (D, 1, "S4 tile_stage bm56", S4_m8_bm56), (D, 1, "S6 splitk S=2 bm56", S6F2_kimi),
    (D, 1, "S6 splitk S=4 bm56", S6F4_kimi), (D, 1, "S6 splitk S=8 bm56", S6F8_kimi),
    (D, 8, "S6 splitk S=2 bm56", S6F2_kimi), (D, 8, "S6 splitk S=4 bm56", S6F4_kimi),
    (D, 8, "S6 splitk S=8 bm56", S6F8_kimi),
]
assert len(SMOKE_CASES) == 50
SUBSET_37 = set(range(26)) | set(range(26, 33)) | set(range(33, 37))

_DEV = {}


def device_case(shape: str, m: int) -> tuple:
    n, k, seed = oracle.SMOKE_SHAPES[shape]
    key = (shape, m)
    if key not in _DEV:
        _DEV.clear()
        w, ws, a, as_, ref = smoke_case(n, k, seed, m)
        _DEV[key] = (DeviceCase(w, ws, a, as_, n), ref)
    return _DEV[key]


def run_reference_config(dc: DeviceCase, kcfg: KC, clear_out=True):
    """Launch through the reference-shaped API (decode_gemm::launch<Cfg>)."""
    import torch
    plan = dg.make_launch_plan(kcfg, dg.Problem(dc.m, dc.n, dc.k))
    assert plan.error is None, plan.error
    slabs = max(kcfg.kSplitKFactor, plan.max_slabs)
    ws_need = slabs * dc.m * dc.n
    if dc.splitk_ws is None or dc.splitk_ws.numel() < ws_need:
        dc.splitk_ws = torch.zeros(ws_need, dtype=torch.float32, device="cuda")
    tiles_need = (dc.n + 15) // 16          # >= ceil(N/BM) for every legal BM (smoke_test.cu:515)
    if dc.sem is None or dc.sem.numel() < tiles_need:
        dc.sem = torch.zeros(tiles_need, dtype=torch.int32, device="cuda")
    if clear_out:
        dc.out.zero_()
    dc.status.zero_()
    weight = dc.w
    if kcfg.PREPACK:
        key = (kcfg.OUTPUT_ROWS_PER_CTA, dg.LAYOUT_PACKED)
        if key not in dc.packed:
            dst = torch.empty(dg.packed_weight_bytes(dc.n, dc.k, kcfg.OUTPUT_ROWS_PER_CTA), dtype=torch.uint8,
                              device="cuda")
            assert dg.launch_prepack_weight(kcfg.OUTPUT_ROWS_PER_CTA, kcfg.TILES_PER_CTA, dc.w, dst, dc.n,
                                            dc.k) == 0
            dc.packed[key] = dst
        weight = dc.packed[key]
    p = dg.Problem(dc.m, dc.n, dc.k, dc.a, weight, dc.ws, dc.as_, dc.out, dc.splitk_ws, dc.sem, dc.status)
    rc = dg.launch(kcfg, p)
    torch.cuda.synchronize()
    return rc, dc.out.float().cpu().numpy(), int(dc.status.item())


@pytest.mark.parametrize("idx", range(len(SMOKE_CASES)),
                         ids=[f"{c[0]}-M{c[1]}-{c[2].replace(' ', '_')}" for c in SMOKE_CASES])
def test_reference_smoke_case(idx):
    shape, m, label, kcfg = SMOKE_CASES[idx]
    dc, ref = device_case(shape, m)
    rc, got, status = run_reference_config(dc, kcfg)
    assert rc == 0 and status == 0, (rc, dg.status_string(status))
    ok, rl2, worst = check_against_oracle(got, ref)
    assert ok, f"{label}: rel_l2={rl2:.3e} worst={worst:.3e}"
    assert dc.sem_clean(), "split-K ticket array not self-reset"
    # Second launch on dirty buffers (kernels/smoke_test.cu:381-405).
    rc, got2, status = run_reference_config(dc, kcfg, clear_out=False)
    assert rc == 0 and status == 0
    ok2, rl2b, _ = check_against_oracle(got2, ref)
    assert ok2, f"second launch: rel_l2={rl2b:.3e}"
    assert np.array_equal(got, got2), "second launch not bit-identical"


@pytest.mark.parametrize("n,k,m,bm,subs,pack,skf", [
    (200, 256, 1, 48, 2, True, 0),      # one chunk per tile, split 4: three CTAs of each cluster idle
    (200, 384, 8, 48, 1, True, 0),      # 3 chunks over 4 CTAs; N below one 240-row CTA tile
    (1000, 512, 3, 40, 1, True, 0),     # BM 40: six packed tiles (240 rows) per CTA, ragged N
    (1000, 512, 17, 24, 2, True, 2),    # BM 24: ten packed tiles per CTA, M_TILE 32 (split max(2, 4))
    (1000, 2048, 64, 56, 2, True, 8),   # M_TILE 64 on BM 56 (224 rows), split 8: one chunk per CTA
    (777, 1024, 100, 64, 1, False, 0),  # raw weights, M_TILE 128 (ring deepened for the partial)
    (136, 2048, 128, 8, 4, True, 0),    # BM 8: 32 packed tiles per CTA, four K blocks per stage
])
def test_reference_config_wide_tiles(n, k, m, bm, subs, pack, skf):
    """A KernelConfig's CTA spans T = 256 // BM packed tiles (one TMA box
    over the tile dimension per stage) on a cluster split fixed by the
    configuration: splits finer than a tile's chunks, N narrower than one CTA
    tile and every batch class match the oracle, leave the ticket array
    untouched and repeat bit for bit."""
    w, ws = oracle.gen_weight_smoke(n, k, n + k)
    a, as_ = oracle.gen_activation_smoke(m, k, m + 5)
    ref = oracle.compute_reference(a, as_, w, ws)
    dc = DeviceCase(w, ws, a, as_, n)
    mt = dg.m_tile_for(m)
    kcfg = cfg(mt, bm, 1, 112, 2, 1, subs, pack, True, False, skf > 1, skf=skf)
    rc, got, status = run_reference_config(dc, kcfg)
    assert rc == 0 and status == 0, (rc, dg.status_string(status))
    ok, rl2, worst = check_against_oracle(got, ref)
    assert ok, (rl2, worst)
    assert dc.sem_clean()
    rc, got2, status = run_reference_config(dc, kcfg, clear_out=False)
    assert rc == 0 and status == 0 and np.array_equal(got, got2)


# ---------------------------------------------------------------------------
# B200 schedules
# ---------------------------------------------------------------------------

_C2 = {}


def c2_case(m: int):
    """C2 shape 7168 x 16384 with per-tensor-scaled N(0,1) inputs (BASELINE mode)."""
    n, k = 7168, 16384
    if "w" not in _C2:
        q, s, _ = oracle.gen_pertensor(n, k, 20260913, scale_rows=(n + 127) // 128, threads=8)
        _C2["w"] = (q, s)
    q, s = _C2["w"]
    key = ("m", m)
    if key not in _C2:
        for kk in [x for x in _C2 if x != "w"]:
            del _C2[kk]
        qa, sa, _ = oracle.gen_pertensor(m, k, 777 + m)
        ref = oracle.compute_reference(qa, sa, q, s, threads=8)
        _C2[key] = (DeviceCase(q, s, qa, sa, n), ref)
    return _C2[key]


@pytest.mark.parametrize("m", [1, 2, 4, 8, 16, 32, 64, 128])
@pytest.mark.parametrize("layout", [dg.LAYOUT_RAW, dg.LAYOUT_PACKED_SWIZZLED])
def test_c2_default_schedule_all_m(m, layout):
    dc, ref = c2_case(m)
    cfg_ = dg.default_config(m, dc.n, dc.k, layout=layout)
    rc, got, status = dc.run(cfg_)
    assert rc == 0 and status == 0
    ok, rl2, worst = check_against_oracle(got, ref)
    assert ok, (rl2, worst)
    assert dc.sem_clean()


@pytest.mark.parametrize("n,k", [(6144, 8192), (2048, 4096)])
@pytest.mark.parametrize("m", [1, 2, 4, 8, 16, 32])
@pytest.mark.parametrize("s", [1, 2, 4, 8])
def test_c4_split_k_parity_and_bit_determinism(n, k, m, s):
    """C4: split factors 1/2/4/8; results must be run-to-run bit-identical."""
    w, ws = oracle.gen_weight_smoke(n, k, 0x0F0F5678)
    a, as_ = oracle.gen_activation_smoke(m, k, 99 + m)
    ref = oracle.compute_reference(a, as_, w, ws, threads=8)
    dc = DeviceCase(w, ws, a, as_, n)
    c = dg.B200Config(m_tile=dg.m_tile_for(m), block_n=128, subs=1, layout=dg.LAYOUT_PACKED, split_k=s, pdl=True)
    runs = [dc.run(c) for _ in range(3)]
    for rc, got, status in runs:
        assert rc == 0 and status == 0
    ok, rl2, worst = check_against_oracle(runs[0][1], ref)
    assert ok, (rl2, worst)
    for _, got, _ in runs[1:]:
        assert np.array_equal(got.view(np.uint32), runs[0][1].view(np.uint32))
    assert dc.sem_clean()


@pytest.mark.parametrize("grid", [-1, 7, 100, 300])
def test_stream_k_bit_determinism(grid):
    n, k, m = 2048, 4096, 8
    w, ws = oracle.gen_weight_smoke(n, k, 5)
    a, as_ = oracle.gen_activation_smoke(m, k, 6)
    ref = oracle.compute_reference(a, as_, w, ws, threads=8)
    dc = DeviceCase(w, ws, a, as_, n)
    c = dg.B200Config(m_tile=8, block_n=128, subs=1, grid_ctas=grid)
    first = None
    for _ in range(4):
        rc, got, status = dc.run(c)
        assert rc == 0 and status == 0
        if first is None:
            first = got
            ok, rl2, worst = check_against_oracle(got, ref)
            assert ok, (rl2, worst)
        else:
            assert np.array_equal(got.view(np.uint32), first.view(np.uint32))


@pytest.mark.parametrize("m", [3, 9, 13, 37, 64, 100, 128])
@pytest.mark.parametrize("ws_offset", [0, 1])
def test_split_workspace_layouts(m, ws_offset):
    """Split tiles through both workspace layouts: 8-row blocks plus row-major
    tail rows (16-byte aligned workspace, bulk-copy reduction), and row-major
    only with plain loads (workspace one float off alignment); with the grid
    on one CTA per SM every contributor helps reduce.  Bit-identical across
    runs, tickets clean."""
    n, k = 2048, 4096
    w, ws = oracle.gen_weight_smoke(n, k, 41)
    a, as_ = oracle.gen_activation_smoke(m, k, 42 + m)
    ref = oracle.compute_reference(a, as_, w, ws, threads=8)
    dc = DeviceCase(w, ws, a, as_, n)
    c = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, schedule="stream_k")
    assert c.plan(m, n, k).max_slabs > 1
    first = None
    for _ in range(3):
        rc, got, status = dc.run(c, ws_offset=ws_offset)
        assert rc == 0 and status == 0, dg.status_string(status)
        if first is None:
            first = got
            ok, rl2, worst = check_against_oracle(got, ref)
            assert ok, (rl2, worst)
        else:
            assert np.array_equal(got.view(np.uint32), first.view(np.uint32))
    assert dc.sem_clean()


@pytest.mark.parametrize("n,k,m,bm", [(1, 128, 1, 128), (129, 256, 3, 128), (200, 384, 8, 48), (1000, 1152, 5, 64),
                                      (136, 4096, 1, 8), (777, 640, 17, 128), (96, 256, 128, 56)])
@pytest.mark.parametrize("layout", [0, 1, 2])
def test_ragged_shapes(n, k, m, bm, layout):
    """N not a multiple of the tile or of 128, a single K block, M at the edge of its bucket."""
    w, ws = oracle.gen_weight_smoke(n, k, n * 7 + k)
    a, as_ = oracle.gen_activation_smoke(m, k, m + 3)
    ref = oracle.compute_reference(a, as_, w, ws)
    dc = DeviceCase(w, ws, a, as_, n)
    for grid in (0, -1):
        c = dg.B200Config(m_tile=dg.m_tile_for(m), block_n=bm, subs=1, layout=layout, grid_ctas=grid)
        rc, got, status = dc.run(c)
        assert rc == 0 and status == 0
        ok, rl2, worst = check_against_oracle(got, ref)
        assert ok, (grid, rl2, worst)


@pytest.mark.parametrize("bm", [8, 32, 48, 56, 64, 128])
@pytest.mark.parametrize("layout", [dg.LAYOUT_PACKED, dg.LAYOUT_PACKED_SWIZZLED])
def test_prepack_bytes_match_oracle(bm, layout):
    import torch
    n, k = 333, 512
    rng = np.random.default_rng(bm)
    w = rng.integers(0, 256, (n, k), dtype=np.uint8)
    dst = dg.prepack_weight(torch.from_numpy(w).cuda(), bm, layout)
    torch.cuda.synchronize()
    want = oracle.prepack(w, bm, swizzled=(layout == dg.LAYOUT_PACKED_SWIZZLED))
    assert np.array_equal(dst.cpu().numpy(), want)


def test_pdl_back_to_back_split_k_stays_correct():
    """Overlapped launches with programmatic serialization on a split-K schedule:
    tickets must stay consistent (the reference's semaphore race case)."""
    import torch
    n, k, m = 2048, 4096, 4
    w, ws = oracle.gen_weight_smoke(n, k, 77)
    a, as_ = oracle.gen_activation_smoke(m, k, 78)
    ref = oracle.compute_reference(a, as_, w, ws)
    dc = DeviceCase(w, ws, a, as_, n)
    c = dg.B200Config(m_tile=8, block_n=64, subs=2, layout=0, pdl=True, split_k=8)
    rc, got, status = dc.run(c)
    assert rc == 0 and status == 0
    p = dg.Problem(m, n, k, dc.a, dc.w, dc.ws, dc.as_, dc.out, dc.splitk_ws, dc.sem, dc.status)
    wm, am = dg.make_weight_tma(c, p), dg.make_activation_tma(c, p)
    for _ in range(200):
        assert dg.launch_with_maps(c, p, wm, am, None, pdl_attr=True) == 0
    torch.cuda.synchronize()
    assert int(dc.status.item()) == 0
    assert dc.sem_clean()
    final = dc.out.float().cpu().numpy()
    assert np.array_equal(final.view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("schedule", ["stream_k", "cluster"])
@pytest.mark.parametrize("independent", [False, True])
def test_pdl_back_to_back_both_modes(independent, schedule):
    """Back-to-back launches (stream-K and cluster split-K) with programmatic
    serialization, with and without FLAG_INDEPENDENT_INPUTS: correct, tickets
    clean, bit-identical."""
    import torch
    n, k, m = 2048, 4096, 2
    w, ws = oracle.gen_weight_smoke(n, k, 81)
    a, as_ = oracle.gen_activation_smoke(m, k, 82)
    ref = oracle.compute_reference(a, as_, w, ws)
    dc = DeviceCase(w, ws, a, as_, n)
    c = dg.default_config(m, n, k, layout=dg.LAYOUT_RAW, independent_inputs=independent, schedule=schedule)
    rc, got, status = dc.run(c)
    assert rc == 0 and status == 0
    assert check_against_oracle(got, ref)[0]
    p = dg.Problem(m, n, k, dc.a, dc.w, dc.ws, dc.as_, dc.out, dc.splitk_ws, dc.sem, dc.status)
    wm, am = dg.make_weight_tma(c, p), dg.make_activation_tma(c, p)
    for _ in range(300):
        assert dg.launch_with_maps(c, p, wm, am, None, pdl_attr=True) == 0
    torch.cuda.synchronize()
    assert int(dc.status.item()) == 0
    assert dc.sem_clean()
    assert np.array_equal(dc.out.float().cpu().numpy().view(np.uint32), got.view(np.uint32))


def test_rejected_launches_return_invalid_value():
    import torch
    dc = DeviceCase(*oracle.gen_weight_smoke(256, 512, 1), *oracle.gen_activation_smoke(2, 512, 2), 256)
    p = dg.Problem(2, 256, 512, dc.a, dc.w, dc.ws, dc.as_, dc.out, None, None, dc.status)
    assert dg.launch(dg.B200Config(m_tile=8, block_n=128, split_k=2), p) == 1      # needs workspace
    assert dg.launch(dg.B200Config(m_tile=8, block_n=128, split_k=3), p) == 1      # 4 chunks % 3
    p_bad_k = dg.Problem(2, 256, 500, dc.a, dc.w, dc.ws, dc.as_, dc.out, None, None, dc.status)
    assert dg.launch(dg.B200Config(m_tile=8), p_bad_k) == 1
    p_big_m = dg.Problem(9, 256, 512, dc.a, dc.w, dc.ws, dc.as_, dc.out, None, None, dc.status)
    assert dg.launch(dg.B200Config(m_tile=8), p_big_m) == 1
    assert dg.launch(S6_m8, p) == 1                                                # reference split-K, no ws
    torch.cuda.synchronize()


def test_bounded_wait_timeout_reports_status_and_context_survives():
    """A wait that can never complete (the test hook) expires, the kernel
    records 0x51 and exits; the next launch on the same context is correct."""
    w, ws = oracle.gen_weight_smoke(512, 1024, 3)
    a, as_ = oracle.gen_activation_smoke(4, 1024, 4)
    ref = oracle.compute_reference(a, as_, w, ws)
    dc = DeviceCase(w, ws, a, as_, 512)
    hook = dg.B200Config(m_tile=8, block_n=128, subs=2, flags=dg.FLAG_INJECT_TIMEOUT, timeout_ns=50_000_000)
    rc, _, status = dc.run(hook)
    assert rc == 0 and status == dg.ERR_INJECTED_TIMEOUT
    rc, got, status = dc.run(dg.B200Config(m_tile=8, block_n=128, subs=2))
    assert rc == 0 and status == 0
    assert check_against_oracle(got, ref)[0]


def test_fp8_decode_gemm_torch_entry_point():
    import torch
    n, k, m = 1024, 2048, 3
    w, ws = oracle.gen_weight_smoke(n, k, 11)
    a, as_ = oracle.gen_activation_smoke(m, k, 12)
    ref = oracle.compute_reference(a, as_, w, ws)
    out = dg.fp8_decode_gemm(torch.from_numpy(a).cuda(), torch.from_numpy(as_).cuda(), torch.from_numpy(w).cuda(),
                             torch.from_numpy(ws).cuda())
    torch.cuda.synchronize()
    assert check_against_oracle(out.float().cpu().numpy(), ref)[0]
