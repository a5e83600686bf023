"""CPU tests of the C ABI library and the host logic (no kernel launches)."""

import ctypes
from dataclasses import replace
import os
import re

import pytest

import decode_opt_b200 as dg
from decode_opt_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for fname in os.listdir(os.path.join(ROOT, "include")):
        if not fname.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", fname)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names |= set(re.findall(r"\b(dg_\w+)\s*\(", text))
    return names


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    declared = declared_functions()
    assert declared, "no declarations found"
    assert declared == set(_lib.EXPORTED_SYMBOLS)
    for name in declared:
        assert hasattr(L, name), name
    assert L.dg_abi_version() == _lib.ABI_VERSION


def test_struct_layouts_match_header(tmp_path):
    """The ctypes mirrors have the C header's sizes and field offsets (compiled
    with the system C compiler against include/decode_gemm_b200.h)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    structs = {"dg_config": _lib.DgConfig, "dg_problem": _lib.DgProblem, "dg_plan_info": _lib.DgPlanInfo,
               "dg_gather": _lib.DgGather, "dg_gather_lines": _lib.DgGatherLines}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "decode_gemm_b200.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'  printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        name, field, val = line.split()
        got[(name, field)] = int(val)
    for cname, py in structs.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
    assert ctypes.sizeof(_lib.TensorMap) == 128


def test_prepack_geometry_matches_reference_formulas():
    # kernels/weight_prepack.cuh:45-52
    for n, bm in [(7168, 48), (7168, 56), (6144, 64), (2048, 32), (200, 128), (1, 8)]:
        assert dg.padded_n(n, bm) == _lib.lib().dg_padded_n(n, bm) == -(-n // bm) * bm
        assert dg.packed_weight_bytes(n, 4096, bm) == _lib.lib().dg_packed_weight_bytes(n, 4096, bm)


def test_status_strings():
    assert dg.status_string(0) == "ok"
    assert "injected" in dg.status_string(dg.ERR_INJECTED_TIMEOUT)
    assert dg.status_string(12345) == "unknown status"


@pytest.mark.parametrize("m", [1, 8, 16, 32, 64, 128])
def test_default_plan_c2_cluster(m):
    """Default schedule (no GPU: the measured B200 cluster occupancy): cluster
    split-K, 224-row tiles x 4 K-splits = 128 CTAs in one wave for dependent
    launches (the default batch class); for independent inputs one CTA per
    256-row tile (28 CTAs, no split; M <= 16 on the swap-AB class with three
    64 KiB stages), and with the tagged-lines gather 2 K-splits; no
    workspace."""
    c = dg.default_config(m, 7168, 16384)
    p = c.plan(m, 7168, 16384)
    assert p.error is None and c.grid_ctas == dg.GRID_CLUSTER and c.block_n == 224
    assert not c.flags & dg.FLAG_SWAP_AB
    assert p.cluster == 4 and p.grid == (32, 4, 1) and p.num_ctas == 128 and p.n_mma == 224
    assert p.stages == (3 if m <= 32 else 2)
    assert p.ws_floats == 0 and p.sem_ints == 0 and p.max_slabs == 1
    ci = dg.default_config(m, 7168, 16384, independent_inputs=True)
    pi = ci.plan(m, 7168, 16384)
    assert bool(ci.flags & dg.FLAG_SWAP_AB) == (m <= 16)
    assert ci.block_n == 256 and pi.cluster == 1 and pi.grid == (28, 1, 1) and pi.num_ctas == 28
    if m <= 16:
        assert (pi.mma_m, pi.n_mma, pi.stages) == (128, 16, 3)
    cl = dg.default_config(m, 7168, 16384, independent_inputs=True, gather_lines=True)
    pl = cl.plan(m, 7168, 16384)
    assert cl.block_n == 256 and pl.cluster == 2 and pl.num_ctas == 56
    assert dg.default_config(m, 7168, 16384, independent_inputs=True, swap_ab=False).block_n == 256
    # a small matrix: 16 chunks per tile, so 8 CTAs per tile (two chunks
    # each) rather than the ragged 10; 10 ragged 224-row tiles stream
    # 224 x 2 rows-chunks per CTA against 256 x 2
    sc = dg.default_config(m, 2048, 4096)
    small = sc.plan(m, 2048, 4096)
    assert sc.block_n == 224 and small.cluster == 8 and small.num_ctas == 80
    # tensor-parallel shards: 896 x 16384 (8 GPUs) on 4 tiles x 16 (a
    # non-portable cluster size), 3584 x 16384 (2 GPUs) on 14 tiles x 8 of
    # 256 rows (8 chunks per CTA) rather than 16 x 6 of 224 (11)
    s8 = dg.default_config(m, 896, 16384).plan(m, 896, 16384)
    assert s8.cluster == 16 and s8.num_ctas == 64
    c2 = dg.default_config(m, 3584, 16384)
    s2 = c2.plan(m, 3584, 16384)
    assert c2.block_n == 256 and s2.cluster == 8 and s2.num_ctas == 112
    # there the default class fits two 64 KiB stages, the swap-AB class three
    assert bool(c2.flags & dg.FLAG_SWAP_AB) == (m <= 16) and s2.stages == (3 if m <= 16 else 2)


@pytest.mark.parametrize("m", [1, 8, 16, 32, 64, 128])
def test_default_plan_c2(m):
    p = dg.default_config(m, 7168, 16384, schedule="stream_k").plan(m, 7168, 16384)
    assert p.error is None
    # weights on the MMA N side (256 rows per tile), batch on M: 64 rows (4
    # copies of 16 or 2 of 32) up to M = 32, else 128 rows (2 copies of 64, 1)
    assert p.mma_m == (64 if m <= 32 else 128) and p.n_mma == 256 and p.num_output_tiles == 28
    assert p.block[0] == {1: 192, 8: 192, 16: 192, 32: 320, 64: 320, 128: 384}[m]
    assert p.epi_warps == {1: 4, 8: 4, 16: 4, 32: 8, 64: 8, 128: 8}[m]
    assert p.a_rows == -(-m // 8) * 8
    assert p.smem_bytes <= 227 * 1024
    assert p.grid[0] == 148 or p.grid[0] > 0
    assert p.ws_floats == p.max_slabs * m * 7168 and p.sem_ints == 28


def test_plan_rejections():
    B = dg.B200Config
    assert B(m_tile=8).validate(9, 256, 512) == "M out of [1, m_tile]"
    assert "multiple of 128" in B(m_tile=8).validate(1, 256, 500)
    assert "subs" in B(m_tile=8, subs=4).validate(1, 256, 384)
    assert "split_k" in B(m_tile=8, split_k=3).validate(1, 256, 512)
    assert "m_tile" in B(m_tile=12).validate(1, 256, 512)
    assert "block_n" in B(m_tile=8, block_n=12).validate(1, 256, 512)
    assert "227" in B(m_tile=128, subs=4, stages=16).validate(128, 256, 4096)
    assert "epi_warps" in B(m_tile=8, epi_warps=5).validate(1, 256, 512)


@pytest.mark.parametrize("m", [1, 4, 16])
@pytest.mark.parametrize("independent", [False, True])
@pytest.mark.parametrize("n,k", [(7168, 16384), (16384, 7168), (2048, 4096), (896, 16384)])
def test_swap_ab_plans(m, n, k, independent):
    """The swap-AB class (FLAG_SWAP_AB): tcgen05.mma M = 128 weight rows x
    N = 16 batch rows, 7 warps (4 epilogue, producer, two MMA issuers), the
    cluster schedule with the split and tile width the default class gets
    for dependent launches, no workspace, one wave, within 227 KiB."""
    sw = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, independent_inputs=independent, swap_ab=True)
    assert sw.flags & dg.FLAG_SWAP_AB and sw.grid_ctas == dg.GRID_CLUSTER
    p = sw.plan(m, n, k)
    assert p.error is None, p.error
    assert (p.mma_m, p.n_mma, p.block[0], p.epi_warps) == (128, 16, 224, 4)
    assert p.ws_floats == 0 and p.sem_ints == 0
    assert p.smem_bytes <= dg.MAX_DYNAMIC_SMEM
    assert 136 <= sw.block_n <= 256 and sw.block_n % 8 == 0
    assert p.grid[0] * p.grid[1] <= 148
    if not independent:
        d = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, independent_inputs=False)
        pd = d.plan(m, n, k)
        assert (sw.block_n, p.grid) == (d.block_n, pd.grid)
        assert p.stages >= pd.stages


def test_swap_ab_plan_rejections():
    sw = dg.default_config(8, 2048, 4096, layout=dg.LAYOUT_RAW, swap_ab=True)
    assert "M must be <= 16" in replace(sw, m_tile=32).validate(17, 2048, 4096)
    assert "block_n" in replace(sw, block_n=128).validate(8, 2048, 4096)
    assert "cluster" in replace(sw, grid_ctas=-1).validate(8, 2048, 4096)
    assert "cluster" in replace(sw, grid_ctas=0, split_k=2).validate(8, 2048, 4096)
    assert replace(sw, grid_ctas=0, split_k=1).validate(8, 2048, 4096) is None
    with pytest.raises(ValueError):
        dg.default_config(17, 2048, 4096, swap_ab=True)
    with pytest.raises(ValueError):
        dg.default_config(8, 2048, 4096, schedule="stream_k", swap_ab=True)


def test_launch_rejections_need_no_gpu():
    B = dg.B200Config
    p = dg.Problem(9, 256, 512)
    assert dg.launch(B(m_tile=8), p) == 1
    assert dg.launch(B(m_tile=8), dg.Problem(1, 256, 500)) == 1
    # the input copy kernel refuses null pointers and empty copies before any CUDA call
    L = _lib.lib()
    assert L.dg_copy_from_host(None, ctypes.c_void_p(16), 16, None, 1) == dg.CUDA_ERROR_INVALID_VALUE
    assert L.dg_copy_from_host(ctypes.c_void_p(16), None, 16, None, 1) == dg.CUDA_ERROR_INVALID_VALUE
    assert L.dg_copy_from_host(ctypes.c_void_p(16), ctypes.c_void_p(32), 0, None, 0) == dg.CUDA_ERROR_INVALID_VALUE


def _units(G, U):
    return [(c * U // G, (c + 1) * U // G) for c in range(G)]


@pytest.mark.parametrize("T,C,G", [(56, 64, 148), (16, 16, 148), (128, 48, 256), (7, 128, 148), (3, 5, 15)])
def test_stream_k_partition_covers_units_once(T, C, G):
    """The kernel's CTA ranges and their inverse (dg_kernel.cuh cta_of_unit)."""
    U = T * C
    G = min(G, U)
    ranges = _units(G, U)
    assert ranges[0][0] == 0 and ranges[-1][1] == U
    for (a0, a1), (b0, _) in zip(ranges, ranges[1:]):
        assert a1 == b0 and a1 > a0
    for u in range(U):
        c = ((u + 1) * G - 1) // U
        lo, hi = ranges[c]
        assert lo <= u < hi


def test_reference_split_k_is_stream_k_special_case():
    """grid (tiles, S) linearised as x*S+y gives CTA y of tile x exactly the
    y-th of S equal K slices (the reference's S-way split)."""
    T, C, S = 64, 16, 4
    U, G = T * C, T * S
    for x in range(T):
        for y in range(S):
            c = x * S + y
            assert (c * U // G, (c + 1) * U // G) == (x * C + y * C // S, x * C + (y + 1) * C // S)


def test_kernel_config_mirror_reference_rules():
    KC = dg.KernelConfig
    s6 = KC(8, 48, 2, 80, 3, 1, 2, True, True, True, True)
    assert s6.kSplitKFactor == 2 and s6.kSplitKCta
    assert KC(8, 32, 2, 80, 3, 1, 2, True, True, True, True, SPLITK_FACTOR=8).kSplitKFactor == 8
    assert KC(8, 48, 2, 80, 3, 1, 2, True, True, True, False).kSplitKFactor == 1
    # k_ok_for_splitk pins of kernels/smoke_test.cu:481-486
    q8 = KC(8, 32, 2, 80, 3, 1, 2, True, True, True, True, SPLITK_FACTOR=8)
    assert q8.k_ok_for_splitk(4096)
    assert KC(8, 56, 2, 80, 3, 1, 2, True, True, True, True, SPLITK_FACTOR=8).k_ok_for_splitk(12288)
    # validate() messages are the reference's
    assert s6.validate(9, 6144, 7168) == "M out of [1, M_TILE]"
    assert s6.validate(1, 6144, 7000) == "K must be a multiple of 128"
    assert KC(8, 64, 1, 112, 4, 1, 4, True, True, True, False).validate(1, 2048, 384) == \
        "K/128 must be a multiple of SUBS_PER_STAGE"
    assert s6.validate(1, 6144, 7168) is None
    # static_assert mirrors
    with pytest.raises(ValueError):
        KC(12, 48, 2, 80, 3, 1, 2, True, True, True, False)
    with pytest.raises(ValueError):
        KC(8, 48, 2, 80, 3, 1, 2, False, True, True, False, PRELOAD_ACT=True)
    with pytest.raises(ValueError):
        KC(8, 48, 4, 168, 3, 1, 2, True, True, True, False)      # register budget
    with pytest.raises(ValueError):
        KC(8, 48, 2, 80, 3, 1, 2, True, True, True, True, SPLITK_FACTOR=1)


def test_kernel_config_maps_onto_b200_config():
    """A reference configuration runs T = 256 // BM of its BM-row tiles per
    CTA (224 rows at BM 56) in the reference's packed layout, on the cluster
    split (4 unless SPLITK_FACTOR says otherwise); the plan keeps the
    reference's meanings of num_output_tiles and padded_n."""
    k = dg.KernelConfig(8, 56, 2, 80, 3, 1, 2, True, True, False, False)
    b = k.to_b200()
    assert (b.m_tile, b.block_n, b.pack_rows, b.subs, b.stages, b.layout, b.pdl, b.split_k, b.grid_ctas) == \
        (8, 224, 56, 2, 6, dg.LAYOUT_PACKED, True, 4, dg.GRID_CLUSTER)
    assert b.packed_rows == 56 and k.kBlockN == 224 and k.num_ctas(7168) == 128
    plan = dg.make_launch_plan(k, dg.Problem(1, 7168, 16384))
    assert plan.error is None and plan.grid == (32, 4, 1) and plan.cluster == 4
    assert plan.mma_m == 64 and plan.n_mma == 224 and plan.ws_floats == 0 and plan.sem_ints == 0
    assert plan.num_output_tiles == 128 and plan.padded_n == 7168
    # BM 48 on N = 7168: 150 packed tiles (padded_n 7200), five per CTA tile.
    k48 = dg.KernelConfig(8, 48, 2, 80, 3, 1, 2, True, True, True, True, SPLITK_FACTOR=8)
    p48 = dg.make_launch_plan(k48, dg.Problem(8, 7168, 16384))
    assert p48.error is None and p48.grid == (30, 8, 1) and p48.n_mma == 240
    assert p48.num_output_tiles == 150 and p48.padded_n == 7200
    # Raw weights: the tile width alone (no packed tile height).
    kr = dg.KernelConfig(128, 64, 1, 232, 2, 1, 1, False, True, False, False, SCALE_IN_SMEM=False)
    br = kr.to_b200()
    assert br.block_n == 256 and br.pack_rows == 0 and br.layout == dg.LAYOUT_RAW
    # The ring is deepened until the cluster partial of M_TILE rows fits.
    assert br.stages >= dg.cluster_min_stages(128, 1, 256, 128) == 3
    assert dg.make_launch_plan(kr, dg.Problem(128, 7168, 16384)).error is None


B200_CLUSTER_OCC = [0, 148, 74, 45, 33, 26, 22, 15, 15,      # clusters of S CTAs resident at once (measured)
                    15, 11, 7, 7, 7, 7, 7, 7]


def _rule_split(t, c, independent):
    """The split rule restated: independent inputs -> one CTA per tile from 24
    tiles, else the smallest one-wave S giving >= 32 CTAs (S <= 8); dependent
    -> the smallest one-wave S (S <= 16, at most 148 - 20 CTAs) with the
    fewest chunks for the busiest CTA, ceil(C / S); both S <= C."""
    if independent and t >= dg.INDEPENDENT_TILE_CTAS:
        return 1
    s_max = min(c, 8 if independent else 16)
    if not independent:
        best, best_chunks = 1, c
        for s in range(2, s_max + 1):
            if t <= B200_CLUSTER_OCC[s] and t * s <= 128 and -(-c // s) < best_chunks:
                best, best_chunks = s, -(-c // s)
        return best
    if independent:
        for s in range(2, s_max + 1):
            if t <= B200_CLUSTER_OCC[s] and t * s >= 32:
                return s
    for s in range(s_max, 1, -1):
        if t <= B200_CLUSTER_OCC[s]:
            return s
    return 1


@pytest.mark.parametrize("n,k", [(7168, 16384), (7168, 12288), (6144, 16384), (6144, 8192), (2048, 4096)])
@pytest.mark.parametrize("m", [1, 8, 16, 17, 32, 33, 64, 65, 128])
@pytest.mark.parametrize("independent", [False, True])
def test_default_plans_follow_the_split_rule(n, k, m, independent):
    """Every BASELINE model shape: the default plan is a one-wave cluster
    split-K plan whose split is the rule's pick for its tile count, with no
    workspace, a ring that fits, and the batch class M calls for."""
    c = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, independent_inputs=independent)
    p = c.plan(m, n, k)
    assert p.error is None
    assert c.grid_ctas == dg.GRID_CLUSTER and c.block_n in (224, 256)
    tiles = -(-n // c.block_n)
    chunks = (k // 128) // c.subs
    assert p.grid == (tiles, p.cluster, 1) and p.num_ctas == tiles * p.cluster
    assert p.cluster == _rule_split(tiles, chunks, independent)
    assert tiles <= B200_CLUSTER_OCC[p.cluster]                  # one wave of clusters
    assert p.ws_floats == 0 and p.sem_ints == 0
    assert p.stages >= 2 and p.smem_bytes <= 227 * 1024
    if c.flags & dg.FLAG_SWAP_AB:
        # swap-AB (M <= 16; independent inputs, or a 256-row dependent plan):
        # MMA M = 128 weight rows x N = 16 batch rows, 7 warps
        assert m <= 16 and c.block_n == 256 and (independent or p.stages == 3)
        assert (p.mma_m, p.n_mma, p.block[0]) == (128, 16, 224)
    else:
        assert not (independent and m <= 16)
        assert p.mma_m == (64 if m <= 32 else 128)
        assert p.block[0] == (192 if m <= 16 else 320 if m <= 64 else 384)
    if independent:
        # one CTA per 256-row tile from 24 tiles, else >= 32 CTAs if a split allows
        assert (p.cluster == 1 and c.block_n == 256 and tiles >= dg.INDEPENDENT_TILE_CTAS) or \
            p.num_ctas >= 32 or p.cluster == min(chunks, 8)


@pytest.mark.parametrize("bn", list(range(32, 257, 8)))
def test_cluster_partial_layout_rules(bn):
    """The cluster reduction's index rules: a row's float4 unit c4 is stored at
    c4 ^ (m % 8) in a row of ceil(bn/32)*32 floats -- one-to-one and inside
    the row for every bn that is a multiple of 8, so the planner takes any
    such width -- and the S ranks' unit ranges [r*q/S, (r+1)*q/S) cover all
    q = M * ceil(bn_t/4) units once."""
    units = bn // 4
    row_units = ((bn + 31) // 32) * 8
    for m in range(8):
        slots = [c ^ m for c in range(units)]
        assert len(set(slots)) == units and max(slots) < row_units
    plan = dg.B200Config(m_tile=8, block_n=bn, subs=2, stages=0, layout=dg.LAYOUT_PACKED_SWIZZLED,
                         grid_ctas=dg.GRID_CLUSTER, split_k=4).plan(1, 7168, 16384)
    assert plan.error is None, plan.error
    for m_rows in (1, 7, 64):
        for bn_t in (bn, max(4, bn - 20)):
            q = m_rows * -(-bn_t // 4)
            for s in (2, 3, 4, 8):
                cover = [u for r in range(s) for u in range(r * q // s, (r + 1) * q // s)]
                assert cover == list(range(q))


@pytest.mark.parametrize("m,n,k", [(1, 7168, 16384), (1, 16384, 7168), (64, 2048, 4096), (3, 640, 512),
                                   (128, 128, 256)])
def test_quantized_output_config(m, n, k):
    """The configuration dg.launch_quantized takes: cluster split-K on
    256-row tiles (whole 128-column quantisation blocks in every tile), no
    workspace; refused where N is not a multiple of 128."""
    c = dg.default_config(m, n, k, layout=dg.LAYOUT_PACKED_SWIZZLED, quantized_output=True)
    p = c.plan(m, n, k)
    assert p.error is None and c.grid_ctas == dg.GRID_CLUSTER and c.block_n == 256
    assert p.grid == (-(-n // 256), p.cluster, 1) and p.cluster >= 2 and p.ws_floats == 0 and p.sem_ints == 0
    with pytest.raises(ValueError):
        dg.default_config(m, n + 64, k, quantized_output=True)
    with pytest.raises(ValueError):
        dg.default_config(m, n, k, schedule="stream_k", quantized_output=True)
