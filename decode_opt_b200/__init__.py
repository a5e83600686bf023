"""B200 (sm_100a) FP8 decode GEMM -- Python host interface.

Mirrors the reference's C++ host API (``namespace decode_gemm`` in
``kernels/decode_gemm.cuh`` and ``kernels/weight_prepack.cuh`` of
ziyuhuang123/decode_opt) over the C ABI of ``libdecode_gemm_b200.so``:

=============================  ===========================================
reference (C++)                here
=============================  ===========================================
``KernelConfig<...>``          :class:`KernelConfig` (same 16 parameters)
``Problem``                    :class:`Problem`
``LaunchPlan``                 :class:`LaunchPlan`
``Cfg::validate(m, n, k)``     :meth:`KernelConfig.validate`
``make_launch_plan<Cfg>``      :func:`make_launch_plan`
``make_weight_tma<Cfg>``       :func:`make_weight_tma`
``make_activation_tma<Cfg>``   :func:`make_activation_tma`
``launch_with_maps<Cfg>``      :func:`launch_with_maps`
``launch<Cfg>``                :func:`launch`
``prepack::padded_n``          :func:`padded_n`
``prepack::packed_weight_bytes`` :func:`packed_weight_bytes`
``prepack::launch_prepack_weight<BM,TILES>`` :func:`launch_prepack_weight`
=============================  ===========================================

Errors follow the reference: launches return a ``cudaError_t`` integer (0 ok,
1 = ``cudaErrorInvalidValue`` for an unsupported shape or a missing split-K
workspace), ``validate`` returns a reason string or None.

:class:`B200Config` exposes the B200 schedule directly (stream-K grid,
descriptor-ready weight layout) and :func:`fp8_decode_gemm` is a one-call
torch entry point.  Everything runs through the CUDA library; when it is
missing, importing the launch functions raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional

from . import _lib
from ._lib import (ERR_INJECTED_TIMEOUT, FLAG_INDEPENDENT_INPUTS, FLAG_INJECT_TIMEOUT, FLAG_SWAP_AB, GRID_CLUSTER,
                   LAYOUT_PACKED, LAYOUT_PACKED_SWIZZLED, LAYOUT_RAW, STATUS_OK, DgConfig, DgPlanInfo, DgProblem,
                   TensorMap)

__all__ = [
    "cluster_min_stages",
    "KernelConfig", "B200Config", "Problem", "LaunchPlan", "make_launch_plan", "make_weight_tma",
    "make_activation_tma", "launch_with_maps", "launch", "launch_gather", "quantize_activation", "padded_n",
    "packed_weight_bytes",
    "launch_prepack_weight", "prepack_weight", "fp8_decode_gemm", "default_config", "status_string",
    "LAYOUT_RAW", "LAYOUT_PACKED", "LAYOUT_PACKED_SWIZZLED", "FLAG_INJECT_TIMEOUT", "FLAG_INDEPENDENT_INPUTS",
    "FLAG_SWAP_AB",
    "ERR_INJECTED_TIMEOUT", "STATUS_OK", "m_tile_for", "flush_l2", "GRID_CLUSTER", "copy_from_host",
]

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1
K_BLOCK = 128
INDEPENDENT_TILE_CTAS = 24     # dg::kIndependentTileCtas: independent inputs run one CTA per tile from here
MAX_DYNAMIC_SMEM = 227 * 1024


def m_tile_for(m: int) -> int:
    """The reference's M ladder (bench/bench_common.cuh:103-109)."""
    for t in (8, 16, 32, 64):
        if m <= t:
            return t
    return 128


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_handle(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(stream.cuda_stream)


# ---------------------------------------------------------------------------
# Configurations
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class B200Config:
    """Runtime configuration of the sm_100a kernel (``dg_config``)."""

    m_tile: int = 8
    block_n: int = 256
    subs: int = 1
    stages: int = 0
    layout: int = LAYOUT_RAW
    pdl: bool = False
    split_k: int = 1
    grid_ctas: int = 0
    epi_warps: int = 0
    flags: int = 0
    timeout_ns: int = 0
    pack_rows: int = 0

    def to_dg(self) -> DgConfig:
        return DgConfig(self.m_tile, self.block_n, self.subs, self.stages, self.layout, int(self.pdl),
                        self.split_k, self.grid_ctas, self.epi_warps, self.flags, self.timeout_ns,
                        self.pack_rows)

    def plan(self, m: int, n: int, k: int) -> "LaunchPlan":
        info = DgPlanInfo()
        _lib.lib().dg_plan(ctypes.byref(self.to_dg()), m, n, k, ctypes.byref(info))
        return LaunchPlan._from_info(info)

    def validate(self, m: int, n: int, k: int) -> Optional[str]:
        return self.plan(m, n, k).error

    def max_active_clusters(self, m: int, n: int, k: int) -> int:
        """Clusters of this plan's size the current GPU holds at once
        (``dg_max_active_clusters``)."""
        out = ctypes.c_int()
        rc = _lib.lib().dg_max_active_clusters(ctypes.byref(self.to_dg()), m, n, k, ctypes.byref(out))
        if rc != 0:
            raise RuntimeError(f"dg_max_active_clusters failed: cudaError {rc}")
        return out.value

    @property
    def prepacked(self) -> bool:
        return self.layout != LAYOUT_RAW

    @property
    def packed_rows(self) -> int:
        """Rows per tile of the packed weight layout this configuration reads
        (the ``block_n`` argument of :func:`prepack_weight`)."""
        return self.pack_rows or self.block_n


def default_config(m: int, n: int, k: int, layout: int = LAYOUT_RAW, pdl: bool = True,
                   independent_inputs: bool = False, schedule: str = "cluster",
                   quantized_output: bool = False, swap_ab: Optional[bool] = None,
                   gather_lines: bool = False) -> B200Config:
    """The B200 schedule used by :func:`fp8_decode_gemm` and the benchmark.

    Two 128-K blocks per stage and weight tiles of 256 rows unless 224 serves
    better:

    * ``schedule="cluster"`` (default): cluster split-K (``GRID_CLUSTER``):
      each tile's K range split over the CTAs of one thread-block cluster,
      reduced through distributed shared memory; the library picks the split
      from the device's cluster occupancy (one wave of clusters).  Dependent
      launches take the split and tile width (256 or 224 rows) whose busiest
      CTA streams the least, block_n x ceil(chunks / S), with clusters of up
      to 16 CTAs (7168 rows: 32 x 4 CTAs of 224 instead of 28 x 4 of 256; a
      3584-row shard: 14 x 8 of 256 instead of 16 x 6 of 224).  Independent
      inputs take 256-row tiles and one CTA per tile where that gives at
      least 24 CTAs (no split, no reduction: C2 runs 28 CTAs per GEMM and
      about five GEMMs stream side by side), else the smallest split giving
      32 CTAs (224 rows where that allows a deeper ring).  Falls back to
      stream-K where the cluster plan does not apply.
    * ``schedule="stream_k"``: a stream-K grid of one CTA per SM with the
      workspace reduction (two 64 KiB stages).

    `independent_inputs` sets FLAG_INDEPENDENT_INPUTS (see
    include/decode_gemm_b200.h).  `quantized_output` asks for a configuration
    :func:`launch_quantized` accepts: the cluster schedule on 256-row tiles
    (whole 128-column quantisation blocks per tile) with at least two CTAs per
    tile; ValueError where the cluster plan does not apply or N is not a
    multiple of 128.  `gather_lines` asks for one the tagged-lines gather
    accepts (``FusedGather(protocol="lines")``): the configuration chosen as
    above with at least two CTAs per tile (the gather stores from the cluster
    reduction), ValueError where the cluster schedule does not apply.

    `swap_ab` picks the batch class for M <= 16.  True: the swap-AB class
    (FLAG_SWAP_AB: the weights on the MMA's M side, 128 rows per
    tcgen05.mma, the batch padded to 16 on its N side, a quarter of the
    multiply-adds per weight byte) with the tile width and split chosen as
    above, ValueError where it does not apply; False: the default class
    (batch on the M side, padded to 64); None (default): the faster of the
    two as measured at C2 on B200 -- swap-AB for independent inputs (256-row
    tiles with 192 KiB in flight each: 16.3 against 17.4 us per GEMM over
    1,000 launches at a split of 2, 17.3 against 19.4 over 10,000 where the
    power limit lowers the clock) and for quantised output (three 64 KiB
    stages where the default class fits two: 22.8 against 23.9 us per layer
    of the 61-layer chain); for dependent launches the default class (22.5
    against 23.3 us at 224-row tiles) unless its plan takes 256-row tiles,
    where the swap class keeps a third stage.
    """
    from dataclasses import replace
    if gather_lines and not quantized_output:
        cfg = default_config(m, n, k, layout=layout, pdl=pdl, independent_inputs=independent_inputs,
                             schedule=schedule, swap_ab=swap_ab)
        pl = cfg.plan(m, n, k)
        if cfg.grid_ctas != GRID_CLUSTER or pl.error is not None:
            raise ValueError(f"no tagged-lines plan for M={m} N={n} K={k}: needs the cluster schedule ({pl.error})")
        if pl.cluster < 2:
            cfg = replace(cfg, split_k=2)
            err = cfg.plan(m, n, k).error
            if err is not None:
                raise ValueError(f"no tagged-lines plan for M={m} N={n} K={k}: {err}")
        return cfg
    reduce_in_cluster = quantized_output
    if swap_ab is None:
        kw = dict(layout=layout, pdl=pdl, independent_inputs=independent_inputs, schedule=schedule,
                  quantized_output=quantized_output)
        plain = default_config(m, n, k, swap_ab=False, **kw)
        if m > 16 or schedule != "cluster" or plain.grid_ctas != GRID_CLUSTER:
            return plain
        if not (independent_inputs or reduce_in_cluster or plain.block_n == 256):
            return plain
        try:
            sw = default_config(m, n, k, swap_ab=True, **kw)
        except ValueError:
            return plain
        psw = sw.plan(m, n, k)
        ok = psw.error is None and sw.block_n == 256 and (psw.cluster >= 2 or (independent_inputs and not
                                                                                 reduce_in_cluster))
        return sw if ok else plain
    if swap_ab and (schedule != "cluster" or m > 16):
        raise ValueError(f"no swap-AB plan for M={m}: needs M <= 16 and the cluster schedule")
    flags = FLAG_INDEPENDENT_INPUTS if independent_inputs else 0
    stream_k = B200Config(m_tile=m_tile_for(m), block_n=256, subs=2, stages=2, layout=layout, pdl=pdl,
                          split_k=1, grid_ctas=-1, flags=flags)
    if schedule == "stream_k" and not reduce_in_cluster:
        return stream_k
    if schedule not in ("cluster", "stream_k"):
        raise ValueError("schedule must be 'cluster' or 'stream_k'")
    base = replace(stream_k, grid_ctas=GRID_CLUSTER, stages=0)
    if swap_ab:
        base = replace(base, flags=base.flags | FLAG_SWAP_AB)
    p256 = base.plan(m, n, k)
    if reduce_in_cluster:
        if schedule != "cluster" or (quantized_output and n % 128 != 0) or p256.error is not None:
            raise ValueError(f"no cluster-reduction plan for M={m} N={n} K={k}: needs the cluster schedule "
                             f"(and N a multiple of 128 for quantised output) ({p256.error})")
        if p256.cluster < 2:
            # The quantisation runs in the cluster reduction: at least two
            # CTAs per tile (a CTA without a K chunk adds a zero partial).
            base = replace(base, split_k=2)
            err = base.plan(m, n, k).error
            if err is not None:
                raise ValueError(f"no cluster-reduction plan for M={m} N={n} K={k}: {err}")
        return base
    if not independent_inputs:
        # Dependent launches stream at ~50 GB/s per SM: the tile width whose
        # busiest CTA streams the fewest weight rows x chunks (block_n x
        # ceil(C / S)), fewer CTAs on a tie.
        alt = replace(base, block_n=224)
        p224 = alt.plan(m, n, k)
        chunks = (k // K_BLOCK) // base.subs
        cands = [(c, pl) for c, pl in ((base, p256), (alt, p224)) if pl.error is None and pl.cluster >= 2]
        if not cands:
            return _no_swap_fallback(swap_ab, stream_k, base, m, n, k, p256.error)
        return min(cands, key=lambda cp: (cp[0].block_n * -(-chunks // cp[1].cluster), cp[1].num_ctas))[0]
    if p256.error is None and p256.cluster == 1 and -(-n // 256) >= INDEPENDENT_TILE_CTAS:
        return base                      # one CTA per 256-row tile
    if p256.error is not None or p256.cluster < 2:
        return _no_swap_fallback(swap_ab, stream_k, base, m, n, k, p256.error)
    if n % 224 == 0:
        alt = replace(base, block_n=224)
        p224 = alt.plan(m, n, k)
        if p224.error is None and p224.cluster >= 2:
            if p224.stages > p256.stages:
                return alt
    return base


def _no_swap_fallback(swap_ab, stream_k, base, m, n, k, err):
    """default_config's stream-K fallback where no cluster split applies.  The
    swap-AB class has no stream-K schedule: it keeps the cluster schedule
    (one CTA per tile, stored directly, when no split fits) or raises."""
    if swap_ab:
        if err is not None:
            raise ValueError(f"no swap-AB cluster plan for M={m} N={n} K={k} ({err})")
        return base
    return stream_k


def cluster_min_stages(m: int, subs: int, block_n: int, mma_m: int) -> int:
    """The shallowest ring whose shared memory holds the fp32 partial of m
    rows (rows padded to a multiple of 32 floats) that cluster split-K keeps
    there (dg::cluster_min_stages)."""
    def align1k(v):
        return (v + 1023) & ~1023
    stride = (block_n + 31) & ~31
    pad = (((block_n + 15) // 16) * 16 - block_n) * K_BLOCK
    s = 1
    while s < 16 and (align1k(s * subs * block_n * K_BLOCK + pad) + align1k(s * subs * mma_m * K_BLOCK)
                      < m * stride * 4):
        s += 1
    return s


@dataclass(frozen=True)
class KernelConfig:
    """The reference's ``decode_gemm::KernelConfig`` (kernels/decode_gemm.cuh:147-347).

    Same parameters, in the same order, with the same defaults.  On sm_100a
    they map onto :class:`B200Config` as follows:

    * ``M_TILE`` -> ``m_tile`` (the batch is the tcgen05 M side, padded to 64,
      or 128 for M_TILE=128);
    * ``OUTPUT_ROWS_PER_CTA`` (BM) -> the packed layout's tile height
      (``pack_rows``); a CTA takes ``T = 256 // BM`` consecutive BM-row tiles
      (the reference's TILES_PER_CTA idea sized for the tcgen05 N side), so
      ``block_n = T * BM`` weight rows per MMA (224-256 for BM 32..64);
    * ``SUBS_PER_STAGE`` -> ``subs``; ``NUM_MATH_WG * STAGES_PER_WG`` -> ``stages``
      (the ring depth, raised to hold the cluster partial and reduced if it
      does not fit in 227 KiB);
    * ``PREPACK`` -> weight layout packed (True) or raw (False);
    * ``PDL`` or ``EPI_OVERLAP`` -> ``griddepcontrol.launch_dependents`` after
      the producer's first ring pass (the sm_100a kernel has one trigger
      point, earlier than the reference's after-the-last-TMA trigger);
      ``launch`` sets programmatic stream serialization when ``PDL``;
    * ``SPLIT_K_CTA`` / ``SPLITK_FACTOR`` -> the cluster split of every tile's
      K range: max(kSplitKFactor, 4), kSplitKFactor with the reference's
      normalisation (0: follow the bool, 1: off, 2/4/8: S) -- the reference's
      factor split BM-row tiles and a CTA tile here spans T of them; grid
      ``(ceil(N / block_n), S)``, one thread-block cluster per tile, reduced
      in rank order through distributed shared memory (deterministic; the
      workspace and semaphore are not touched);
    * ``NUM_MATH_WG``, ``MATH_REGS``, ``PROD_REGS``, ``SINGLE_PRODUCER_WARP``,
      ``PRELOAD_ACT``, ``SCALE_IN_SMEM``, ``TILES_PER_CTA`` describe the SM90
      warp-group / register split.  They are range-checked exactly as the
      reference's static_asserts check them and otherwise do not change the
      sm_100a kernel, whose warp roles are fixed (TMA warp, MMA warp,
      epilogue warps).
    """

    M_TILE: int
    OUTPUT_ROWS_PER_CTA: int
    NUM_MATH_WG: int
    MATH_REGS: int
    STAGES_PER_WG: int
    TILES_PER_CTA: int
    SUBS_PER_STAGE: int
    PREPACK: bool
    PDL: bool
    EPI_OVERLAP: bool
    SPLIT_K_CTA: bool
    PROD_REGS: int = 32
    SINGLE_PRODUCER_WARP: bool = False
    PRELOAD_ACT: bool = False
    SCALE_IN_SMEM: Optional[bool] = None
    SPLITK_FACTOR: int = 0

    def __post_init__(self):
        # The reference's static_asserts (kernels/decode_gemm.cuh:166-198), kept
        # as construction-time errors.
        mt, bm, wg = self.M_TILE, self.OUTPUT_ROWS_PER_CTA, self.NUM_MATH_WG
        if mt not in (8, 16, 32, 64, 128):
            raise ValueError("M_TILE must be one of 8/16/32/64/128")
        if not (0 < bm <= 64 and bm % 8 == 0) and bm not in (128, 256):
            raise ValueError("OUTPUT_ROWS_PER_CTA (BM) must be a multiple of 8 in (0, 64] "
                             "(or 128 / 256, the B200 wide-tile extension)")
        if wg not in (1, 2, 4):
            raise ValueError("NUM_MATH_WG must be 1, 2 or 4")
        if self.TILES_PER_CTA <= 0 or wg % self.TILES_PER_CTA != 0:
            raise ValueError("NUM_MATH_WG must be divisible by TILES_PER_CTA")
        if self.STAGES_PER_WG <= 0:
            raise ValueError("STAGES_PER_WG must be positive")
        if not (0 < self.SUBS_PER_STAGE <= 64):
            raise ValueError("SUBS_PER_STAGE must be in [1, 64]")
        for name in ("MATH_REGS", "PROD_REGS"):
            v = getattr(self, name)
            if not (24 <= v <= 256 and v % 8 == 0):
                raise ValueError(f"{name} must be a multiple of 8 in the PTX range [24, 256]")
        if (wg * self.MATH_REGS + self.PROD_REGS) * 128 > 65536:
            raise ValueError("register budget exceeded: (WG*MATH_REGS + PROD_REGS)*128 <= 65536")
        if self.PRELOAD_ACT and not (mt == 8 and self.PREPACK):
            raise ValueError("PRELOAD_ACT is only allowed for M_TILE=8 + PREPACK (CONTRACT 4)")
        if self.SPLITK_FACTOR not in (0, 1, 2, 4, 8):
            raise ValueError("SPLITK_FACTOR must be 0 (legacy: follow SPLIT_K_CTA), 1 (off), 2, 4 or 8")
        if self.SPLITK_FACTOR == 1 and self.SPLIT_K_CTA:
            raise ValueError("SPLITK_FACTOR=1 means split-K off and contradicts SPLIT_K_CTA=true")

    # ---- the reference's derived constants ---------------------------------
    @property
    def kMTile(self) -> int:
        return self.M_TILE

    @property
    def kOutputRows(self) -> int:
        return self.OUTPUT_ROWS_PER_CTA

    @property
    def kNumMathWgs(self) -> int:
        return self.NUM_MATH_WG

    @property
    def kStagesPerMathWg(self) -> int:
        return self.STAGES_PER_WG

    @property
    def kOutputTilesPerCta(self) -> int:
        return self.TILES_PER_CTA

    @property
    def kSubsPerStage(self) -> int:
        return self.SUBS_PER_STAGE

    @property
    def kPrepack(self) -> bool:
        return self.PREPACK

    @property
    def kPdl(self) -> bool:
        return self.PDL

    @property
    def kEpiOverlap(self) -> bool:
        return self.EPI_OVERLAP

    @property
    def kSplitKFactor(self) -> int:
        s = self.SPLITK_FACTOR
        if s >= 2:
            return s
        return 1 if (s == 1 or not self.SPLIT_K_CTA) else 2

    @property
    def kSplitKCta(self) -> bool:
        return self.kSplitKFactor > 1

    @property
    def kScaleInSmem(self) -> bool:
        return self.M_TILE <= 16 if self.SCALE_IN_SMEM is None else bool(self.SCALE_IN_SMEM)

    @property
    def kWgsPerOutputTile(self) -> int:
        return self.NUM_MATH_WG // self.TILES_PER_CTA

    @property
    def kStages(self) -> int:
        return self.NUM_MATH_WG * self.STAGES_PER_WG

    @property
    def kPackTiles(self) -> int:
        """BM-row tiles one CTA tile spans."""
        bm = self.OUTPUT_ROWS_PER_CTA
        return 256 // bm if bm <= 128 else 1

    @property
    def kBlockN(self) -> int:
        """Weight rows per CTA tile (the tcgen05 N side)."""
        return self.OUTPUT_ROWS_PER_CTA * self.kPackTiles

    @property
    def kClusterSplit(self) -> int:
        """CTAs per tile (one cluster), splitting its K range: at least 4,
        SPLITK_FACTOR when that asks for more."""
        return max(self.kSplitKFactor, 4)

    def to_b200(self) -> B200Config:
        bn = self.kBlockN
        mma_m = 64 if self.M_TILE <= 32 else 128
        stages = min(max(self.kStages, cluster_min_stages(self.M_TILE, self.SUBS_PER_STAGE, bn, mma_m)), 16)
        return B200Config(m_tile=self.M_TILE, block_n=bn,
                          pack_rows=self.OUTPUT_ROWS_PER_CTA if (self.PREPACK and self.kPackTiles > 1) else 0,
                          subs=self.SUBS_PER_STAGE, stages=stages,
                          layout=LAYOUT_PACKED if self.PREPACK else LAYOUT_RAW,
                          pdl=bool(self.PDL or self.EPI_OVERLAP), split_k=self.kClusterSplit,
                          grid_ctas=GRID_CLUSTER)

    def _fitted(self, m: int, n: int, k: int) -> B200Config:
        # The ring depth asked for, reduced until it fits.
        cfg = self.to_b200()
        stages = cfg.stages
        while stages > 1:
            c = B200Config(**{**cfg.__dict__, "stages": stages})
            if c.plan(m, n, k).error != "dynamic shared memory exceeds 227 KiB":
                return c
            stages -= 1
        return B200Config(**{**cfg.__dict__, "stages": 1})

    def num_output_tiles(self, n: int) -> int:
        return (n + self.OUTPUT_ROWS_PER_CTA - 1) // self.OUTPUT_ROWS_PER_CTA

    def num_ctas_x(self, n: int) -> int:
        return (n + self.kBlockN - 1) // self.kBlockN

    def num_ctas(self, n: int) -> int:
        return self.num_ctas_x(n) * self.kClusterSplit

    def k_ok_for_splitk(self, k: int) -> bool:
        return k % (K_BLOCK * self.SUBS_PER_STAGE * self.kWgsPerOutputTile * self.kSplitKFactor) == 0

    def validate(self, m: int, n: int, k: int) -> Optional[str]:
        """The reference's rules (kernels/decode_gemm.cuh:319-346), same messages."""
        if m < 1 or m > self.M_TILE:
            return "M out of [1, M_TILE]"
        if n < 1:
            return "N must be positive"
        if k % K_BLOCK != 0:
            return "K must be a multiple of 128"
        kb = k // K_BLOCK
        if kb % self.SUBS_PER_STAGE != 0:
            return "K/128 must be a multiple of SUBS_PER_STAGE"
        chunks = kb // self.SUBS_PER_STAGE
        if chunks % self.kWgsPerOutputTile != 0:
            return "K/(128*SUBS) must be a multiple of WGsPerOutputTile"
        if self.kSplitKCta:
            s = self.kSplitKFactor
            if chunks % s != 0:
                return "SPLIT_K: K/(128*SUBS) must be a multiple of SPLITK_FACTOR"
            if (chunks // s) % self.kWgsPerOutputTile != 0:
                return "SPLIT_K: (K/S)/(128*SUBS) must be a multiple of WGsPerOutputTile"
            if chunks // s < self.kWgsPerOutputTile:
                return "SPLIT_K: not even one k group per warp group"
        err = self._fitted(m, n, k).plan(m, n, k).error
        return err

    def dynamic_smem_bytes(self, m: int, k: int) -> int:
        plan = self._fitted(m, 128, k).plan(m, 128, k)
        return plan.smem_bytes


# ---------------------------------------------------------------------------
# Problem / plan
# ---------------------------------------------------------------------------

@dataclass
class Problem:
    """The reference's ``decode_gemm::Problem`` (kernels/decode_gemm.cuh:352-363).

    Tensor fields take torch tensors or raw device pointers (int).  ``status``
    (a B200 addition) is an optional device int32 the kernel sets on a
    bounded-wait timeout.
    """

    M: int = 0
    N: int = 0
    K: int = 0
    activation: object = None
    weight: object = None
    weight_scales: object = None
    activation_scales: object = None
    output: object = None
    splitk_ws: object = None
    splitk_sem: object = None
    status: object = None

    def to_dg(self) -> DgProblem:
        return DgProblem(self.M, self.N, self.K, _ptr(self.activation), _ptr(self.weight),
                         _ptr(self.weight_scales), _ptr(self.activation_scales), _ptr(self.output),
                         _ptr(self.splitk_ws), _ptr(self.splitk_sem), _ptr(self.status))


@dataclass
class LaunchPlan:
    """The reference's ``LaunchPlan`` (kernels/decode_gemm.cuh:373-380) plus B200 fields."""

    grid: tuple = (0, 0, 0)
    block: tuple = (0, 0, 0)
    smem_bytes: int = 0
    num_output_tiles: int = 0
    padded_n: int = 0
    error: Optional[str] = None
    stages: int = 0
    n_mma: int = 0
    a_rows: int = 0
    mma_m: int = 0
    epi_warps: int = 0
    num_ctas: int = 0
    max_slabs: int = 1
    ws_floats: int = 0
    sem_ints: int = 0
    cluster: int = 1

    @classmethod
    def _from_info(cls, info: DgPlanInfo) -> "LaunchPlan":
        err = info.error.decode() or None
        return cls(grid=(info.grid_x, info.grid_y, info.grid_z), block=(info.block_x, 1, 1),
                   smem_bytes=info.smem_bytes, num_output_tiles=info.num_output_tiles,
                   padded_n=info.padded_n, error=err, stages=info.stages, n_mma=info.n_mma,
                   a_rows=info.a_rows, mma_m=info.mma_m, epi_warps=info.epi_warps, num_ctas=info.num_ctas,
                   max_slabs=info.max_slabs, ws_floats=info.ws_floats, sem_ints=info.sem_ints,
                   cluster=info.cluster)


def _b200(cfg, p: Problem) -> B200Config:
    if isinstance(cfg, KernelConfig):
        return cfg._fitted(p.M, p.N, p.K)
    return cfg


def make_launch_plan(cfg, p: Problem) -> LaunchPlan:
    if isinstance(cfg, KernelConfig):
        ref_err = cfg.validate(p.M, p.N, p.K)
        plan = _b200(cfg, p).plan(p.M, p.N, p.K)
        if ref_err is not None:
            plan.error = ref_err
        # The reference's meanings: BM-row tiles and the packed layout's rows.
        plan.num_output_tiles = cfg.num_output_tiles(p.N)
        plan.padded_n = padded_n(p.N, cfg.OUTPUT_ROWS_PER_CTA)
        return plan
    return cfg.plan(p.M, p.N, p.K)


def make_weight_tma(cfg, p: Problem) -> TensorMap:
    m = TensorMap()
    rc = _lib.lib().dg_make_weight_map(ctypes.byref(_b200(cfg, p).to_dg()), _ptr(p.weight), p.N, p.K, m)
    if rc != 0:
        raise RuntimeError(f"cuTensorMapEncodeTiled(weight) failed: cudaError {rc}")
    return m


def make_activation_tma(cfg, p: Problem) -> TensorMap:
    m = TensorMap()
    rc = _lib.lib().dg_make_activation_map(ctypes.byref(_b200(cfg, p).to_dg()), _ptr(p.activation), p.M,
                                            p.K, m)
    if rc != 0:
        raise RuntimeError(f"cuTensorMapEncodeTiled(activation) failed: cudaError {rc}")
    return m


def launch_with_maps(cfg, p: Problem, w_map: TensorMap, a_map: TensorMap, stream=None,
                     pdl_attr: Optional[bool] = None) -> int:
    """Launch with pre-built maps; returns a cudaError_t value.

    ``pdl_attr`` None follows the configuration's PDL switch (the reference's
    launch_with_maps); True/False sets programmatic stream serialization
    explicitly (the reference harness's direct launch).
    """
    if isinstance(cfg, KernelConfig) and cfg.validate(p.M, p.N, p.K) is not None:
        return CUDA_ERROR_INVALID_VALUE
    b = _b200(cfg, p)
    attr = b.pdl if pdl_attr is None else pdl_attr
    if isinstance(cfg, KernelConfig) and pdl_attr is None:
        attr = cfg.PDL
    return _lib.lib().dg_launch_with_maps(ctypes.byref(b.to_dg()), ctypes.byref(p.to_dg()), w_map, a_map,
                                          _stream_handle(stream), int(bool(attr)))


def launch_quantized(cfg, p: Problem, w_map: TensorMap, a_map: TensorMap, q_out, q_scales, stream=None,
                     pdl_attr: Optional[bool] = None) -> int:
    """``launch_with_maps`` that also writes the next layer's activation:
    e4m3 ``q_out`` [M, N] (uint8) and fp32 ``q_scales`` [M, N/128], the
    block quantisation of this GEMM's bf16 output (bench/bench_decode.cu:459-467)
    -- the bytes ``quantize_activation`` would make from it -- computed in the
    cluster reduction (``dg_launch_quantized``).  Needs the cluster schedule
    and N, block_n multiples of 128.  Returns a cudaError_t value."""
    b = _b200(cfg, p)
    attr = b.pdl if pdl_attr is None else pdl_attr
    if tuple(q_out.shape) != (p.M, p.N) or tuple(q_scales.shape) != (p.M, p.N // 128) or \
            not q_out.is_contiguous() or not q_scales.is_contiguous():
        return CUDA_ERROR_INVALID_VALUE
    return _lib.lib().dg_launch_quantized(ctypes.byref(b.to_dg()), ctypes.byref(p.to_dg()), w_map, a_map,
                                          q_out.data_ptr(), q_scales.data_ptr(), _stream_handle(stream),
                                          int(bool(attr)))


def launch_gather(cfg, p: Problem, gather, w_map: TensorMap, a_map: TensorMap, stream=None,
                  pdl_attr: Optional[bool] = None) -> int:
    """Tensor-parallel launch with the all-gather fused into the kernel
    (``gather`` a ``DgGather``: ``dg_launch_gather``, epoch flags; or a
    ``DgGatherLines``: ``dg_launch_gather_lines``, tagged lines; both from
    ``tp.FusedGather.descriptor``).  Returns a cudaError_t value."""
    b = _b200(cfg, p)
    attr = b.pdl if pdl_attr is None else pdl_attr
    if isinstance(gather, _lib.DgGatherLines):
        return _lib.lib().dg_launch_gather_lines(ctypes.byref(b.to_dg()), ctypes.byref(p.to_dg()),
                                                 ctypes.byref(gather), w_map, a_map, _stream_handle(stream),
                                                 int(bool(attr)))
    return _lib.lib().dg_launch_gather(ctypes.byref(b.to_dg()), ctypes.byref(p.to_dg()), ctypes.byref(gather),
                                       w_map, a_map, _stream_handle(stream), int(bool(attr)))


def quantize_activation(x, out=None, scales=None, stream=None, pdl_attr: bool = False):
    """bf16 [M, K] (row stride >= K) -> (e4m3 [M, K] as uint8, fp32 scales
    [M, K/128]) on the GPU: the reference's block quantisation
    (bench/bench_decode.cu:459-467)."""
    import torch
    m, k = x.shape
    if x.dtype != torch.bfloat16 or x.stride(1) != 1:
        raise ValueError("x must be bf16 with unit column stride")
    if out is None:
        out = torch.empty((m, k), dtype=torch.uint8, device=x.device)
    if scales is None:
        scales = torch.empty((m, k // 128), dtype=torch.float32, device=x.device)
    rc = _lib.lib().dg_quantize_act(x.data_ptr(), x.stride(0), m, k, out.data_ptr(), scales.data_ptr(),
                                    _stream_handle(stream), int(bool(pdl_attr)))
    if rc != 0:
        raise RuntimeError(f"dg_quantize_act failed: cudaError {rc}")
    return out, scales


def host_device_pointer(t) -> int:
    """Device address of a pinned host tensor (``tensor.pin_memory()``), for a
    zero-copy output: a GEMM given it as its output writes the result
    straight into host memory (``dg_host_device_pointer``).  Raises for
    memory that is not mapped pinned memory."""
    if not t.is_pinned():
        raise ValueError("host_device_pointer needs a pinned host tensor")
    out = ctypes.c_void_p()
    rc = _lib.lib().dg_host_device_pointer(ctypes.c_void_p(t.data_ptr()), ctypes.byref(out))
    if rc != 0 or out.value is None:
        raise RuntimeError(f"dg_host_device_pointer failed: cudaError {rc}")
    return int(out.value)


def copy_from_host(dst, src, stream=None, pdl_attr: bool = True, src_device: Optional[int] = None) -> None:
    """dst (device tensor) <- src (pinned host tensor, same number of bytes),
    copied by a kernel that reads the host memory over PCIe
    (``dg_copy_from_host``).  Launched with ``pdl_attr`` it releases the next
    kernel at once and waits for the previous one before writing dst, so a
    stream of "copy request i's input, GEMM request i" stays one request at a
    time while every GEMM's launch and weight prefetch overlap the one before
    it.  ``src_device``: src's device address from :func:`host_device_pointer`,
    looked up once (e.g. before a CUDA graph capture) instead of per call."""
    nbytes = dst.numel() * dst.element_size()
    if src.numel() * src.element_size() != nbytes or not dst.is_cuda or not dst.is_contiguous() \
            or not src.is_contiguous():
        raise ValueError("copy_from_host: contiguous device dst and pinned host src of the same size")
    src_dev = src_device if src_device is not None else host_device_pointer(src)
    rc = _lib.lib().dg_copy_from_host(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src_dev), nbytes,
                                      _stream_handle(stream), int(bool(pdl_attr)))
    if rc != 0:
        raise RuntimeError(f"dg_copy_from_host failed: cudaError {rc}")


def launch(cfg, p: Problem, stream=None) -> int:
    """Encode both tensor maps, then launch (reference ``launch<Cfg>``)."""
    if isinstance(cfg, KernelConfig):
        if cfg.validate(p.M, p.N, p.K) is not None:
            return CUDA_ERROR_INVALID_VALUE
        if cfg.kSplitKCta and (p.splitk_ws is None or p.splitk_sem is None):
            return CUDA_ERROR_INVALID_VALUE
        # Trigger follows PDL or EPI_OVERLAP; the launch attribute follows PDL
        # only (kernels/decode_gemm.cuh:1139-1144).
        return launch_with_maps(cfg, p, make_weight_tma(cfg, p), make_activation_tma(cfg, p), stream,
                                pdl_attr=bool(cfg.PDL))
    return _lib.lib().dg_launch(ctypes.byref(cfg.to_dg()), ctypes.byref(p.to_dg()), _stream_handle(stream))


# ---------------------------------------------------------------------------
# Prepack (kernels/weight_prepack.cuh)
# ---------------------------------------------------------------------------

def padded_n(n: int, output_rows_per_cta: int) -> int:
    return (n + output_rows_per_cta - 1) // output_rows_per_cta * output_rows_per_cta


def packed_weight_bytes(n: int, k: int, output_rows_per_cta: int) -> int:
    return padded_n(n, output_rows_per_cta) * k


def launch_prepack_weight(output_rows_per_cta: int, output_tiles_per_cta: int, source, destination,
                          n: int, k: int, stream=None, layout: int = LAYOUT_PACKED) -> int:
    """``prepack::launch_prepack_weight<BM, TILES>`` (TILES does not change the layout)."""
    if k % K_BLOCK != 0:
        return CUDA_ERROR_INVALID_VALUE
    del output_tiles_per_cta
    return _lib.lib().dg_prepack_weight(_ptr(source), _ptr(destination), n, k, output_rows_per_cta, layout,
                                        _stream_handle(stream))


def prepack_weight(weight, block_n: int, layout: int = LAYOUT_PACKED, stream=None):
    """torch convenience: returns a new uint8 tensor in ``layout``."""
    import torch
    n, k = weight.shape
    out = torch.empty(packed_weight_bytes(n, k, block_n), dtype=torch.uint8, device=weight.device)
    rc = launch_prepack_weight(block_n, 1, weight, out, n, k, stream, layout)
    if rc != 0:
        raise RuntimeError(f"prepack failed: cudaError {rc}")
    return out


def status_string(code: int) -> str:
    return _lib.lib().dg_status_string(code).decode()


def flush_l2(buf, stream=None) -> None:
    rc = _lib.lib().dg_flush_l2(_ptr(buf), buf.numel() * buf.element_size(), _stream_handle(stream))
    if rc != 0:
        raise RuntimeError(f"flush failed: cudaError {rc}")


# ---------------------------------------------------------------------------
# One-call torch entry point
# ---------------------------------------------------------------------------

@dataclass
class _Workspace:
    ws: object = None
    sem: object = None
    status: object = None
    ws_floats: int = 0
    sem_ints: int = 0


_WORKSPACES: dict = {}


def _workspace(device, ws_floats: int, sem_ints: int) -> _Workspace:
    import torch
    key = (device.type, device.index)
    w = _WORKSPACES.get(key)
    if w is None:
        w = _Workspace(status=torch.zeros(1, dtype=torch.int32, device=device))
        _WORKSPACES[key] = w
    if ws_floats > w.ws_floats:
        w.ws = torch.empty(ws_floats, dtype=torch.float32, device=device)
        w.ws_floats = ws_floats
    if sem_ints > w.sem_ints:
        w.sem = torch.zeros(sem_ints, dtype=torch.int32, device=device)
        w.sem_ints = sem_ints
    return w


def fp8_decode_gemm(act, act_scales, weight, weight_scales, out=None, config: Optional[B200Config] = None,
                    n: Optional[int] = None, stream=None):
    """``out[M,N] = act[M,K] . W[N,K]^T`` with per-128 block scales, bf16 out.

    ``act`` and ``weight`` are uint8 (e4m3 bits) or float8_e4m3fn tensors on
    the GPU; ``weight`` is in ``config.layout`` (raw ``[N,K]`` by default, or
    the packed byte buffer with ``n`` given).  The split-K workspace and the
    ticket array are kept per device and reused.
    """
    import torch
    m, k = act.shape
    if n is None:
        n = weight.shape[0]
    if config is None:
        config = default_config(m, n, k)
    plan = config.plan(m, n, k)
    if plan.error is not None:
        raise ValueError(plan.error)
    if out is None:
        out = torch.empty((m, n), dtype=torch.bfloat16, device=act.device)
    w = _workspace(act.device, plan.ws_floats, plan.sem_ints)
    p = Problem(m, n, k, act, weight, weight_scales, act_scales, out, w.ws, w.sem, w.status)
    if stream is None:
        stream = torch.cuda.current_stream(act.device)
    rc = launch(config, p, stream)
    if rc != 0:
        raise RuntimeError(f"decode GEMM launch failed: cudaError {rc}")
    return out
