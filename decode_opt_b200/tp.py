"""N-sharded tensor-parallel decode GEMM over torch.distributed.

The weight matrix W[N, K] is split by rows: rank r of g owns rows
[r*N/g, (r+1)*N/g) together with the matching rows of the 128-row weight
scales, so every GPU streams 1/g of the weights.  The activation and its
scales are replicated.  Each rank computes its [M, N/g] output slice with the
sm_100a kernel, then one NCCL all-gather assembles [M, N] on every rank:
`all_gather_into_tensor` lays the slices out as [g*M, N/g] = [g, M, N/g], and for M > 1 a
permute to [M, g, N/g] gives the row-major [M, N] result (M = 1 needs none).

N/g must be a multiple of 128, so shard boundaries coincide with weight-scale
groups (7168/8 = 896 = 7 x 128).

The reference is single-GPU; this module is the B200 multi-GPU extension the
benchmark uses (`bench.py --gpus N`).
"""

from __future__ import annotations

from typing import Optional, Tuple

SCALE_ROWS = 128


def shard_rows(n: int, world: int, rank: int, align: int = SCALE_ROWS) -> Tuple[int, int]:
    """Row range [start, stop) of W owned by `rank`; shards are equal and
    aligned to `align` rows."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if n % world != 0 or (n // world) % align != 0:
        raise ValueError(f"N={n} does not split into {world} shards of a multiple of {align} rows")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_scales(w_scales, world: int, rank: int, n: int):
    """Rows of the [ceil(N/128), K/128] weight-scale array for the shard."""
    start, stop = shard_rows(n, world, rank)
    return w_scales[start // SCALE_ROWS: stop // SCALE_ROWS]


def assemble(gathered, m: int):
    """[g, M, N/g] all-gather output -> [M, N] (a view for M == 1)."""
    g, mm, n_loc = gathered.shape
    if mm != m:
        raise ValueError("gathered tensor does not match M")
    if m == 1:
        return gathered.reshape(1, g * n_loc)
    return gathered.permute(1, 0, 2).reshape(m, g * n_loc)


def gather_slices(local, group=None, out: Optional[object] = None):
    """All-gather each rank's [M, N/g] slice and return [M, N]."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    m, n_loc = local.shape
    if out is None:
        out = torch.empty((world * m, n_loc), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return assemble(out.view(world, m, n_loc), m)


class TPDecodeGemm:
    """One rank's share of an N-sharded decode GEMM.

    Holds this rank's weight shard (in the configured layout) and its
    scales; `forward(act, act_scales)` computes the local slice with the
    sm_100a kernel and all-gathers the full [M, N] bf16 output.
    """

    def __init__(self, w_shard, w_scales_shard, n_total: int, config=None, group=None):
        import torch
        import torch.distributed as dist
        import decode_opt_b200 as dg
        self.dg = dg
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_total = n_total
        self.n_loc, self.k = w_shard.shape
        if self.n_loc * self.world != n_total:
            raise ValueError("shard rows x world != N")
        self.config = config
        self.w_scales = w_scales_shard
        self.w_raw = w_shard
        self._packed = {}
        self.torch = torch

    def _weight(self, cfg):
        if cfg.layout == self.dg.LAYOUT_RAW:
            return self.w_raw
        key = (cfg.block_n, cfg.layout)
        if key not in self._packed:
            self._packed[key] = self.dg.prepack_weight(self.w_raw, cfg.block_n, cfg.layout)
        return self._packed[key]

    def forward(self, act, act_scales, stream=None):
        m = act.shape[0]
        cfg = self.config or self.dg.default_config(m, self.n_loc, self.k)
        local = self.dg.fp8_decode_gemm(act, act_scales, self._weight(cfg), self.w_scales, config=cfg,
                                        n=self.n_loc, stream=stream)
        return gather_slices(local, self.group)
