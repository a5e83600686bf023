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

The fused alternative (`FusedGather`, `dg_launch_gather`) drops the
collective: each rank's GEMM stores every output element straight into all
ranks' gathered [M, N] buffers over NVLink (peer memory mapped with CUDA IPC)
and its grid completes only when every rank's slices of that launch have
arrived, signalled through per-rank epoch flags with bounded waits
(`dg_launch_gather_lines` instead sends the slices as tagged lines whose
8-byte words carry the launch's epoch beside the data, so the data signals
itself: no flags, no system-scope fences).

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
        key = (cfg.packed_rows, cfg.layout)
        if key not in self._packed:
            self._packed[key] = self.dg.prepack_weight(self.w_raw, cfg.packed_rows, cfg.layout)
        return self._packed[key]

    def forward(self, act, act_scales, stream=None):
        m = act.shape[0]
        cfg = self.config or self.dg.default_config(m, self.n_loc, self.k)
        local = self.dg.fp8_decode_gemm(act, act_scales, self._weight(cfg), self.w_scales, config=cfg,
                                        n=self.n_loc, stream=stream)
        return gather_slices(local, self.group)


def gather_descriptor(world: int, rank: int, n_loc: int, out_bases, flag_ptrs, sync_ptr):
    """The dg_gather for rank `rank`: out_bases[q] is rank q's gathered
    [M, world*n_loc] bf16 buffer as mapped in this process, flag_ptrs[q] its
    int[world] flag array; this rank writes columns [rank*n_loc,
    (rank+1)*n_loc) of every buffer."""
    from ._lib import DgGather, MAX_RANKS
    if not 1 <= world <= MAX_RANKS or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    g = DgGather()
    g.world = world
    g.rank = rank
    g.ldo = world * n_loc
    for q in range(world):
        g.outputs[q] = int(out_bases[q]) + 2 * rank * n_loc
        g.flags[q] = int(flag_ptrs[q])
    g.sync = int(sync_ptr)
    return g


def lines_descriptor(world: int, rank: int, n_loc: int, output, line_bases, sync_ptr, q_out=0, q_scales=0):
    """The dg_gather_lines for rank `rank`: `output` is this rank's gathered
    [M, world*n_loc] bf16 buffer, line_bases[q] rank q's line buffer of the
    launch's set as mapped in this process; q_out / q_scales (optional) the
    e4m3 [M, world*n_loc] and fp32 [M, world*n_loc/128] quantisation of the
    gathered output the unpack also writes."""
    from ._lib import DgGatherLines, MAX_RANKS
    if not 1 <= world <= MAX_RANKS or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    g = DgGatherLines()
    g.world = world
    g.rank = rank
    g.ldo = world * n_loc
    g.output = int(output)
    for q in range(world):
        g.lines[q] = int(line_bases[q])
    g.sync = int(sync_ptr)
    g.q_out = int(q_out)
    g.q_scales = int(q_scales)
    return g


def serving_schedule(base: int, count: int, group: int):
    """The operations of the N-GPU serving loop for requests base .. base+count-1,
    in issue order, as (kind, j, waits).

    kind: "h2d" (request j's inputs host -> input slot j % (2*group), copy
    stream A), "gemm" (the fused GEMM + gather of request j into gathered set
    j % (2*group), the compute stream) or "d2h" (set j % (2*group) -> host,
    copy stream B).  waits: (kind, index) operations of OTHER streams this one
    must follow; each stream also runs its own operations in order, and waits
    never reach before `base` (a CUDA graph of one chunk starts after the
    previous chunk's graph has completed).

    Requests go in groups of `group`: the group's H2D copies are issued first,
    then its GEMMs, each followed by its D2H copy.  Only the group's first GEMM
    waits on a copy stream -- for its group's last H2D copy and for the D2H
    copy of the previous group's first request -- so the other GEMMs of the
    group keep their programmatic (PDL) edge to the GEMM before them.  H2D j
    waits for GEMM j - 2*group (the previous reader of its slot).  With that,
    D2H j - 2*group (the previous reader of set j % (2*group)) finishes before
    this rank's GEMM j - 1, after which a peer's GEMM j may store into the set.
    """
    if group < 1 or count < 0:
        raise ValueError("group must be >= 1 and count >= 0")
    nset = 2 * group
    ops = []
    end = base + count
    for g0 in range(base, end, group):
        g1 = min(end, g0 + group)
        for j in range(g0, g1):
            ops.append(("h2d", j, [("gemm", j - nset)] if j - nset >= base else []))
        for j in range(g0, g1):
            waits = []
            if j == g0:
                waits.append(("h2d", g1 - 1))
                if g0 - group >= base:
                    waits.append(("d2h", g0 - group))
            ops.append(("gemm", j, waits))
            ops.append(("d2h", j, [("gemm", j)]))
    return ops


class FusedGather:
    """Gathered output buffers of a tensor-parallel group for the fused-gather
    launch.

    Every rank allocates `buffers` gathered [m_max, world*n_loc] bf16 buffers
    (slices of one allocation, so a peer opens one IPC mapping for all of
    them), one int[world] flag array and an int[2] launch counter, exports
    CUDA IPC handles for the buffers and flags, exchanges them with
    `all_gather_object` over `group`, and maps every other rank's.
    `descriptor(i)` is the dg_gather of buffer set i: alternate i between
    consecutive launches (a rank must never overwrite slices a peer has not
    consumed yet).  Every rank must make the same launches in the same order.

    ``protocol="lines"`` (dg_launch_gather_lines): peers store tagged 16-byte
    lines {2 bf16, epoch, 2 bf16, epoch} into `buffers` line buffers of
    m_max x world*n_loc/4 lines on every rank (exported and mapped instead of
    the gathered buffers and flags); each rank's kernel unpacks its own into
    its local gathered buffers.  `descriptor(i)` is then a dg_gather_lines.
    """

    def __init__(self, m_max: int, n_loc: int, group=None, buffers: int = 2, device=None,
                 protocol: str = "flags"):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _lib
        self._lib = _lib.lib()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n_loc = n_loc
        self.m_max = m_max
        if protocol not in ("flags", "lines"):
            raise ValueError("protocol must be 'flags' or 'lines'")
        if protocol == "lines" and n_loc % 4 != 0:
            raise ValueError("the lines protocol needs n_loc % 4 == 0")
        self.protocol = protocol
        dev = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.storage = torch.zeros((buffers, m_max, self.world * n_loc), dtype=torch.bfloat16, device=dev)
        self.buffers = [self.storage[i] for i in range(buffers)]
        self.flags = torch.zeros(self.world, dtype=torch.int32, device=dev)
        self.sync = torch.zeros(2, dtype=torch.int32, device=dev)
        if protocol == "lines":
            # 16-byte lines: two int64 words {payload, epoch} per 4 columns
            self.line_storage = torch.zeros((buffers, m_max, self.world * n_loc // 4, 2), dtype=torch.int64,
                                            device=dev)
        torch.cuda.synchronize(dev)

        def export(t):
            h = _lib.IpcHandle()
            off = ctypes.c_ulonglong()
            rc = self._lib.dg_ipc_export(t.data_ptr(), h, ctypes.byref(off))
            if rc != 0:
                raise RuntimeError(f"dg_ipc_export failed: cudaError {rc}")
            return bytes(h), off.value

        self._imported = []
        if protocol == "lines":
            sets = [self.line_storage[i] for i in range(buffers)]
            everyone = [None] * self.world
            dist.all_gather_object(everyone, [export(t) for t in sets], group=group)
            self.peer_lines = [[sets[i].data_ptr() if q == self.rank else self._import(*everyone[q][i])
                                for q in range(self.world)] for i in range(buffers)]
            return
        mine = [export(b) for b in self.buffers] + [export(self.flags)]
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self.peer_bufs = []    # [set][rank] base pointers in this process
        self.peer_flags = []
        for i in range(buffers):
            row = []
            for q in range(self.world):
                row.append(self.buffers[i].data_ptr() if q == self.rank else self._import(*everyone[q][i]))
            self.peer_bufs.append(row)
        self.peer_flags = [self.flags.data_ptr() if q == self.rank else self._import(*everyone[q][buffers])
                           for q in range(self.world)]

    def _import(self, handle: bytes, offset: int) -> int:
        import ctypes
        from . import _lib
        h = _lib.IpcHandle.from_buffer_copy(handle)
        ptr = ctypes.c_void_p()
        rc = self._lib.dg_ipc_import(h, offset, ctypes.byref(ptr))
        if rc != 0:
            raise RuntimeError(f"dg_ipc_import failed: cudaError {rc}")
        self._imported.append(ptr.value)
        return ptr.value

    def descriptor(self, i: int, q_out=None, q_scales=None):
        """The launch descriptor of buffer set i.  Lines protocol only:
        q_out (uint8 [M, world*n_loc]) and q_scales (fp32 [M, world*n_loc/128])
        make the launch also write the gathered output's e4m3 block
        quantisation (the next layer's activation)."""
        if self.protocol == "lines":
            return lines_descriptor(self.world, self.rank, self.n_loc, self.buffers[i].data_ptr(),
                                    self.peer_lines[i], self.sync.data_ptr(),
                                    q_out.data_ptr() if q_out is not None else 0,
                                    q_scales.data_ptr() if q_scales is not None else 0)
        if q_out is not None or q_scales is not None:
            raise ValueError("a quantised gather needs protocol='lines'")
        return gather_descriptor(self.world, self.rank, self.n_loc, self.peer_bufs[i], self.peer_flags,
                                 self.sync.data_ptr())

    def wait(self, i: int, stream=None, status=None, timeout_ns: int = 0) -> None:
        """Enqueue the completion wait for the last fused launch (buffer set i
        is then complete on this rank).  Under the lines protocol a completed
        launch has already unpacked the whole set: nothing to enqueue."""
        import ctypes
        import torch
        if self.protocol == "lines":
            return
        d = self.descriptor(i)
        s = (stream if stream is not None else torch.cuda.current_stream()).cuda_stream
        rc = self._lib.dg_gather_wait(ctypes.byref(d), status.data_ptr() if status is not None else None,
                                      timeout_ns, s)
        if rc != 0:
            raise RuntimeError(f"dg_gather_wait failed: cudaError {rc}")

    def output(self, i: int, m: int):
        """This rank's gathered [m, world*n_loc] result of buffer set i."""
        return self.buffers[i][:m]

    def close(self):
        for ptr in self._imported:
            self._lib.dg_ipc_release(ptr)
        self._imported = []
