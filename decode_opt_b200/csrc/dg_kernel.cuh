// SPDX-License-Identifier: MIT
//
// dg_kernel.cuh -- the B200 (sm_100a) FP8 decode GEMM kernel.
//
//   out[M,N] (bf16) = act[M,K] (e4m3) . W[N,K]^T (e4m3), with per-128-K block
//   scales w_scales[ceil(N/128), K/128] and a_scales[M, K/128]:
//     out[m][n] = bf16( sum_kb  (w_s[n/128][kb] * a_s[m][kb]) * raw_kb[m][n] )
//   where raw_kb is the exact fp8 dot product over one 128-wide K block.
//
// This is the hot path the reference implements as fp8_decode_gemm<Cfg>
// (kernels/decode_gemm.cuh:574-1081).  It is a new design for Blackwell.
//
// Operand placement.  A tcgen05.mma takes the same ~161 cycles whatever its
// M and N (measured on B200 for kind::f8f6f4, M in {64,128}, N in 16..256), so
// the weights -- the only large operand -- go on the MMA's N side with up to
// N = 256 rows per instruction: 8 KiB of weights per MMA, twice what an
// M=128 weight tile could carry.  The decode batch (M = 1..128 rows) is the
// MMA's M side, padded to 64 or 128; rows past M are never read back.  One
// MMA covers K = 32; four cover one 128-wide scale block, which accumulates
// into its own TMEM buffer (the first of the four does not accumulate), so
// the per-block dequantisation stays exact:
//     partial[m][n] = fmaf(w_s * a_s[m], raw_kb[m][n], partial[m][n])   (fp32)
// the reference's numerical path (kernels/decode_gemm.cuh:897-946).
//
// Warp roles (one CTA per SM):
//   warps 0 .. 4E-1   epilogue.  Warp w reads TMEM lane quarter w % 4, i.e.
//                     the batch rows of that quarter, and column group w / 4
//                     (64 or 128 weight rows) of the tile: tcgen05.ld, scale
//                     fold into fp32 partials held in registers (packed
//                     fma.rn.f32x2), then bf16 store or the split reduction.
//                     Warps whose rows are all >= M, or whose columns are past
//                     the tile, stay idle.
//   warp 4E           TMA producer: weight and activation tiles of one
//                     (tile, chunk) unit per pipeline stage, `stages` deep.
//   warp 4E+1         MMA issuer and TMEM owner: one lane issues the MMAs;
//                     tcgen05.commit frees smem stages and publishes finished
//                     accumulators.
//   warps 4E+2, 4E+3  only when each epilogue warp folds 128 columns: idle
//                     warps that complete the control warpgroup, which then
//                     hands registers to the epilogue warpgroups (setmaxnreg).
//
// Work decomposition (stream-K).  The (tile, chunk) units, chunk = `subs`
// consecutive 128-K blocks, are numbered tile-major; CTA c of G processes the
// contiguous range [floor(c*U/G), floor((c+1)*U/G)).  A tile whose units all
// fall in one CTA is written directly in bf16.  Otherwise each contributing
// CTA stores its fp32 partial into workspace slab (c - first contributor) and
// counts itself in the tile's state word.  When a CTA has finished its range
// it reduces chunks of its split tiles -- each element summed over the slabs
// in slab order 0,1,2,..., a fixed order, so results are run-to-run
// bit-identical -- and stores bf16: every contributor helps when the whole
// grid is resident at once (kFlagCoopReduce), else the last arriver alone;
// the finisher of the last chunk re-zeroes the word.  The reference's S-way CTA split-K
// (gridDim.y = S, kernels/decode_gemm.cuh:1015-1077) is the special case
// G = tiles*S, where every range is one S-th of one tile.
//
// Cluster split-K (kFlagCluster).  The grid is (tiles, S) as in the
// reference's split-K, and the S CTAs of a tile form one thread-block cluster
// (cluster dims (1, S, 1)), so CTA s owns K range [s*C/S, (s+1)*C/S) of its
// tile.  Each CTA writes its fp32 partial [M][BN] into its own shared memory
// (the drained ring; float4 columns XOR-swizzled by row so that the rows of a
// warp hit distinct banks); after one cluster barrier, cluster rank r sums
// the r-th S-th of the tile's elements over the S partials, read through
// distributed shared memory in rank order 0..S-1 (run-to-run bit-identical),
// and stores bf16; a second cluster barrier keeps every CTA's partial alive
// until all its readers are done.  No workspace, semaphore or global atomic:
// the reduction never waits on L2, whose round trips take 1-2 us while the
// GPU streams weights at full bandwidth.
//
// Programmatic dependent launch.  Weight tiles for the first ring pass are
// requested before griddepcontrol.wait (weights are never written by a
// preceding kernel); activation loads, scale reads and every global write
// come after it -- unless kFlagIndependentInputs declares that the inputs are
// not produced by the preceding grid, in which case only the writes wait.  The
// producer issues griddepcontrol.launch_dependents right after its first ring
// pass when kFlagPdlTrigger is set -- earlier than the reference, which
// triggers after its last TMA (kernels/decode_gemm.cuh:708-713): measured back
// to back, a late trigger left each SM idle ~3.6 us between this grid's CTA
// exiting and the next grid's CTA starting there.
//
// Failure behaviour.  Every wait is bounded (sm100::mbar_wait_bounded).  On a
// timeout the CTA records an error code in *status, raises a CTA-wide abort
// flag, stops issuing work, waits (bounded) for its own TMA copies and MMAs
// still in flight, frees its TMEM and exits.  No trap, no unbounded spin.

#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100.cuh"

namespace dg {

constexpr int kKBlock = 128;                       // one scale group of K
constexpr uint32_t kMaxDynamicSmem = 227u * 1024u; // per CTA on sm_100
constexpr int kMaxStages = 16;
constexpr int kMaxAccumBuffers = 8;
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s
constexpr int kMaxOutputs = 8;                     // output copies: one per tensor-parallel rank

enum Layout : int {
  kLayoutRaw = 0,             // W[N,K], K contiguous
  kLayoutPacked = 1,          // [tile][kb][BN rows][128 B] (reference prepack)
  kLayoutPackedSwizzled = 2,  // same order, bytes pre-swizzled for SWIZZLE_128B
};

enum Flags : int {
  kFlagPdlTrigger = 1,     // producer issues griddepcontrol.launch_dependents
  kFlagInjectTimeout = 2,  // test hook: CTA 0's MMA warp waits on a barrier nobody arrives on
  // The activation and both scale arrays are not written by the preceding
  // grid of the stream (e.g. back-to-back GEMMs on one activation): they may
  // be read before griddepcontrol.wait.  Global writes still wait.
  kFlagIndependentInputs = 4,
  // Set by the planner when the whole grid can be resident at once: every
  // contributor of a split tile helps reduce it (bounded wait for the others).
  kFlagCoopReduce = 8,
  // Cluster split-K (set by the planner): grid (tiles, S) with cluster
  // (1, S, 1); the S CTAs of a tile reduce through distributed shared memory
  // instead of the workspace.
  kFlagCluster = 16,
  // Host planning only: take the batch class from m_tile instead of M.
  kFlagClassFromMTile = 32,
  // Cluster split-K only (set by dg_launch_quantized): the reduction also
  // writes the e4m3 block quantisation of the bf16 output (q_out, q_scales).
  kFlagQuantizeOut = 64,
  // Cluster split-K only (set by dg_launch_gather_lines): the fused gather
  // stores every output element as tagged lines into every rank's line buffer
  // and each CTA unpacks a slice of this rank's buffer once it is whole (no
  // flags, no system-scope fences).
  kFlagGatherLines = 128,
  // With kFlagGatherLines (q_out / q_scales set): the unpack also writes the
  // e4m3 block quantisation of the gathered output, one warp per 128-column
  // block.
  kFlagGatherLinesQuant = 256,
  // Host planning only: the swap-AB batch class (SwapTraits; M <= 16,
  // block_n 256, cluster split-K schedule).
  kFlagSwapAB = 512,
};

constexpr int kMaxClusterSplit = 16;   // CTAs per cluster (above 8: non-portable size)

// State word of a split tile (one int per tile, zero between launches):
//   bits  0..9   contributors that have stored their slab (arrivals)
//   bits 10..20  reduction chunks claimed
//   bits 21..31  reduction chunks finished
// The CTA that finishes the last chunk stores zero.
constexpr int kArrivalMask = 0x3ff;
constexpr int kMaxContributors = kArrivalMask;   // 1023 CTAs per tile at most
constexpr int kClaimShift = 10;
constexpr int kDoneShift = 21;
constexpr int kCountMask = 0x7ff;
// How long a contributor that has finished its own work waits for the other
// contributors of its split tiles before leaving their reduction to the last
// arriver (no error: the last arriver reduces every chunk nobody claimed).
constexpr uint64_t kHelpWaitNs = 20000ull;

enum Status : int {
  kStatusOk = 0,
  kErrProducerEmptyWait = 0x11,
  kErrMmaFullWait = 0x21,
  kErrMmaAccumWait = 0x22,
  kErrEpilogueAccumWait = 0x31,
  kErrDrainTma = 0x41,
  kErrDrainMma = 0x42,
  kErrInjectedTimeout = 0x51,
  kErrBadLaunchShape = 0x61,
  kErrReduceWait = 0x71,      // split reduction: a workspace bulk copy did not land in time
  kErrGatherWait = 0x81,      // fused gather: a peer's slices did not arrive in time
};

// Everything the kernel needs, computed on the host (dg_host.cuh) and passed
// by value as a __grid_constant__ parameter.
struct KernelParams {
  int M, N, K;
  int block_n;          // BN: weight rows (output columns) per tile
  int pack_tiles;       // kLayoutPacked: packed tiles of pack_rows rows one CTA tile spans (1: pack_rows = BN)
  int pack_rows;        // kLayoutPacked: rows per tile of the packed layout (BN / pack_tiles)
  int n_mma;            // MMA N: BN rounded up to 16
  int a_rows;           // activation rows per TMA box: M rounded up to 8
  int subs;             // 128-K blocks per pipeline stage
  int stages;           // smem ring depth
  int layout;           // Layout
  int num_tiles;        // ceil(N / BN)
  int chunks_per_tile;  // (K/128) / subs
  int num_kb;           // K/128
  int num_ctas;         // G
  int flags;
  long long total_units;     // num_tiles * chunks_per_tile
  uint32_t w_stage_bytes;    // subs * BN * 128
  uint32_t a_stage_bytes;    // subs * MMA_M * 128 (smem per stage)
  uint32_t a_tx_bytes;       // subs * copies * a_rows * 128 (bytes TMA delivers)
  uint32_t w_region_bytes;   // stages * w_stage_bytes + pad, 1 KiB aligned
  uint32_t a_region_bytes;   // stages * a_stage_bytes + pad, 1 KiB aligned
  uint32_t smem_bytes;       // total dynamic smem incl. 1 KiB alignment slack
  unsigned long long timeout_ns;
  __nv_bfloat16* output;     // [M, ldo], this GEMM's N columns (= outs[0])
  int ldo;                   // output row stride in elements (N unless gathering)
  int n_outs;                // destinations of every output element: 1, or the TP world size
  __nv_bfloat16* outs[kMaxOutputs];  // outs[0] = output; outs[r] another rank's gathered buffer
  int world, rank;           // tensor-parallel group of the fused gather (world 1: none)
  int* peer_flags[kMaxOutputs];      // rank r's flag array (one int per writer rank)
  int* my_flags;             // this rank's flag array
  int* sync_ctr;             // [2]: CTAs finished in this launch, launches completed (epoch)
  const float* w_scales;     // [ceil(N/128), K/128]
  const float* a_scales;     // [M, K/128]
  float* ws;                 // [slabs][M][N] fp32 (split tiles only)
  int* sem;                  // [num_tiles] tickets, zero between launches
  int* status;               // first error code, may be null
  const uint8_t* weight;     // kLayoutPackedSwizzled: bulk-copy source
  uint8_t* q_out;            // kFlagQuantizeOut: e4m3 [M, N] of the bf16 output
  float* q_scales;           // kFlagQuantizeOut: fp32 [M, N/128]
  uint4* lines[kMaxOutputs]; // kFlagGatherLines: rank r's line buffer of this launch's set, [M][lines_per_row]
  int lines_per_row;         // kFlagGatherLines: world * N / 4 (4 output columns per 16-byte line)
};

// Epilogue geometry shared with the host planner: weight columns one
// epilogue warp folds, control warps, threads per CTA.
__host__ __device__ constexpr int cols_per_warp(int copies, int epw) { return 256 / (copies * epw); }
// 128 fp32 partials per thread need more registers than an even split of the
// register file gives, so the control warps then fill a whole warpgroup that
// hands registers to the epilogue warpgroups (setmaxnreg).
__host__ __device__ constexpr bool uses_reg_realloc(int copies, int epw) { return cols_per_warp(copies, epw) > 64; }
__host__ __device__ constexpr int ctrl_warps(int copies, int epw) { return uses_reg_realloc(copies, epw) ? 4 : 2; }
__host__ __device__ constexpr int block_threads(int copies, int epw) {
  return (4 * epw + ctrl_warps(copies, epw)) * 32;
}
constexpr uint32_t kCtrlRegs = 40;    // per thread, control warpgroup after setmaxnreg.dec
constexpr uint32_t kEpiRegs = 232;    // per thread, epilogue warpgroups after setmaxnreg.inc

// Compile-time geometry of one kernel instantiation: the MMA M (batch rows,
// padded), the number of batch copies along it and the number of epilogue
// warps per TMEM lane quarter.
//
// Batch replication.  TMEM lane quarter q holds accumulator rows
// [q*R4, (q+1)*R4), R4 = MMA_M/4.  A batch that fills fewer quarters than
// there are is replicated: the activation tile is loaded kCopies times, into
// row blocks of MMA_M/kCopies rows, so the quarters of copy c hold the whole
// batch and fold only the weight columns [c*256/kCopies, (c+1)*256/kCopies).
// The MMA costs the same (its M is padded anyway); the epilogue's TMEM reads
// and FMAs are spread over all four quarters instead of landing on the
// quarters that hold the real rows.
template <int MMA_M_, int COPIES_, int EPW_>
struct KernelTraits {
  static constexpr int kMmaM = MMA_M_;
  static constexpr int kCopies = COPIES_;            // batch copies along the MMA M side
  static constexpr int kEpw = EPW_;                  // epilogue warps per lane quarter
  static_assert(kMmaM == 64 || kMmaM == 128, "tcgen05 cta_group::1 M is 64 or 128");
  static_assert(kCopies == 1 || kCopies == 2 || kCopies == 4, "1, 2 or 4 batch copies");
  static_assert(kEpw == 1 || kEpw == 2 || kEpw == 4, "1, 2 or 4 epilogue warps per quarter");
  static constexpr int kBnMax = 256;                 // accumulator columns per buffer
  static constexpr int kQuartersPerCopy = 4 / kCopies;
  static constexpr int kColsPerCopy = kBnMax / kCopies;
  static constexpr int kColsPerWarp = cols_per_warp(kCopies, kEpw);
  static_assert(kColsPerWarp == 64 || kColsPerWarp == 128, "64 or 128 columns per epilogue warp");
  static constexpr int kRowsPerQuarter = kMmaM / 4;  // accumulator rows per lane quarter
  static constexpr int kRowsPerCopy = kMmaM / kCopies;
  static constexpr int kEpiWarps = 4 * kEpw;
  static constexpr int kEpiThreads = kEpiWarps * 32;
  static constexpr bool kRegRealloc = uses_reg_realloc(kCopies, kEpw);
  static constexpr int kProducerWarp = kEpiWarps;
  static constexpr int kMmaWarp = kEpiWarps + 1;
  static constexpr int kThreads = block_threads(kCopies, kEpw);
  static constexpr int kLdBatch = 4;                 // 16-column TMEM loads per wait
  static constexpr int kRedGroups = 2;               // plain-path reduction units in flight per thread
  // Cluster reduction units a thread may hold in registers while its grid
  // still waits on the preceding one (the deferred reduction of
  // cluster_sum_units).  Four covers M <= 32 in every class (a thread folds
  // kColsPerWarp columns of one row, so S >= 2 ranks leave it at most
  // kColsPerWarp / 8 units: 4 at M <= 32); measured with independent inputs
  // at C2, deferring took M = 32 from 21.8 to 19.3-20.2 us, left M <= 16
  // and M = 64 unchanged within noise and took M = 128 from 23.9 to 28.3 us,
  // so larger shares keep the wait-first order.
  static constexpr int kDeferUnits = 4;
  static constexpr int kNumBufs = 2;                 // 2 x 256 columns = all of TMEM
  static constexpr uint32_t kTmemCols = 512u;
  static constexpr bool kSwap = false;
  static constexpr int kActRows = kMmaM;             // activation rows per 128-K block in smem
  static constexpr int kMmaIssuers = 1;
  static_assert(kColsPerCopy == kEpw * kColsPerWarp, "column split");
  static_assert((kColsPerWarp / 16) % kLdBatch == 0, "whole load batches");
  static_assert(!kRegRealloc || (kEpiWarps % 4 == 0 && kThreads == (kEpiWarps + 4) * 32),
                "register reallocation needs whole warpgroups");
};

// Swap-AB batch class (M <= 16): the weights are the MMA's M side and the
// batch its N side, tcgen05.mma M = 128 weight rows x N = 16 batch rows x
// K = 32, so an instruction multiplies 4 KiB of weights by the batch padded to
// 16 instead of padding the batch to 64 rows: a quarter of the multiply-adds
// per weight byte of the M = 64 class, and with them the tensor pipe's power
// draw.  A tile of block_n = 136..256 rows is covered by two 128-row halves,
// rows [0, 128) and [128, 256): below 256 rows the second half also reads
// the 256 - block_n rows after the tile (the next block of the ring, or its
// tail pad), whose accumulator lanes are never folded; two MMA warps issue one half each into their
// own 16 accumulator columns (one issuing thread needs ~72 cycles per MMA,
// two bring the pair to ~39 each, so a 128-K block takes ~4 x 78 cycles
// against 448 for the M = 64 x N = 224 class).  TMEM lane = row within a
// half, column = batch row: epilogue warp q folds lanes 32q..32q+31 of both
// halves (of half 1 only the rows inside the tile), 2 x 16 values per thread,
// and writes them transposed into the same
// [M][block_n] shared-memory partial the cluster reduction of the other
// classes reads.
struct SwapTraits {
  static constexpr bool kSwap = true;
  static constexpr int kMmaM = 128;                  // weight rows per MMA (one tile half)
  static constexpr int kMmaN = 16;                   // batch rows per MMA, padded
  static constexpr int kActRows = kMmaN;             // activation rows per 128-K block in smem
  static constexpr int kCopies = 1;
  static constexpr int kRowsPerCopy = kMmaN;
  static constexpr int kEpw = 1;
  static constexpr int kEpiWarps = 4;
  static constexpr int kEpiThreads = kEpiWarps * 32;
  static constexpr bool kRegRealloc = false;
  static constexpr int kProducerWarp = kEpiWarps;
  static constexpr int kMmaWarp = kEpiWarps + 1;     // issues tile rows 0..127
  static constexpr int kMmaIssuers = 2;              // warp kMmaWarp + 1 issues rows 128..255
  static constexpr int kThreads = (kEpiWarps + 2 + 1) * 32;
  static constexpr int kBnMax = 2 * kMmaN;           // accumulator columns per buffer
  // Four 32-column buffers: the MMA warps run up to three 128-K blocks ahead
  // of the epilogue's fold (MMA issue is on the critical path).
  static constexpr int kNumBufs = 4;
  static constexpr uint32_t kTmemCols = 128u;
  static constexpr int kDeferUnits = 4;              // as the other classes (M <= 16: <= 4 units)
};

// Where epilogue warp w works: lane quarter, batch rows, weight columns.
template <class Tr>
struct EpiWarp {
  int quarter;   // TMEM lane quarter (w % 4)
  int row0;      // first batch row of this quarter within its copy
  int col0;      // first tile column folded by this warp
  bool active;   // holds a batch row < M and a column < block_n
  __host__ __device__ __forceinline__ EpiWarp(int w, int M, int block_n) {
    quarter = w & 3;
    const int group = w >> 2;
    const int copy = quarter / Tr::kQuartersPerCopy;
    row0 = (quarter % Tr::kQuartersPerCopy) * Tr::kRowsPerQuarter;
    col0 = copy * Tr::kColsPerCopy + group * Tr::kColsPerWarp;
    active = (row0 < M) && (col0 < block_n);
  }
};

template <class Tr>
__host__ __device__ __forceinline__ int active_epilogue_warps(int M, int block_n) {
  if constexpr (Tr::kSwap) {
    return Tr::kEpiWarps;   // every lane quarter holds tile rows
  } else {
    int n = 0;
    for (int w = 0; w < Tr::kEpiWarps; ++w) n += EpiWarp<Tr>(w, M, block_n).active ? 1 : 0;
    return n;
  }
}

// Rank of warp w among the active epilogue warps.
template <class Tr>
__device__ __forceinline__ int active_epilogue_rank(int w, int M, int block_n) {
  if constexpr (Tr::kSwap) {
    return w;
  } else {
    int n = 0;
    for (int v = 0; v < w; ++v) n += EpiWarp<Tr>(v, M, block_n).active ? 1 : 0;
    return n;
  }
}

// mbarriers (ring full/empty, accumulator full/empty, drain, test hook, two
// for the split reduction), then the TMEM address slot, the CTA abort flag,
// the two-int mailbox of the split reduction and the "stored output" flag.
struct SmemBarriers {
  static __host__ __device__ constexpr uint32_t bytes(int stages, int bufs) {
    return static_cast<uint32_t>((2 * stages + 2 * bufs + 4) * 8 + 32);
  }
};

// Row stride, in floats, of a CTA's fp32 partial [M][BN] in shared memory
// under cluster split-K: BN rounded up to 32, so that float4 column c4 of row
// m, stored at c4 ^ (m & 7), stays inside its row for every BN (a multiple
// of 8).
__host__ __device__ constexpr int cluster_partial_stride(int block_n) { return (block_n + 31) & ~31; }

__host__ __device__ __forceinline__ long long cta_of_unit(long long u, long long G, long long U) {
  // CTA c owns [floor(c*U/G), floor((c+1)*U/G)); this inverts it.
  return ((u + 1) * G - 1) / U;
}

// Bounded wait that ignores the abort flag: used while draining after an
// abort, when the copies or MMAs being waited for complete on their own.
__device__ __forceinline__ bool wait_for_completion(uint64_t* bar, uint32_t parity,
                                                    uint64_t timeout_ns) {
  if (sm100::mbar_try_wait(bar, parity)) return true;
  const uint64_t start = sm100::global_timer_ns();
  while (!sm100::mbar_try_wait(bar, parity)) {
    if (sm100::global_timer_ns() - start > timeout_ns) return false;
  }
  return true;
}

// Stores `ncols` fp32 partials of one output row as bf16 (16-byte stores when
// the row start is 16-byte aligned and the run is full), else element-wise.
template <int COLS>
__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const float (&v)[COLS], int ncols,
                                               bool aligned) {
  if (aligned && ncols == COLS) {
#pragma unroll
    for (int j = 0; j < COLS; j += 8) {
      uint4 pk;
      __nv_bfloat162 h0 = __floats2bfloat162_rn(v[j], v[j + 1]);
      __nv_bfloat162 h1 = __floats2bfloat162_rn(v[j + 2], v[j + 3]);
      __nv_bfloat162 h2 = __floats2bfloat162_rn(v[j + 4], v[j + 5]);
      __nv_bfloat162 h3 = __floats2bfloat162_rn(v[j + 6], v[j + 7]);
      pk.x = *reinterpret_cast<uint32_t*>(&h0);
      pk.y = *reinterpret_cast<uint32_t*>(&h1);
      pk.z = *reinterpret_cast<uint32_t*>(&h2);
      pk.w = *reinterpret_cast<uint32_t*>(&h3);
      *reinterpret_cast<uint4*>(dst + j) = pk;
    }
  } else {
#pragma unroll
    for (int j = 0; j < COLS; ++j)
      if (j < ncols) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

// Stores `ncols` (a multiple of 4) fp32 partials of row m < M8 of a blocked
// workspace slab (layout: see ws_blocked_offset): 16 bytes per 4 columns.
__device__ __forceinline__ size_t ws_blocked_offset(int m, int n, int N);
template <int COLS>
__device__ __forceinline__ void store_row_f32_blocked(float* slab, int m, int n0, int N, const float (&v)[COLS],
                                                      int ncols) {
#pragma unroll
  for (int j = 0; j < COLS; j += 4)
    if (j < ncols)
      __stcg(reinterpret_cast<float4*>(slab + ws_blocked_offset(m, n0 + j, N)),
             make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
}

// Stores `ncols` fp32 partials of one row to the split workspace (L2 only).
template <int COLS>
__device__ __forceinline__ void store_row_f32(float* dst, const float (&v)[COLS], int ncols, bool aligned) {
  if (aligned && ncols == COLS) {
#pragma unroll
    for (int j = 0; j < COLS; j += 4)
      __stcg(reinterpret_cast<float4*>(dst + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
  } else {
#pragma unroll
    for (int j = 0; j < COLS; ++j)
      if (j < ncols) __stcg(dst + j, v[j]);
  }
}

// ------------------------------------------------------ split workspace ----
// Slab layout (M x N floats per slab, the reference's workspace size).  When
// N % 4 == 0 and the workspace is 16-byte aligned ("blocked"), rows
// [0, M8), M8 = M rounded down to a multiple of 8, are stored as
// [M8/8][N/4][8][4]: the 8 rows x 4 columns of one (row block, column group)
// are 128 contiguous bytes -- the 8 lanes of a warp that hold one row block
// store one full line per float4 store, and one row block of one tile is
// bn*32 contiguous bytes for a single bulk copy.  Rows [M8, M), and every row
// when not blocked, are row-major.
__device__ __forceinline__ size_t ws_blocked_offset(int m, int n, int N) {   // m < M8, n % 4 == 0
  return ((static_cast<size_t>(m >> 3) * static_cast<size_t>(N >> 2) + static_cast<size_t>(n >> 2)) * 8u +
          static_cast<size_t>(m & 7)) * 4u;
}

// The reduction of one split tile walks "row blocks": 8-row blocks of the
// blocked rows, then single rows.  Chunks are contiguous runs of row blocks:
// one per contributor at most, and at least 32 KiB of slab data each (a
// smaller chunk costs more in claim round trips than it saves).  Every CTA
// computes the same count.
struct SplitGeometry {
  int M;
  int m8;         // rows in 8-row blocks
  int nb;         // row blocks of a tile
  __device__ __forceinline__ SplitGeometry(int M_, bool blocked) : M(M_) {
    m8 = blocked ? (M & ~7) : 0;
    nb = m8 / 8 + (M - m8);
  }
  __device__ __forceinline__ int chunks(int contributors, int bn_t) const {
    const long long bytes = static_cast<long long>(contributors) * M * bn_t * 4;
    const int by_size = static_cast<int>(bytes / 32768);
    return max(1, min(min(contributors, nb), by_size));
  }
};

// Sums slabs 0, 1, ..., n_c-1 -- in that order, whoever runs it, so results
// are bit-identical run to run -- of row blocks [b0, b1) of `tile` and stores
// bf16.  Bulk path: the leader copies all slabs of one row block into half
// of the (now idle) smem ring with cp.async.bulk while the CTA sums the
// previous block from the other half.  Plain path (unaligned pointers, or a
// block whose slabs do not fit half the ring): cached loads from L2.
// Returns false if a copy did not land in time (status set, copies drained).
template <int GROUPS>
__device__ __noinline__ bool reduce_row_blocks(const KernelParams& p, int tile, int n_c, int b0, int b1,
                                               bool blocked, bool out_vec, bool allow_bulk, uint8_t* ring,
                                               uint32_t ring_bytes,
                                               uint64_t* red_bar, uint32_t& red_phase, bool leader, int tid,
                                               int nthreads, volatile int* mailbox, volatile int* abort_flag) {
  using namespace sm100;
  const int N = p.N;
  const int bn = p.block_n;
  const int bn_t = min(bn, N - tile * bn);
  const int col0 = tile * bn;
  const SplitGeometry geo(p.M, blocked);
  const size_t slab_stride = static_cast<size_t>(p.M) * N;
  const uint32_t half = (ring_bytes / 2u) & ~127u;
  // Bulk copies pay off for blocked row blocks of at least 32 KiB over all
  // slabs (below that, plain loads have the lower latency) and need all
  // slabs of the largest piece, a blocked row block of bn_t * 32 bytes, to fit
  // half the ring.
  const uint32_t block_bytes = static_cast<uint32_t>(n_c) * static_cast<uint32_t>(bn_t) * 32u;
  const bool bulk = allow_bulk && blocked && geo.m8 > 0 && block_bytes >= 32768u && block_bytes <= half;
  auto piece = [&](int b, int s, uint32_t& bytes) -> const float* {
    const float* slab = p.ws + static_cast<size_t>(s) * slab_stride;
    if (b < geo.m8 / 8) {
      bytes = static_cast<uint32_t>(bn_t) * 32u;
      return slab + ws_blocked_offset(8 * b, col0, N);
    }
    const int m = geo.m8 + (b - geo.m8 / 8);
    bytes = static_cast<uint32_t>(bn_t) * 4u;
    return slab + static_cast<size_t>(m) * N + col0;
  };
  // Output of one float4 unit: row m, columns c .. c+3 of the tile, to every
  // output copy.
  auto emit4 = [&](int m, int c, const float4& v) {
    const size_t off = static_cast<size_t>(m) * p.ldo + col0 + c;
    __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y);
    __nv_bfloat162 hi = __floats2bfloat162_rn(v.z, v.w);
    for (int r = 0; r < p.n_outs; ++r) {
      __nv_bfloat16* dst = p.outs[r] + off;
      if (out_vec) {
        uint2 pk;
        pk.x = *reinterpret_cast<uint32_t*>(&lo);
        pk.y = *reinterpret_cast<uint32_t*>(&hi);
        *reinterpret_cast<uint2*>(dst) = pk;
      } else {
        dst[0] = lo.x;
        dst[1] = lo.y;
        dst[2] = hi.x;
        dst[3] = hi.y;
      }
    }
  };

  if (bulk) {
    const uint64_t pol = policy_evict_first();
    auto issue = [&](int b, int buf) {
      uint32_t bytes = 0;
      piece(b, 0, bytes);
      uint8_t* dst = ring + buf * half;
      mbar_arrive_expect_tx(&red_bar[buf], bytes * static_cast<uint32_t>(n_c));
      for (int s = 0; s < n_c; ++s) {
        uint32_t pb = 0;
        const float* src = piece(b, s, pb);
        bulk_load(dst + static_cast<size_t>(s) * pb, src, pb, &red_bar[buf], pol);
      }
    };
    bool ok = true;
    bool inflight[2] = {false, false};
    if (leader) {
      fence_proxy_async_global();   // slabs acquired from other CTAs -> bulk copies
      issue(b0, 0);
    }
    inflight[0] = true;
    for (int b = b0, k = 0; b < b1; ++b, ++k) {
      const int buf = k & 1;
      if (b + 1 < b1) {
        if (leader) issue(b + 1, buf ^ 1);
        inflight[buf ^ 1] = true;
      }
      // The leader waits (bounded) and shares the outcome, so every thread
      // takes the same path through the barriers below; then each thread
      // observes the completed phase itself.
      if (leader)
        mailbox[0] = mbar_wait_bounded(&red_bar[buf], (red_phase >> buf) & 1u, abort_flag, p.status,
                                       kErrReduceWait, p.timeout_ns) ? 1 : 0;
      named_barrier_sync(1, static_cast<uint32_t>(nthreads));
      const bool landed = mailbox[0] != 0;
      named_barrier_sync(1, static_cast<uint32_t>(nthreads));
      if (!landed) {
        ok = false;
        break;
      }
      mbar_try_wait(&red_bar[buf], (red_phase >> buf) & 1u);
      red_phase ^= 1u << buf;
      inflight[buf] = false;
      uint32_t pb = 0;
      piece(b, 0, pb);
      const float4* src = reinterpret_cast<const float4*>(ring + buf * half);
      const int units = static_cast<int>(pb / 16u);
      const int stride4 = units;    // float4s per slab piece
      for (int u = tid; u < units; u += nthreads) {
        float4 tot = src[u];
        for (int s = 1; s < n_c; ++s) {
          const float4 v = src[s * stride4 + u];
          tot.x += v.x;
          tot.y += v.y;
          tot.z += v.z;
          tot.w += v.w;
        }
        if (b < geo.m8 / 8) emit4(8 * b + (u & 7), 4 * (u >> 3), tot);   // [col group][8 rows][4]
        else emit4(geo.m8 + (b - geo.m8 / 8), 4 * u, tot);
      }
      named_barrier_sync(1, static_cast<uint32_t>(nthreads));   // buffer free for block b+2
    }
    if (!ok) {
      // Copies still landing in smem must finish before the CTA moves on.
      for (int buf = 0; buf < 2; ++buf)
        if (inflight[buf]) {
          wait_for_completion(&red_bar[buf], (red_phase >> buf) & 1u, p.timeout_ns);
          red_phase ^= 1u << buf;
        }
      named_barrier_sync(1, static_cast<uint32_t>(nthreads));
    }
    return ok;
  }

  // Plain path: one flat run of units over the chunk's row blocks, so that
  // GROUPS units x 8 slabs of loads stay in flight per thread whatever the
  // row count.  A unit is 4 columns of one row (1 column when the workspace
  // is row-major with N % 4 != 0 or unaligned).
  const bool vec4 = blocked || ((N & 3) == 0 && (reinterpret_cast<uintptr_t>(p.ws) & 15u) == 0);
  const int nb8 = geo.m8 / 8;
  const int ub = bn_t * 2;                     // units of a blocked row block (8 rows x bn_t / 4)
  const int ut = vec4 ? bn_t / 4 : bn_t;       // units of a row-major row
  auto before = [&](int b) { return min(b, nb8) * ub + max(0, b - nb8) * ut; };
  const int g_end = before(b1);
  for (int g0 = before(b0) + tid; g0 < g_end; g0 += GROUPS * nthreads) {
    size_t off[GROUPS];
    int orow[GROUPS];
    int ocol[GROUPS];
#pragma unroll
    for (int q = 0; q < GROUPS; ++q) {
      const int g = min(g0 + q * nthreads, g_end - 1);
      if (g < nb8 * ub) {
        const int b = g / ub;
        const int u = g - b * ub;
        off[q] = ws_blocked_offset(8 * b, col0, N) + static_cast<size_t>(u) * 4u;
        orow[q] = 8 * b + (u & 7);
        ocol[q] = 4 * (u >> 3);
      } else {
        const int gg = g - nb8 * ub;
        const int r = gg / ut;
        const int u = gg - r * ut;
        orow[q] = geo.m8 + r;
        ocol[q] = vec4 ? 4 * u : u;
        off[q] = static_cast<size_t>(orow[q]) * N + col0 + ocol[q];
      }
    }
    float4 tot[GROUPS];
    for (int s0 = 0; s0 < n_c; s0 += 8) {
      float4 v[GROUPS][8];
#pragma unroll
      for (int q = 0; q < GROUPS; ++q)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[q][j] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if (s0 + j < n_c) {
            const float* src = p.ws + static_cast<size_t>(s0 + j) * slab_stride + off[q];
            if (vec4) v[q][j] = __ldcg(reinterpret_cast<const float4*>(src));
            else v[q][j].x = __ldcg(src);
          }
        }
#pragma unroll
      for (int q = 0; q < GROUPS; ++q)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (s0 + j >= n_c) continue;
          if (s0 + j == 0) {
            tot[q] = v[q][j];
          } else {
            tot[q].x += v[q][j].x;
            tot[q].y += v[q][j].y;
            tot[q].z += v[q][j].z;
            tot[q].w += v[q][j].w;
          }
        }
    }
#pragma unroll
    for (int q = 0; q < GROUPS; ++q) {
      if (g0 + q * nthreads >= g_end) continue;
      if (vec4) emit4(orow[q], ocol[q], tot[q]);
      else
        for (int r = 0; r < p.n_outs; ++r)
          p.outs[r][static_cast<size_t>(orow[q]) * p.ldo + col0 + ocol[q]] = __float2bfloat16_rn(tot[q].x);
    }
  }
  return true;
}

// Reduction of this CTA's split tiles of more than one chunk (at most two:
// its first and last segments), run by the active epilogue threads after
// their last segment.
// The leader polls each tile's state word; once every contributor has
// arrived it claims a chunk by compare-and-swap (a claim can never land after
// the word is reset), the CTA reduces it, and the leader counts it finished;
// whoever finishes the tile's last chunk resets the word to zero.  With
// kFlagCoopReduce every contributor helps and waits at most kHelpWaitNs for
// the others; otherwise only the last arriver (bit set in `completed`)
// reduces, and never waits.  An arrival
// count of zero means the tile is already reduced and reset.
template <int GROUPS>
__device__ __noinline__ void reduce_split_tiles(const KernelParams& p, const int (&tiles)[2], const int (&contrib)[2],
                                                int n_split, int completed, bool leader, int tid, int nthreads,
                                                bool blocked, bool out_vec, uint8_t* ring, uint32_t ring_bytes,
                                                uint64_t* red_bar, volatile int* mailbox, volatile int* abort_flag) {
  using namespace sm100;
  const bool coop = (p.flags & kFlagCoopReduce) != 0;
  const SplitGeometry geo(p.M, blocked);
  auto tile_chunks = [&](int i) { return geo.chunks(contrib[i], min(p.block_n, p.N - tiles[i] * p.block_n)); };
  const int pending_init = coop ? ((1 << n_split) - 1) : completed;
  int pending = pending_init;   // meaningful on the leader only
  uint32_t red_phase = 0;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (leader) {
      int action = -1;   // (split index << 16) | chunk
      for (int i = 0; i < n_split && action < 0; ++i) {
        if (!(pending & (1 << i))) continue;
        const int tile = tiles[i];
        const int n_c = contrib[i];
        const int R = tile_chunks(i);
        int s = load_acquire_gpu(p.sem + tile);
        while (true) {
          const int arrived = s & kArrivalMask;
          if (arrived == 0) {                 // reduced and reset already
            pending &= ~(1 << i);
            break;
          }
          if (arrived != n_c) break;          // a contributor is still running
          const int claimed = (s >> kClaimShift) & kCountMask;
          if (claimed >= R) {                 // every chunk taken
            pending &= ~(1 << i);
            break;
          }
          const int prev = atomic_cas_acq_rel_gpu(p.sem + tile, s, s + (1 << kClaimShift));
          if (prev == s) {
            action = (i << 16) | claimed;
            break;
          }
          s = prev;
        }
      }
      if (action < 0 && pending != 0 && (*abort_flag != 0 || global_timer_ns() - start > kHelpWaitNs))
        pending = 0;
      mailbox[0] = action;
      mailbox[1] = pending;
    }
    named_barrier_sync(1, static_cast<uint32_t>(nthreads));
    const int action = mailbox[0];
    const int more = mailbox[1];
    named_barrier_sync(1, static_cast<uint32_t>(nthreads));   // all have read it
    if (action >= 0) {
      const int i = action >> 16;
      const int chunk = action & 0xffff;
      const int tile = tiles[i];
      const int n_c = contrib[i];
      const int R = tile_chunks(i);
      const int b0 = static_cast<int>(static_cast<long long>(geo.nb) * chunk / R);
      const int b1 = static_cast<int>(static_cast<long long>(geo.nb) * (chunk + 1) / R);
      const bool ok = reduce_row_blocks<GROUPS>(p, tile, n_c, b0, b1, blocked, out_vec, true, ring, ring_bytes,
                                                red_bar, red_phase, leader, tid, nthreads, mailbox, abort_flag);
      if (!ok) break;
      named_barrier_sync(1, static_cast<uint32_t>(nthreads));
      if (leader) {
        const int prev = atomic_add_acq_rel_gpu(p.sem + tile, 1 << kDoneShift);
        if (((prev >> kDoneShift) & kCountMask) == R - 1) store_relaxed_gpu(p.sem + tile, 0);
      }
    } else if (more == 0) {
      break;
    } else if (leader) {
      __nanosleep(200);
    }
  }
}

// Fused gather in lines (kFlagGatherLines).  The tag of this launch: the
// epoch of the last launch completed on this rank + 1.  Read only after
// griddepcontrol.wait (the last CTA of the previous launch stored it), and
// only before this CTA counts itself done in gather_lines_count.
__device__ __forceinline__ uint32_t gather_lines_epoch(const KernelParams& p) {
  return static_cast<uint32_t>(sm100::load_relaxed_gpu(p.sync_ctr + 1)) + 1u;
}

// Cluster split-K reduction of tile `tile` (kFlagCluster), run by the active
// epilogue threads of every CTA of the tile's cluster between the two
// cluster barriers.  `buf` is the shared::cta address of this CTA's partial
// [M][block_n] fp32 (float4 column c4 of row m stored at c4 ^ (m & 7)); the
// same offset holds each peer's.  Cluster rank r sums float4 units
// [r*Q/S, (r+1)*Q/S) of the Q = M * ceil(bn_t/4) units, peers in rank order.
__device__ __forceinline__ void cluster_reduce_tile(const KernelParams& p, uint32_t buf, int tile, int tid,
                                                    int nthreads, bool out_vec) {
  using namespace sm100;
  const int S = static_cast<int>(gridDim.y);
  const int r = static_cast<int>(cluster_ctarank());
  const int bn = p.block_n;
  const int bn_s = cluster_partial_stride(bn);
  const int bn_t = min(bn, p.N - tile * bn);
  const int u4 = (bn_t + 3) / 4;
  const long long q_all = static_cast<long long>(p.M) * u4;
  const long long lo = r * q_all / S;
  const long long hi = (r + 1) * q_all / S;
  const int col_base = tile * bn;
  // kFlagGatherLines: this launch's tag (read after griddepcontrol.wait).
  const uint32_t epoch = (p.flags & kFlagGatherLines) ? gather_lines_epoch(p) : 0u;
  for (long long u = lo + tid; u < hi; u += nthreads) {
    const int m = static_cast<int>(u / u4);
    const int c4 = static_cast<int>(u - static_cast<long long>(m) * u4);
    const uint32_t off = buf + static_cast<uint32_t>((m * bn_s + 4 * (c4 ^ (m & 7))) * 4);
    // Eight peers' loads in flight at a time, summed in rank order.
    float4 tot = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int q0 = 0; q0 < kMaxClusterSplit; q0 += 8) {
      if (q0 >= S) break;
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (q0 + j < S) v[j] = ld_shared_cluster_f4(map_shared_rank(off, static_cast<uint32_t>(q0 + j)));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (q0 + j >= S) continue;
        if (q0 + j == 0) {
          tot = v[j];
        } else {
          tot.x += v[j].x;
          tot.y += v[j].y;
          tot.z += v[j].z;
          tot.w += v[j].w;
        }
      }
    }
    const int c = 4 * c4;
    const int valid = min(4, bn_t - c);
    const __nv_bfloat162 lo2 = __floats2bfloat162_rn(tot.x, tot.y);
    const __nv_bfloat162 hi2 = __floats2bfloat162_rn(tot.z, tot.w);
    if (p.flags & kFlagGatherLines) {
      // N % 4 == 0 (checked on the host), so every unit is whole.
      const size_t line = static_cast<size_t>(m) * p.lines_per_row +
                          static_cast<size_t>(p.rank * p.N + col_base + c) / 4;
      const uint64_t w0 = (static_cast<uint64_t>(epoch) << 32) | *reinterpret_cast<const uint32_t*>(&lo2);
      const uint64_t w1 = (static_cast<uint64_t>(epoch) << 32) | *reinterpret_cast<const uint32_t*>(&hi2);
      for (int i = 1; i <= p.world; ++i) {            // peers first, this rank last
        const int dst = (p.rank + i) % p.world;
        st_volatile_line(p.lines[dst] + line, w0, w1);
      }
      continue;
    }
    for (int o = 0; o < p.n_outs; ++o) {
      __nv_bfloat16* dst = p.outs[o] + static_cast<size_t>(m) * p.ldo + col_base + c;
      if (out_vec && valid == 4) {
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&lo2);
        pk.y = *reinterpret_cast<const uint32_t*>(&hi2);
        *reinterpret_cast<uint2*>(dst) = pk;
      } else {
        const __nv_bfloat16 e[4] = {lo2.x, lo2.y, hi2.x, hi2.y};
        for (int j = 0; j < valid; ++j) dst[j] = e[j];
      }
    }
  }
}

// The cluster reduction in two passes, for a grid whose inputs do not come
// from the preceding grid (kFlagIndependentInputs): pass one sums this
// thread's units over the S partials (the same rank order as
// cluster_reduce_tile, so the same bits) into registers as packed bf16,
// before the grid waits on the preceding one; pass two stores them after it.
// Only the global stores must follow the preceding grid, so the cluster
// barriers and the distributed-shared-memory reads overlap its tail instead
// of holding the SM idle.  Needs every unit of the thread in `R` registers
// (cluster_units_per_thread <= R).
__device__ __forceinline__ int cluster_units_per_thread(const KernelParams& p, int tile, int nthreads) {
  const int S = static_cast<int>(gridDim.y);
  const int bn_t = min(p.block_n, p.N - tile * p.block_n);
  const int q_all = p.M * ((bn_t + 3) / 4);   // at most 128 x 64
  const int share = (q_all + S - 1) / S;
  return (share + nthreads - 1) / nthreads;
}

template <int R>
__device__ __forceinline__ void cluster_sum_units(const KernelParams& p, uint32_t buf, int tile, int tid, int nthreads,
                                                  uint2 (&staged)[R]) {
  using namespace sm100;
  const int S = static_cast<int>(gridDim.y);
  const int r = static_cast<int>(cluster_ctarank());
  const int bn = p.block_n;
  const int bn_s = cluster_partial_stride(bn);
  const int bn_t = min(bn, p.N - tile * bn);
  const int u4 = (bn_t + 3) / 4;
  const int q_all = p.M * u4;   // at most 128 x 64
  const int lo = r * q_all / S;
  const int hi = (r + 1) * q_all / S;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int u = lo + tid + j * nthreads;
    if (u >= hi) continue;
    const int m = u / u4;
    const int c4 = u - m * u4;
    const uint32_t off = buf + static_cast<uint32_t>((m * bn_s + 4 * (c4 ^ (m & 7))) * 4);
    float4 tot = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int q0 = 0; q0 < kMaxClusterSplit; q0 += 4) {
      if (q0 >= S) break;
      float4 v[4];
#pragma unroll
      for (int jj = 0; jj < 4; ++jj)
        if (q0 + jj < S) v[jj] = ld_shared_cluster_f4(map_shared_rank(off, static_cast<uint32_t>(q0 + jj)));
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        if (q0 + jj >= S) continue;
        if (q0 + jj == 0) {
          tot = v[jj];
        } else {
          tot.x += v[jj].x;
          tot.y += v[jj].y;
          tot.z += v[jj].z;
          tot.w += v[jj].w;
        }
      }
    }
    const __nv_bfloat162 lo2 = __floats2bfloat162_rn(tot.x, tot.y);
    const __nv_bfloat162 hi2 = __floats2bfloat162_rn(tot.z, tot.w);
    staged[j].x = *reinterpret_cast<const uint32_t*>(&lo2);
    staged[j].y = *reinterpret_cast<const uint32_t*>(&hi2);
  }
}

template <int R>
__device__ __forceinline__ void cluster_store_units(const KernelParams& p, int tile, int tid, int nthreads,
                                                    bool out_vec, const uint2 (&staged)[R]) {
  using namespace sm100;
  const int S = static_cast<int>(gridDim.y);
  const int r = static_cast<int>(cluster_ctarank());
  const int bn = p.block_n;
  const int bn_t = min(bn, p.N - tile * bn);
  const int u4 = (bn_t + 3) / 4;
  const int q_all = p.M * u4;   // at most 128 x 64
  const int lo = r * q_all / S;
  const int hi = (r + 1) * q_all / S;
  const int col_base = tile * bn;
#pragma unroll
  for (int j = 0; j < R; ++j) {
    const int u = lo + tid + j * nthreads;
    if (u >= hi) continue;
    const int m = u / u4;
    const int c = 4 * (u - m * u4);
    const int valid = min(4, bn_t - c);
    for (int o = 0; o < p.n_outs; ++o) {
      __nv_bfloat16* dst = p.outs[o] + static_cast<size_t>(m) * p.ldo + col_base + c;
      if (out_vec && valid == 4) {
        *reinterpret_cast<uint2*>(dst) = staged[j];
      } else {
        const uint32_t w2[2] = {staged[j].x, staged[j].y};
        for (int e = 0; e < valid; ++e)
          dst[e] = reinterpret_cast<const __nv_bfloat16*>(w2)[e];
      }
    }
  }
}

// The cluster reduction with the next layer's activation quantisation
// (kFlagQuantizeOut; block_n and N multiples of 128, so every 128-column
// block of the output lies in one tile).  Ownership is split in whole blocks:
// rank r owns blocks [r*B/S, (r+1)*B/S) of the tile's B = M * bn_t/128, one
// warp per block, lane l summing float4 unit 32*j + l of its row over the
// peers in rank order -- the same sums, so the bf16 output is bit-identical
// to cluster_reduce_tile's.  The warp then quantises its 128 bf16 values the
// way dg_quantize_act does (bench/bench_decode.cu:459-467 of the reference):
// amax over the block (each lane's four values in order, then a shuffle
// tree), scale = max(amax, 1e-4) / 448, q = e4m3(clamp(v / scale, +-448)),
// with the same comparisons, division and conversion, so the bytes and
// scales equal the standalone quantiser's on this output.
__device__ __forceinline__ float quant_max(float a, float b) { return a < b ? b : a; }   // std::max
__device__ __forceinline__ float quant_min(float a, float b) { return b < a ? b : a; }   // std::min

__device__ __forceinline__ void cluster_reduce_tile_quant(const KernelParams& p, uint32_t buf, int tile, int wid,
                                                          int lane, int nwarps) {
  using namespace sm100;
  const int S = static_cast<int>(gridDim.y);
  const int r = static_cast<int>(cluster_ctarank());
  const int bn = p.block_n;
  const int bn_s = cluster_partial_stride(bn);
  const int bn_t = min(bn, p.N - tile * bn);
  const int bpr = bn_t / 128;                  // 128-column blocks per row of this tile
  const int blocks = p.M * bpr;
  const int blo = r * blocks / S;
  const int bhi = (r + 1) * blocks / S;
  const int col_base = tile * bn;
  const int kb_next = p.N / 128;
  for (int blk = blo + wid; blk < bhi; blk += nwarps) {
    const int m = blk / bpr;
    const int jb = blk - m * bpr;
    const int c4 = jb * 32 + lane;
    const uint32_t off = buf + static_cast<uint32_t>((m * bn_s + 4 * (c4 ^ (m & 7))) * 4);
    float4 tot = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
    for (int q0 = 0; q0 < kMaxClusterSplit; q0 += 8) {
      if (q0 >= S) break;
      float4 v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (q0 + j < S) v[j] = ld_shared_cluster_f4(map_shared_rank(off, static_cast<uint32_t>(q0 + j)));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (q0 + j >= S) continue;
        if (q0 + j == 0) {
          tot = v[j];
        } else {
          tot.x += v[j].x;
          tot.y += v[j].y;
          tot.z += v[j].z;
          tot.w += v[j].w;
        }
      }
    }
    const __nv_bfloat162 lo2 = __floats2bfloat162_rn(tot.x, tot.y);
    const __nv_bfloat162 hi2 = __floats2bfloat162_rn(tot.z, tot.w);
    const size_t col = static_cast<size_t>(col_base) + 4u * static_cast<uint32_t>(c4);
    uint2 pk;
    pk.x = *reinterpret_cast<const uint32_t*>(&lo2);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi2);
    *reinterpret_cast<uint2*>(p.output + static_cast<size_t>(m) * p.ldo + col) = pk;
    const float v4[4] = {__low2float(lo2), __high2float(lo2), __low2float(hi2), __high2float(hi2)};
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) amax = quant_max(amax, fabsf(v4[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = quant_max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = quant_max(amax, 1.0e-4f) / 448.0f;
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float c = quant_min(quant_max(v4[j] / scale, -448.0f), 448.0f);
      packed |= static_cast<uint32_t>(__nv_fp8_e4m3(c).__x) << (8 * j);
    }
    *reinterpret_cast<uint32_t*>(p.q_out + static_cast<size_t>(m) * p.N + col) = packed;
    if (lane == 0) p.q_scales[static_cast<size_t>(m) * kb_next + col_base / 128 + jb] = scale;
  }
}

// Fused gather (tensor parallel, world > 1), run by thread 0 of every CTA
// after the CTA's last output store.  Every output element was stored to all
// world ranks' gathered buffers (peer memory mapped over NVLink).  Each CTA
// that stored output makes its stores visible at system scope (one release
// fence) and every CTA counts itself done; the last CTA of the grid
// publishes the launch's epoch (this rank's previous epoch + 1) into its own
// and every peer's flag slot for this rank, then waits -- at most
// p.timeout_ns, status kErrGatherWait otherwise -- until every peer has
// published the same epoch here.  So the grid completes only when all ranks'
// slices of this launch have landed in this rank's buffer, which also keeps
// every rank within one launch of the others (the two alternating buffer
// sets rely on it).  Flags are written and polled relaxed around one fence
// per side: a release or acquire on every access at system scope measured
// microseconds each on a GPU streaming at full bandwidth.  A launch that
// recorded an error publishes nothing, so its peers' waits run out and
// report it too.  The done count and the epoch are touched only after the
// previous grid on the stream has completed (griddepcontrol.wait first).
// inline: one definition however many translation units include this header.
__device__ __noinline__ inline void gather_complete(const KernelParams& p, bool wrote_output) {
  using namespace sm100;
  griddep_wait();
  if (wrote_output) fence_acq_rel_sys();   // this CTA's peer stores before its count
  const int done = atomic_add_acq_rel_gpu(p.sync_ctr, 1);
  if (done != p.num_ctas - 1) return;
  store_relaxed_gpu(p.sync_ctr, 0);
  if (p.status != nullptr && load_relaxed_gpu(p.status) != 0) return;
  const int epoch = load_relaxed_gpu(p.my_flags + p.rank) + 1;
  fence_acq_rel_sys();
  for (int r = 0; r < p.world; ++r) store_relaxed_sys(p.peer_flags[r] + p.rank, epoch);
  const uint64_t start = global_timer_ns();
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    while (load_relaxed_sys(p.my_flags + r) - epoch < 0) {
      if (global_timer_ns() - start > p.timeout_ns) {
        if (p.status != nullptr) atomicCAS(p.status, 0, kErrGatherWait);
        return;
      }
    }
  }
  fence_acq_rel_sys();
}

// Completion of the fused gather in lines, run after the CTA's own line
// stores by its epilogue threads (`tid` of `nthreads`; the control warps may
// hold a reduced register budget and only join the barrier).  Each output
// element travels as half of an 8-byte word {2 bf16, epoch} that the writing
// rank stored into every rank's line buffer; a word is single-copy atomic, so
// seeing this launch's epoch in it means its payload has landed -- no fence
// or flag round trip.
// CTA c polls lines [c*L/G, (c+1)*L/G) of this rank's buffer (L = M *
// lines_per_row) until both words of each carry the epoch (bounded by
// p.timeout_ns, status kErrGatherWait otherwise) and unpacks them into the
// gathered [M, ldo] output.  So the grid completes only when this rank's
// gathered output is whole, which also keeps every rank within one launch of
// the others (the two alternating line-buffer sets rely on it).  The last CTA
// to finish stores the epoch for the next launch.
// Waits (bounded) until line `i` of this rank's buffer carries `epoch`.
__device__ __forceinline__ bool gather_lines_wait(const KernelParams& p, long long i, uint32_t epoch, uint64_t start,
                                                  uint64_t& w0, uint64_t& w1) {
  using namespace sm100;
  for (;;) {
    ld_volatile_line(p.lines[p.rank] + i, w0, w1);
    if (static_cast<uint32_t>(w0 >> 32) == epoch && static_cast<uint32_t>(w1 >> 32) == epoch) return true;
    if (global_timer_ns() - start > p.timeout_ns) return false;
  }
}

// kFlagGatherLinesQuant: the unpack by 128-column blocks of the gathered row
// (32 lines, one per lane; world * N % 128 == 0, checked on the host), each
// warp also quantising its block the way dg_quantize_act does
// (bench/bench_decode.cu:459-467 of the reference): amax of the block's bf16
// values (each lane's four in order, then a shuffle tree), scale =
// max(amax, 1e-4) / 448, q = e4m3(clamp(v / scale, +-448)) -- the bytes and
// scales the standalone quantiser makes from the gathered output.  q_out is
// [M, world * N], q_scales [M, world * N / 128].
__device__ __noinline__ inline void gather_lines_poll_quant(const KernelParams& p, long long cta, int tid,
                                                            int nthreads) {
  using namespace sm100;
  griddep_wait();
  const uint32_t epoch = gather_lines_epoch(p);
  const int bpr = p.lines_per_row / 32;
  const long long total = static_cast<long long>(p.M) * bpr;
  const long long lo = cta * total / p.num_ctas;
  const long long hi = (cta + 1) * total / p.num_ctas;
  const int lane = tid & 31;
  const uint64_t start = global_timer_ns();
  for (long long b = lo + tid / 32; b < hi; b += nthreads / 32) {
    uint64_t w0 = 0, w1 = 0;
    const bool ok = gather_lines_wait(p, b * 32 + lane, epoch, start, w0, w1);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0 && p.status != nullptr) atomicCAS(p.status, 0, kErrGatherWait);
      break;
    }
    const int m = static_cast<int>(b / bpr);
    const int jb = static_cast<int>(b - static_cast<long long>(m) * bpr);
    const int col = jb * 128 + lane * 4;
    uint2 v;
    v.x = static_cast<uint32_t>(w0);
    v.y = static_cast<uint32_t>(w1);
    *reinterpret_cast<uint2*>(p.output + static_cast<size_t>(m) * p.ldo + col) = v;
    const __nv_bfloat162 lo2 = *reinterpret_cast<const __nv_bfloat162*>(&v.x);
    const __nv_bfloat162 hi2 = *reinterpret_cast<const __nv_bfloat162*>(&v.y);
    const float v4[4] = {__low2float(lo2), __high2float(lo2), __low2float(hi2), __high2float(hi2)};
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) amax = quant_max(amax, fabsf(v4[j]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = quant_max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float scale = quant_max(amax, 1.0e-4f) / 448.0f;
    uint32_t packed = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float c = quant_min(quant_max(v4[j] / scale, -448.0f), 448.0f);
      packed |= static_cast<uint32_t>(__nv_fp8_e4m3(c).__x) << (8 * j);
    }
    *reinterpret_cast<uint32_t*>(p.q_out + static_cast<size_t>(m) * bpr * 128 + col) = packed;
    if (lane == 0) p.q_scales[static_cast<size_t>(m) * bpr + jb] = scale;
  }
}

__device__ __noinline__ inline void gather_lines_poll(const KernelParams& p, long long cta, int tid, int nthreads) {
  using namespace sm100;
  griddep_wait();
  const uint32_t epoch = gather_lines_epoch(p);
  const long long total = static_cast<long long>(p.M) * p.lines_per_row;
  const long long lo = cta * total / p.num_ctas;
  const long long hi = (cta + 1) * total / p.num_ctas;
  const uint64_t start = global_timer_ns();
  for (long long i = lo + tid; i < hi; i += nthreads) {
    uint64_t w0 = 0, w1 = 0;
    if (!gather_lines_wait(p, i, epoch, start, w0, w1)) {
      if (p.status != nullptr) atomicCAS(p.status, 0, kErrGatherWait);
      break;
    }
    const int m = static_cast<int>(i / p.lines_per_row);
    const int col = static_cast<int>(i - static_cast<long long>(m) * p.lines_per_row) * 4;
    uint2 v;
    v.x = static_cast<uint32_t>(w0);
    v.y = static_cast<uint32_t>(w1);
    *reinterpret_cast<uint2*>(p.output + static_cast<size_t>(m) * p.ldo + col) = v;
  }
}

// After every thread of the CTA is past its polling (a CTA barrier), one
// thread counts the CTA done; the last CTA of the grid resets the count and
// stores this launch's epoch for the next one.
__device__ __noinline__ inline void gather_lines_count(const KernelParams& p) {
  using namespace sm100;
  const uint32_t epoch = gather_lines_epoch(p);
  const int done = atomic_add_acq_rel_gpu(p.sync_ctr, 1);
  if (done == p.num_ctas - 1) {
    store_relaxed_gpu(p.sync_ctr, 0);
    store_relaxed_gpu(p.sync_ctr + 1, static_cast<int>(epoch));
  }
}

// Cluster split-K after the main loop, for every active epilogue thread: the
// tile's S partials (each CTA's in its own shared memory at w_region, rows of
// cluster_partial_stride floats) are summed in rank order and stored -- plain,
// quantised or as gather lines.  Takes part in both cluster barriers.  With
// independent inputs a thread whose share fits in registers reduces before
// waiting on the preceding grid.
template <class Tr>
__device__ __forceinline__ void cluster_epilogue(const KernelParams& p, uint8_t* w_region, bool waited,
                                                 int active_tid, int epi_threads, bool leader, bool out_vec,
                                                 volatile int* abort_flag, volatile int* wrote_output) {
  using namespace sm100;
  const int tile = static_cast<int>(blockIdx.x);
  const bool quant = (p.flags & kFlagQuantizeOut) != 0;
  const bool defer = !waited && !quant && !(p.flags & kFlagGatherLines) &&
                     cluster_units_per_thread(p, tile, epi_threads) <= Tr::kDeferUnits;
  if (!waited && !defer) griddep_wait();   // a CTA without units still stores its share
  cluster_sync_acq_rel();        // every partial of the tile is in place
  if (defer) {
    uint2 staged[Tr::kDeferUnits];
    const bool live = *abort_flag == 0;
    if (live) cluster_sum_units<Tr::kDeferUnits>(p, smem_addr(w_region), tile, active_tid, epi_threads, staged);
    cluster_sync_acq_rel();      // no peer reads this CTA's partial any more
    griddep_wait();              // the stores follow the preceding grid
    if (live) {
      if (leader) *wrote_output = 1;
      cluster_store_units<Tr::kDeferUnits>(p, tile, active_tid, epi_threads, out_vec, staged);
    }
  } else {
    if (*abort_flag == 0) {
      if (leader) *wrote_output = 1;
      if (quant)
        cluster_reduce_tile_quant(p, smem_addr(w_region), tile, active_tid / 32, active_tid & 31, epi_threads / 32);
      else
        cluster_reduce_tile(p, smem_addr(w_region), tile, active_tid, epi_threads, out_vec);
    }
    cluster_sync_acq_rel();      // no peer reads this CTA's partial any more
  }
}

// Epilogue of the swap-AB class (SwapTraits), run by its four epilogue warps.
// Warp q reads TMEM lane quarter q: thread (q, lane) holds tile rows (output
// columns) r = 32q + lane and 128 + r (only where that row is inside the
// tile, 128 + r < block_n), each for the 16 batch rows in the
// accumulator's columns, and folds every 128-K block with the other classes'
// arithmetic (combined = w_s * a_s, then one fma per element), each row with
// the weight scale of its own 128-row group.  Under cluster split-K the
// partial goes to shared memory in the [M][block_n] layout of the other
// classes and cluster_epilogue reduces it; a tile with one contributor (no
// split) is stored directly.
template <class Tr>
__device__ __forceinline__ void swap_epilogue(const KernelParams& p, uint32_t tmem_base, uint64_t* accum_full,
                                              uint64_t* accum_empty, volatile int* abort_flag,
                                              volatile int* wrote_output, uint8_t* w_region, long long u_begin,
                                              long long u_end) {
  using namespace sm100;
  const uint32_t warp = threadIdx.x / 32u;
  const uint32_t lane = threadIdx.x & 31u;
  const int M = p.M;
  const int N = p.N;
  const int KB = p.num_kb;
  const int bn = p.block_n;
  const int C = p.chunks_per_tile;
  const int r = static_cast<int>(warp * 32u + lane);   // tile row in half 0
  const int h1 = Tr::kMmaM;                            // first tile row of half 1
  const bool has1 = h1 + r < bn;                       // half 1's row is inside the tile
  const uint32_t t_lane = tmem_base + ((warp * 32u) << 16);
  const bool leader = threadIdx.x == 0;
  const bool cluster = (p.flags & kFlagCluster) != 0;
  bool out_vec = (p.ldo & 7) == 0;
  for (int o = 0; o < p.n_outs; ++o) out_vec = out_vec && (reinterpret_cast<uintptr_t>(p.outs[o]) & 15u) == 0;
  bool waited = !(p.flags & kFlagIndependentInputs);
  if (waited) griddep_wait();

  float* const part_rows = reinterpret_cast<float*>(w_region);
  const int stride = cluster_partial_stride(bn);
  // Column c of batch row j in the shared-memory partial: float4 unit c/4 of
  // the row at unit (c/4) xor (j mod 8), as the other classes store it.
  auto part_at = [&](int j, int c) -> float* {
    return part_rows + static_cast<size_t>(j) * stride + 4 * ((c >> 2) ^ (j & 7)) + (c & 3);
  };

  int acc = 0;
  long long u = u_begin;
  while (u < u_end) {
    const int tile = static_cast<int>(u / C);
    const long long tile_first = static_cast<long long>(tile) * C;
    const long long seg_end = (tile_first + C) < u_end ? (tile_first + C) : u_end;
    const int last_g = (N - 1) / kKBlock;
    const int g0 = min((tile * bn + r) / kKBlock, last_g);
    const int g1 = min((tile * bn + h1 + r) / kKBlock, last_g);
    const float* w0 = p.w_scales + static_cast<size_t>(g0) * KB;
    const float* w1 = p.w_scales + static_cast<size_t>(g1) * KB;
    float part0[Tr::kMmaN];
    float part1[Tr::kMmaN];
#pragma unroll
    for (int j = 0; j < Tr::kMmaN; ++j) part0[j] = part1[j] = 0.0f;

    for (long long uu = u; uu < seg_end; ++uu) {
      const int chunk = static_cast<int>(uu - tile_first);
      for (int s = 0; s < p.subs; ++s, ++acc) {
        const int kb = chunk * p.subs + s;
        const int buf = acc % Tr::kNumBufs;
        // Scales before the accumulator wait, so their latency hides behind it.
        float a_s[Tr::kMmaN];
#pragma unroll
        for (int j = 0; j < Tr::kMmaN; ++j) a_s[j] = __ldg(p.a_scales + static_cast<size_t>(min(j, M - 1)) * KB + kb);
        const float ws0 = __ldg(w0 + kb);
        const float ws1 = __ldg(w1 + kb);
        int ready = 0;
        if (lane == 0) {
          ready = mbar_wait_bounded(&accum_full[buf], static_cast<uint32_t>((acc / Tr::kNumBufs) & 1), abort_flag,
                                    p.status, kErrEpilogueAccumWait, p.timeout_ns)
                      ? 1
                      : 0;
        }
        ready = __shfl_sync(0xffffffffu, ready, 0);
        if (!ready) continue;
        tc_fence_after();
        uint32_t raw0[Tr::kMmaN];
        uint32_t raw1[Tr::kMmaN];
        const uint32_t t = t_lane + static_cast<uint32_t>(buf * Tr::kBnMax);
        tmem_ld_x16(t, raw0);
        tmem_ld_x16(t + static_cast<uint32_t>(Tr::kMmaN), raw1);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < Tr::kMmaN; ++j) {
          part0[j] = fmaf(ws0 * a_s[j], __uint_as_float(raw0[j]), part0[j]);
          part1[j] = fmaf(ws1 * a_s[j], __uint_as_float(raw1[j]), part1[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&accum_empty[buf]);
      }
    }

    // ------------------------------------------------------------ emit ----
    if (cluster) {
      if (*abort_flag == 0) {
#pragma unroll
        for (int j = 0; j < Tr::kMmaN; ++j) {
          if (j < M) {
            *part_at(j, r) = part0[j];
            if (has1) *part_at(j, h1 + r) = part1[j];
          }
        }
      }
    } else {
      // One contributor per tile: the tile's output, after the preceding grid.
      if (!waited) {
        griddep_wait();
        waited = true;
      }
      if (leader) *wrote_output = 1;
      const int n0 = tile * bn + r;
      if (*abort_flag == 0) {
        for (int o = 0; o < p.n_outs; ++o) {
          __nv_bfloat16* out = p.outs[o];
#pragma unroll
          for (int j = 0; j < Tr::kMmaN; ++j) {
            if (j < M) {
              if (n0 < N) out[static_cast<size_t>(j) * p.ldo + n0] = __float2bfloat16_rn(part0[j]);
              if (has1 && n0 + h1 < N) out[static_cast<size_t>(j) * p.ldo + n0 + h1] = __float2bfloat16_rn(part1[j]);
            }
          }
        }
      }
    }
    u = seg_end;
  }
  if (!cluster) return;
  // A cluster CTA without units (a split finer than the tile's chunks)
  // contributes a zero partial.
  if (u_begin == u_end && *abort_flag == 0) {
    for (int j = 0; j < M; ++j) {
      *part_at(j, r) = 0.0f;
      if (has1) *part_at(j, h1 + r) = 0.0f;
    }
  }
  cluster_epilogue<Tr>(p, w_region, waited, static_cast<int>(threadIdx.x), Tr::kEpiThreads, leader, out_vec,
                       abort_flag, wrote_output);
}

template <class Tr>
__device__ __forceinline__ void decode_gemm_body(const KernelParams& p,
                                                 const CUtensorMap* w_map,
                                                 const CUtensorMap* a_map) {
  using namespace sm100;
  const uint32_t warp = threadIdx.x / 32u;
  const uint32_t lane = threadIdx.x & 31u;

  const long long G = p.num_ctas;
  const long long U = p.total_units;
  const long long cta = static_cast<long long>(blockIdx.x) * gridDim.y + blockIdx.y;
  // The grid, block and shared memory of the plan, and under cluster split-K
  // clusters of all gridDim.y CTAs of a tile (a launch without them could
  // not reduce).
  if (static_cast<long long>(gridDim.x) * gridDim.y != G || blockDim.x != Tr::kThreads ||
      dynamic_smem_size() < p.smem_bytes || ((p.flags & kFlagCluster) && cluster_dim_y() != gridDim.y)) {
    if (threadIdx.x == 0 && p.status != nullptr) atomicCAS(p.status, 0, kErrBadLaunchShape);
    return;
  }
  const long long u_begin = cta * U / G;
  const long long u_end = (cta + 1) * U / G;
  const int n_units = static_cast<int>(u_end - u_begin);
  const int C = p.chunks_per_tile;
  const int stages = p.stages;
  const uint64_t timeout = p.timeout_ns;
  const int active_warps = active_epilogue_warps<Tr>(p.M, p.block_n);

  // ------------------------------------------------------------ smem ------
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~static_cast<uintptr_t>(1023u));
  uint8_t* w_region = smem;
  uint8_t* a_region = smem + p.w_region_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(a_region + p.a_region_bytes);
  uint64_t* full_bar = bars;                         // [stages] TMA -> MMA
  uint64_t* empty_bar = bars + stages;               // [stages] MMA -> TMA
  uint64_t* accum_full = bars + 2 * stages;          // [bufs]   MMA -> epilogue
  uint64_t* accum_empty = accum_full + Tr::kNumBufs; // [bufs]   epilogue -> MMA
  uint64_t* drain_bar = accum_empty + Tr::kNumBufs;  // MMA drain after abort
  uint64_t* never_bar = drain_bar + 1;               // test hook: nobody arrives
  uint64_t* red_bar = never_bar + 1;                 // [2] split reduction bulk copies
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* red_mailbox = abort_flag + 1;   // [2]
  volatile int* wrote_output = red_mailbox + 2; // this CTA stored output elements

  if (warp == Tr::kProducerWarp && lane == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], Tr::kMmaIssuers);
    }
    for (int b = 0; b < Tr::kNumBufs; ++b) {
      mbar_init(&accum_full[b], Tr::kMmaIssuers);
      mbar_init(&accum_empty[b], static_cast<uint32_t>(active_warps));
    }
    mbar_init(drain_bar, 1);
    mbar_init(never_bar, 1);
    mbar_init(&red_bar[0], 1);
    mbar_init(&red_bar[1], 1);
    *abort_flag = 0;
    *wrote_output = 0;
    fence_barrier_init();
  }
  if (warp == Tr::kMmaWarp) {
    tmem_alloc(tmem_slot, Tr::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // With register reallocation the control warpgroup (producer, MMA, two
  // idle warps) gives registers to the epilogue warpgroups: each warpgroup
  // runs its setmaxnreg once, at the top of its branch, so the code below it
  // is compiled for the new budget.  The host checks that the launch's
  // register pool covers the split before it launches.
  if (warp >= static_cast<uint32_t>(Tr::kEpiWarps)) {
  if constexpr (Tr::kRegRealloc) regs_decrease<kCtrlRegs>();
  if (warp == Tr::kProducerWarp) {
    // ======================================================== PRODUCER ====
    if (lane == 0) {
      const bool bulk = (p.layout == kLayoutPackedSwizzled);
      if (!bulk) prefetch_tensor_map(w_map);
      prefetch_tensor_map(a_map);
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      const uint32_t tx_bytes = p.w_stage_bytes + p.a_tx_bytes;
      auto issue_weight = [&](int i) {
        const long long u = u_begin + i;
        const int tile = static_cast<int>(u / C);
        const int chunk = static_cast<int>(u - static_cast<long long>(tile) * C);
        const int slot = i % stages;
        uint8_t* dst = w_region + static_cast<size_t>(slot) * p.w_stage_bytes;
        const int kb0 = chunk * p.subs;
        if (p.layout == kLayoutRaw) {
          tma_load_4d(w_map, &full_bar[slot], dst, 0, tile * p.block_n, kb0, 0, pol_w);
        } else if (p.layout == kLayoutPacked) {
          // Map dims {128, pack_rows, packed tiles, K blocks}: the box's
          // pack_tiles consecutive packed tiles of each K block land back to
          // back as BN contiguous 128-byte rows (tiles past the end read as
          // zeros).
          tma_load_4d(w_map, &full_bar[slot], dst, 0, 0, tile * p.pack_tiles, kb0, pol_w);
        } else {
          const size_t src_off =
              (static_cast<size_t>(tile) * p.num_kb + kb0) * static_cast<size_t>(p.block_n) * kKBlock;
          bulk_load(dst, p.weight + src_off, p.w_stage_bytes, &full_bar[slot], pol_w);
        }
      };
      auto issue_act = [&](int i) {
        const long long u = u_begin + i;
        const int tile = static_cast<int>(u / C);
        const int chunk = static_cast<int>(u - static_cast<long long>(tile) * C);
        const int slot = i % stages;
        uint8_t* a_stage = a_region + static_cast<size_t>(slot) * p.a_stage_bytes;
        for (int s = 0; s < p.subs; ++s)
#pragma unroll
          for (int c = 0; c < Tr::kCopies; ++c)
            tma_load_3d(a_map, &full_bar[slot],
                        a_stage + (s * Tr::kActRows + c * Tr::kRowsPerCopy) * kKBlock, 0, 0,
                        chunk * p.subs + s, pol_a);
      };
      // First ring pass: weights before the grid dependency resolves.
      const int first = n_units < stages ? n_units : stages;
      for (int i = 0; i < first; ++i) {
        mbar_arrive_expect_tx(&full_bar[i], tx_bytes);
        issue_weight(i);
      }
      // Release the dependent grid now, not after the last copy: its CTAs
      // take each SM the moment this grid's CTA there exits (one CTA fits
      // per SM), instead of after the slowest CTA of this grid has issued its
      // last copy.  Its griddepcontrol.wait still waits for this whole grid
      // to complete and flush, so nothing it reads or writes is affected.
      if (p.flags & kFlagPdlTrigger) griddep_launch_dependents();
      if (!(p.flags & kFlagIndependentInputs)) griddep_wait();
      for (int i = 0; i < first; ++i) issue_act(i);
      int issued = first;
      for (int i = first; i < n_units; ++i) {
        const int slot = i % stages;
        const uint32_t parity = static_cast<uint32_t>((i / stages) & 1) ^ 1u;
        if (!mbar_wait_bounded(&empty_bar[slot], parity, abort_flag, p.status,
                               kErrProducerEmptyWait, timeout))
          break;
        mbar_arrive_expect_tx(&full_bar[slot], tx_bytes);
        issue_weight(i);
        issue_act(i);
        issued = i + 1;
      }
      // Nothing may still be landing in smem when the CTA exits.  In the
      // normal path every stage has been consumed and these waits return at
      // once; after an abort they bound the wait for copies still in flight.
      if (*abort_flag != 0) {
        const int lo = issued > stages ? issued - stages : 0;
        for (int i = lo; i < issued; ++i) {
          if (!wait_for_completion(&full_bar[i % stages], static_cast<uint32_t>((i / stages) & 1),
                                   timeout) &&
              p.status != nullptr)
            atomicCAS(p.status, 0, kErrDrainTma);
        }
      }
    }
    __syncwarp();
  } else if (warp >= static_cast<uint32_t>(Tr::kMmaWarp) &&
             warp < static_cast<uint32_t>(Tr::kMmaWarp + Tr::kMmaIssuers)) {
    // ============================================================= MMA ====
    // Swap-AB: issuer `half` multiplies tile rows [128 half, 128 half + 128)
    // into accumulator columns [16 half, 16 half + 16) of each buffer; the
    // ring and accumulator barriers count one commit per issuer.  It drains
    // its own MMAs after an abort on its own barrier (the swap class has no
    // workspace reduction, so red_bar[1] is free for issuer 1).
    const int half = static_cast<int>(warp) - Tr::kMmaWarp;
    uint64_t* my_drain = half == 0 ? drain_bar : &red_bar[1];
    if (lane == 0) {
      const uint32_t idesc = Tr::kSwap ? make_idesc_e4m3_f32(Tr::kMmaM, 16u)
                                       : make_idesc_e4m3_f32(Tr::kMmaM, static_cast<uint32_t>(p.n_mma));
      const uint32_t w_sub_bytes = static_cast<uint32_t>(p.block_n) * kKBlock;
      const uint32_t a_sub_bytes = static_cast<uint32_t>(Tr::kActRows) * kKBlock;
      const uint32_t w_base = smem_addr(w_region);
      const uint32_t a_base = smem_addr(a_region);
      bool any_issued = false;
      bool ok = true;
      // Test hook: CTA 0 waits on a barrier nobody arrives on, so its bounded
      // wait runs out and it aborts while the other CTAs finish (a split tile
      // it shares is then left with a partial arrival count).
      if ((p.flags & kFlagInjectTimeout) && cta == 0) {
        ok = mbar_wait_bounded(never_bar, 0, abort_flag, p.status, kErrInjectedTimeout, timeout);
      }
      int acc = 0;  // running accumulator-buffer index
      for (int i = 0; ok && i < n_units; ++i) {
        const int slot = i % stages;
        if (!mbar_wait_bounded(&full_bar[slot], static_cast<uint32_t>((i / stages) & 1),
                               abort_flag, p.status, kErrMmaFullWait, timeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int s = 0; s < p.subs; ++s, ++acc) {
          const int buf = acc % Tr::kNumBufs;
          const uint32_t parity = static_cast<uint32_t>((acc / Tr::kNumBufs) & 1) ^ 1u;
          if (!mbar_wait_bounded(&accum_empty[buf], parity, abort_flag, p.status,
                                 kErrMmaAccumWait, timeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = a_base + slot * p.a_stage_bytes + s * a_sub_bytes;
          const uint32_t b_addr = w_base + slot * p.w_stage_bytes + s * w_sub_bytes;
          if constexpr (Tr::kSwap) {
            // A = this half's 128 weight rows (MMA M side), B = the batch
            // rows (MMA N side).  Rows past the tile (block_n < 256) come
            // from the next block of the ring or its tail pad and only feed
            // accumulator lanes the epilogue never folds.
            const uint32_t d_tmem =
                tmem_base + static_cast<uint32_t>(buf * Tr::kBnMax + half * Tr::kMmaN);
            const uint32_t w_half = b_addr + static_cast<uint32_t>(half * Tr::kMmaM * kKBlock);
#pragma unroll
            for (int k = 0; k < kKBlock / 32; ++k) {
              mma_f8f6f4(d_tmem, make_desc_k_sw128(w_half + 32u * k),
                         make_desc_k_sw128(a_addr + 32u * k), idesc, k > 0 ? 1u : 0u);
            }
          } else {
            const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * Tr::kBnMax);
            // A = activation rows (MMA M side), B = weight rows (MMA N side).
#pragma unroll
            for (int k = 0; k < kKBlock / 32; ++k) {
              mma_f8f6f4(d_tmem, make_desc_k_sw128(a_addr + 32u * k),
                         make_desc_k_sw128(b_addr + 32u * k), idesc, k > 0 ? 1u : 0u);
            }
          }
          any_issued = true;
          mma_commit(&accum_full[buf]);
        }
        if (!ok) break;
        mma_commit(&empty_bar[slot]);
      }
      if (*abort_flag != 0 && any_issued) {
        mma_commit(my_drain);
        if (!wait_for_completion(my_drain, 0, timeout) && p.status != nullptr)
          atomicCAS(p.status, 0, kErrDrainMma);
      }
    }
    __syncwarp();
  }
  // Control warps take part in the epilogue's two cluster barriers.
  if (p.flags & kFlagCluster) {
    __syncwarp();
    cluster_sync_acq_rel();
    cluster_sync_acq_rel();
  }
  } else {
    // ======================================================== EPILOGUE ====
    if constexpr (Tr::kSwap) {
      swap_epilogue<Tr>(p, tmem_base, accum_full, accum_empty, abort_flag, wrote_output, w_region, u_begin, u_end);
    } else {
    if constexpr (Tr::kRegRealloc) regs_increase<kEpiRegs>();
    const int M = p.M;
    const int N = p.N;
    const int KB = p.num_kb;
    const int bn = p.block_n;
    const EpiWarp<Tr> ew(static_cast<int>(warp), M, bn);
    const int quarter = ew.quarter;
    const int col0 = ew.col0;                          // first tile column owned
    if (ew.active) {
      const int m = ew.row0 + static_cast<int>(lane);
      const bool row_ok = (static_cast<int>(lane) < Tr::kRowsPerQuarter) && (m < M);
      const int m_c = m < M ? m : M - 1;
      const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
      const bool leader = (warp == 0 && lane == 0);
      const uint32_t epi_threads = static_cast<uint32_t>(active_warps * 32);
      // Index of this thread among the active epilogue threads.
      const int active_tid = active_epilogue_rank<Tr>(static_cast<int>(warp), M, bn) * 32 + static_cast<int>(lane);
      const float* a_s_row = p.a_scales + static_cast<size_t>(m_c) * KB;

      // Activation scales, the output and the workspace follow the preceding
      // grid; with independent inputs only the writes do (waited for at the
      // first emit).
      bool waited = !(p.flags & kFlagIndependentInputs);
      if (waited) griddep_wait();

      // 16-byte output and workspace rows need N and the base pointers aligned.
      bool out_vec = (p.ldo & 7) == 0;
      for (int r = 0; r < p.n_outs; ++r) out_vec = out_vec && (reinterpret_cast<uintptr_t>(p.outs[r]) & 15u) == 0;
      const bool ws_vec = (N & 3) == 0 && (reinterpret_cast<uintptr_t>(p.ws) & 15u) == 0;
      const int m8 = ws_vec ? (M & ~7) : 0;   // workspace rows stored in 8-row blocks
      // Split tiles this CTA contributed to (only its first and last segments
      // can be split); `completed` (leader only): bit i set when this CTA's
      // arrival was the tile's last.
      int split_tile[2] = {0, 0};
      int split_contrib[2] = {0, 0};
      int n_split = 0;
      int completed = 0;

      int acc = 0;
      long long u = u_begin;
      while (u < u_end) {
        const int tile = static_cast<int>(u / C);
        const long long tile_first = static_cast<long long>(tile) * C;
        const long long seg_end = (tile_first + C) < u_end ? (tile_first + C) : u_end;
        // Output columns n0 .. n0+63 of this warp; at most two 128-row weight
        // scale groups, split at tile column `split`.
        const int n0 = tile * bn + col0;
        const int last_scale_row = (N - 1) / kKBlock;
        const int g_lo = min(n0 / kKBlock, last_scale_row);
        const int g_hi = min(g_lo + 1, last_scale_row);
        const int split = (g_lo + 1) * kKBlock - n0;     // columns >= split use g_hi
        const float* w_lo = p.w_scales + static_cast<size_t>(g_lo) * KB;
        const float* w_hi = p.w_scales + static_cast<size_t>(g_hi) * KB;

        float partial[Tr::kColsPerWarp];
#pragma unroll
        for (int j = 0; j < Tr::kColsPerWarp; ++j) partial[j] = 0.0f;

        for (long long uu = u; uu < seg_end; ++uu) {
          const int chunk = static_cast<int>(uu - tile_first);
          for (int s = 0; s < p.subs; ++s, ++acc) {
            const int kb = chunk * p.subs + s;
            const int buf = acc % Tr::kNumBufs;
            // Scales are requested before the accumulator wait so their
            // latency hides behind it.  The reference's fold:
            // combined = w_s * a_s, then one fma per element.
            const float a_s = __ldg(a_s_row + kb);
            const float c_lo = __ldg(w_lo + kb) * a_s;
            const float c_hi = __ldg(w_hi + kb) * a_s;
            int ready = 0;
            if (lane == 0) {
              ready = mbar_wait_bounded(&accum_full[buf], static_cast<uint32_t>((acc / Tr::kNumBufs) & 1),
                                        abort_flag, p.status, kErrEpilogueAccumWait, timeout)
                          ? 1
                          : 0;
            }
            ready = __shfl_sync(0xffffffffu, ready, 0);
            if (!ready) continue;
            tc_fence_after();
            // kLdBatch 16-column loads in flight per wait.  Columns past the
            // tile width are folded too (they lie inside the 256-column
            // buffer) and never stored.  An 8-column run starts on a multiple
            // of 8 of the output, as does every 128-row scale group, so one
            // scale covers the run; each pair is one packed fma.
            const uint32_t t_row = tmem_base + lane_addr + static_cast<uint32_t>(buf * Tr::kBnMax + col0);
#pragma unroll
            for (int b = 0; b < Tr::kColsPerWarp / 16; b += Tr::kLdBatch) {
              uint32_t raw[Tr::kLdBatch][16];
#pragma unroll
              for (int q = 0; q < Tr::kLdBatch; ++q) tmem_ld_x16(t_row + static_cast<uint32_t>((b + q) * 16), raw[q]);
              tmem_wait_ld();
#pragma unroll
              for (int q = 0; q < Tr::kLdBatch; ++q) {
#pragma unroll
                for (int h = 0; h < 16; h += 8) {
                  const int c8 = (b + q) * 16 + h;
                  const float c = c8 < split ? c_lo : c_hi;
#pragma unroll
                  for (int j = 0; j < 8; j += 2)
                    ffma2(partial[c8 + j], partial[c8 + j + 1], c, __uint_as_float(raw[q][h + j]),
                          __uint_as_float(raw[q][h + j + 1]));
                }
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accum_empty[buf]);
          }
        }

        // ----------------------------------------------------- emit ------
        // Global writes follow the preceding grid; a cluster CTA's partial
        // goes to its own shared memory, and the wait comes before its first
        // global store, after the cluster reduction.
        if (!waited && !(p.flags & kFlagCluster)) {
          griddep_wait();
          waited = true;
        }
        const long long c_first = cta_of_unit(tile_first, G, U);
        const long long c_last = cta_of_unit(tile_first + C - 1, G, U);
        const int contributors = static_cast<int>(c_last - c_first + 1);
        const int ncols = min(Tr::kColsPerWarp, min(bn - col0, N - n0));   // valid columns here
        if (p.flags & kFlagCluster) {
          // This CTA's partial of its one tile -> its shared memory, reduced
          // by the cluster after the loop.
          if (row_ok && *abort_flag == 0) {
            float* row = reinterpret_cast<float*>(w_region) + static_cast<size_t>(m) * cluster_partial_stride(bn);
#pragma unroll
            for (int j4 = 0; j4 < Tr::kColsPerWarp / 4; ++j4) {
              const int c4 = (col0 >> 2) + j4;
              if (4 * c4 < bn)
                *reinterpret_cast<float4*>(row + 4 * (c4 ^ (m & 7))) =
                    make_float4(partial[4 * j4], partial[4 * j4 + 1], partial[4 * j4 + 2], partial[4 * j4 + 3]);
            }
          }
        } else if (contributors == 1) {
          if (leader) *wrote_output = 1;
          if (row_ok && *abort_flag == 0)
            for (int r = 0; r < p.n_outs; ++r)
              store_row_bf16<Tr::kColsPerWarp>(p.outs[r] + static_cast<size_t>(m) * p.ldo + n0, partial, ncols,
                                               out_vec);
        } else {
          const int slab = static_cast<int>(cta - c_first);
          const size_t slab_stride = static_cast<size_t>(M) * N;
          if (row_ok) {
            float* slab_base = p.ws + slab * slab_stride;
            if (ws_vec && m < m8)
              store_row_f32_blocked<Tr::kColsPerWarp>(slab_base, m, n0, N, partial, ncols);
            else
              store_row_f32<Tr::kColsPerWarp>(slab_base + static_cast<size_t>(m) * N + n0, partial, ncols, ws_vec);
          }
          // Arrival: the CTA barrier orders every thread's workspace stores
          // before the leader's acquire-release increment (cumulative at GPU
          // scope); whoever later sees every arrival acquires them all.
          named_barrier_sync(1, epi_threads);
          int last = 0;
          if (leader && *abort_flag == 0) {
            const int previous = atomic_add_acq_rel_gpu(p.sem + tile, 1);
            last = (previous & kArrivalMask) == contributors - 1 ? 1 : 0;
          }
          const int bn_t = min(bn, N - tile * bn);
          if (SplitGeometry(M, ws_vec).chunks(contributors, bn_t) == 1) {
            // One chunk: the last arriver reduces it at once (plain loads,
            // the smem ring is still streaming) and resets the word.
            if (leader) red_mailbox[0] = last;
            named_barrier_sync(1, epi_threads);
            last = red_mailbox[0];
            named_barrier_sync(1, epi_threads);
            if (last) {
              if (leader) *wrote_output = 1;
              uint32_t no_phase = 0;
              reduce_row_blocks<Tr::kRedGroups>(p, tile, contributors, 0, SplitGeometry(M, ws_vec).nb, ws_vec,
                                                out_vec, false, smem, 0, red_bar, no_phase, leader, active_tid,
                                                static_cast<int>(epi_threads), red_mailbox, abort_flag);
              named_barrier_sync(1, epi_threads);
              if (leader) store_relaxed_gpu(p.sem + tile, 0);
            }
          } else {
            if (last) completed |= 1 << n_split;
            split_tile[n_split] = tile;
            split_contrib[n_split] = contributors;
            ++n_split;
          }
        }
        u = seg_end;
      }
      // A cluster CTA without units (a split finer than the tile's chunks)
      // contributes a zero partial.
      if ((p.flags & kFlagCluster) && n_units == 0 && row_ok && *abort_flag == 0) {
        float* row = reinterpret_cast<float*>(w_region) + static_cast<size_t>(m) * cluster_partial_stride(bn);
#pragma unroll
        for (int j4 = 0; j4 < Tr::kColsPerWarp / 4; ++j4) {
          const int c4 = (col0 >> 2) + j4;
          if (4 * c4 < bn) *reinterpret_cast<float4*>(row + 4 * (c4 ^ (m & 7))) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      // ----------------------------------------------- split reduction ----
      // Only a CTA with reduction work enters the (cold) reduction code: any
      // recorded tile (all have more than one chunk) under kFlagCoopReduce,
      // else a tile this CTA completed.
      bool red_work = false;
      if (n_split > 0) {
        red_work = (p.flags & kFlagCoopReduce) != 0;
        if (!red_work) {
          if (leader) red_mailbox[0] = completed;
          named_barrier_sync(1, epi_threads);
          red_work = red_mailbox[0] != 0;
          named_barrier_sync(1, epi_threads);
        }
      }
      if (red_work && leader) *wrote_output = 1;
      if (red_work)
        reduce_split_tiles<Tr::kRedGroups>(p, split_tile, split_contrib, n_split, completed, leader,
                                           active_tid, static_cast<int>(epi_threads), ws_vec, out_vec, smem,
                                           p.w_region_bytes + p.a_region_bytes, red_bar, red_mailbox, abort_flag);
      if (p.flags & kFlagCluster)
        cluster_epilogue<Tr>(p, w_region, waited, active_tid, static_cast<int>(epi_threads), leader, out_vec,
                             abort_flag, wrote_output);
    } else if (p.flags & kFlagCluster) {
      cluster_sync_acq_rel();
      cluster_sync_acq_rel();
    }
    }
  }

  // --------------------------------------------------------- teardown ----
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == Tr::kMmaWarp) tmem_dealloc(tmem_base, Tr::kTmemCols);
  if (p.world > 1 && (p.flags & kFlagGatherLines)) {
    if (warp < static_cast<uint32_t>(Tr::kEpiWarps)) {
      if (p.flags & kFlagGatherLinesQuant)
        gather_lines_poll_quant(p, cta, static_cast<int>(threadIdx.x), Tr::kEpiWarps * 32);
      else
        gather_lines_poll(p, cta, static_cast<int>(threadIdx.x), Tr::kEpiWarps * 32);
    }
    __syncthreads();
    if (threadIdx.x == 0) gather_lines_count(p);
  } else if (p.world > 1 && threadIdx.x == 0) {
    gather_complete(p, *wrote_output != 0);
  }
}

// The swap-AB batch class (Tr = SwapTraits: M <= 16, 256-row tiles).
template <class Tr>
__global__ void __launch_bounds__(Tr::kThreads, 1)
    dg_decode_gemm_swap_kernel(const __grid_constant__ KernelParams p,
                               const __grid_constant__ CUtensorMap w_map,
                               const __grid_constant__ CUtensorMap a_map) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  decode_gemm_body<Tr>(p, &w_map, &a_map);
#else
  if (threadIdx.x == 0 && p.status != nullptr) atomicCAS(p.status, 0, kErrBadLaunchShape);
#endif
}

template <int MMA_M, int COPIES, int EPW>
__global__ void __launch_bounds__(KernelTraits<MMA_M, COPIES, EPW>::kThreads, 1)
    dg_decode_gemm_kernel(const __grid_constant__ KernelParams p,
                          const __grid_constant__ CUtensorMap w_map,
                          const __grid_constant__ CUtensorMap a_map) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  decode_gemm_body<KernelTraits<MMA_M, COPIES, EPW>>(p, &w_map, &a_map);
#else
  if (threadIdx.x == 0 && p.status != nullptr) atomicCAS(p.status, 0, kErrBadLaunchShape);
#endif
}

}  // namespace dg
