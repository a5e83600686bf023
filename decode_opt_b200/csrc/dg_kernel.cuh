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
// Operand placement.  A tcgen05.mma takes the same ~180 cycles whatever its
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
//                     (up to 128 weight rows) of the tile: tcgen05.ld, scale fold into fp32
//                     partials held in registers, then bf16 store or the split
//                     reduction.  Warps whose rows are all >= M, or whose
//                     columns are past the tile, stay idle.
//   warp 4E           TMA producer: weight and activation tiles of one
//                     (tile, chunk) unit per pipeline stage, `stages` deep.
//   warp 4E+1         MMA issuer and TMEM owner: one lane issues the MMAs;
//                     tcgen05.commit frees smem stages and publishes finished
//                     accumulators.
//
// Work decomposition (stream-K).  The (tile, chunk) units, chunk = `subs`
// consecutive 128-K blocks, are numbered tile-major; CTA c of G processes the
// contiguous range [floor(c*U/G), floor((c+1)*U/G)).  A tile whose units all
// fall in one CTA is written directly in bf16.  Otherwise each contributing
// CTA stores its fp32 partial into workspace slab (c - first contributor);
// a per-tile ticket elects the last arriver, which sums the slabs in slab
// order 0,1,2,... -- a fixed order, so results are run-to-run bit-identical --
// stores bf16 and re-zeroes the ticket.  The reference's S-way CTA split-K
// (gridDim.y = S, kernels/decode_gemm.cuh:1015-1077) is the special case
// G = tiles*S, where every range is one S-th of one tile.
//
// Programmatic dependent launch.  Weight tiles for the first ring pass are
// requested before griddepcontrol.wait (weights are never written by a
// preceding kernel); activation loads, scale reads and every global write
// come after it -- unless kFlagIndependentInputs declares that the inputs are
// not produced by the preceding grid, in which case only the writes wait.  The producer issues griddepcontrol.launch_dependents after
// its last TMA when kFlagPdlTrigger is set (kernels/decode_gemm.cuh:708-713).
//
// Failure behaviour.  Every wait is bounded (sm100::mbar_wait_bounded).  On a
// timeout the CTA records an error code in *status, raises a CTA-wide abort
// flag, stops issuing work, waits (bounded) for its own TMA copies and MMAs
// still in flight, frees its TMEM and exits.  No trap, no unbounded spin.

#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "sm100.cuh"

namespace dg {

constexpr int kKBlock = 128;                       // one scale group of K
constexpr uint32_t kMaxDynamicSmem = 227u * 1024u; // per CTA on sm_100
constexpr int kMaxStages = 16;
constexpr int kMaxAccumBuffers = 8;
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s

enum Layout : int {
  kLayoutRaw = 0,             // W[N,K], K contiguous
  kLayoutPacked = 1,          // [tile][kb][BN rows][128 B] (reference prepack)
  kLayoutPackedSwizzled = 2,  // same order, bytes pre-swizzled for SWIZZLE_128B
};

enum Flags : int {
  kFlagPdlTrigger = 1,     // producer issues griddepcontrol.launch_dependents
  kFlagInjectTimeout = 2,  // test hook: the MMA warp waits on a barrier nobody arrives on
  // The activation and both scale arrays are not written by the preceding
  // grid of the stream (e.g. back-to-back GEMMs on one activation): they may
  // be read before griddepcontrol.wait.  Global writes still wait.
  kFlagIndependentInputs = 4,
};

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
};

// Everything the kernel needs, computed on the host (dg_host.cuh) and passed
// by value as a __grid_constant__ parameter.
struct KernelParams {
  int M, N, K;
  int block_n;          // BN: weight rows (output columns) per tile
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
  __nv_bfloat16* output;     // [M, N]
  const float* w_scales;     // [ceil(N/128), K/128]
  const float* a_scales;     // [M, K/128]
  float* ws;                 // [slabs][M][N] fp32 (split tiles only)
  int* sem;                  // [num_tiles] tickets, zero between launches
  int* status;               // first error code, may be null
  const uint8_t* weight;     // kLayoutPackedSwizzled: bulk-copy source
};

// Compile-time geometry of one kernel instantiation: the MMA M (batch rows,
// padded) and the number of epilogue warps per TMEM lane quarter.
//
// Batch replication.  TMEM lane quarter q holds accumulator rows
// [q*R4, (q+1)*R4), R4 = MMA_M/4.  A batch that fills fewer quarters than
// there are is replicated: the activation tile is loaded kCopies = 4/EPW
// times, into row blocks of MMA_M/kCopies rows, so every quarter holds the
// whole batch (or half of it) and quarter q folds only the weight columns of
// its copy.  The MMA costs the same (its M is padded anyway); the epilogue's
// TMEM reads and FMAs are spread over all four quarters instead of landing on
// the one quarter that holds the real rows.
template <int MMA_M_, int EPW_>
struct KernelTraits {
  static constexpr int kMmaM = MMA_M_;
  static constexpr int kEpw = EPW_;                  // epilogue warps per lane quarter
  static_assert(kMmaM == 64 || kMmaM == 128, "tcgen05 cta_group::1 M is 64 or 128");
  static_assert(kEpw == 1 || kEpw == 2 || kEpw == 4, "1, 2 or 4 epilogue warps per quarter");
  static constexpr int kBnMax = 256;                 // accumulator columns per buffer
  static constexpr int kColsPerWarp = 64;            // weight columns one epilogue warp folds
  static constexpr int kCopies = 4 / kEpw;           // batch copies along the MMA M side
  static constexpr int kQuartersPerCopy = 4 / kCopies;
  static constexpr int kColsPerCopy = kBnMax / kCopies;
  static constexpr int kRowsPerQuarter = kMmaM / 4;  // accumulator rows per lane quarter
  static constexpr int kRowsPerCopy = kMmaM / kCopies;
  static constexpr int kEpiWarps = 4 * kEpw;
  static constexpr int kEpiThreads = kEpiWarps * 32;
  static constexpr int kProducerWarp = kEpiWarps;
  static constexpr int kMmaWarp = kEpiWarps + 1;
  static constexpr int kThreads = (kEpiWarps + 2) * 32;
  static constexpr int kNumBufs = 2;                 // 2 x 256 columns = all of TMEM
  static constexpr uint32_t kTmemCols = 512u;
  static_assert(kColsPerCopy == kEpw * kColsPerWarp, "column split");
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
  int n = 0;
  for (int w = 0; w < Tr::kEpiWarps; ++w) n += EpiWarp<Tr>(w, M, block_n).active ? 1 : 0;
  return n;
}

// Rank of warp w among the active epilogue warps.
template <class Tr>
__device__ __forceinline__ int active_epilogue_rank(int w, int M, int block_n) {
  int n = 0;
  for (int v = 0; v < w; ++v) n += EpiWarp<Tr>(v, M, block_n).active ? 1 : 0;
  return n;
}

struct SmemBarriers {
  static __host__ __device__ constexpr uint32_t bytes(int stages, int bufs) {
    return static_cast<uint32_t>((2 * stages + 2 * bufs + 2) * 8 + 16);
  }
};

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
  if (static_cast<long long>(gridDim.x) * gridDim.y != G || blockDim.x != Tr::kThreads) {
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
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(never_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* ticket_flag = abort_flag + 1;

  if (warp == Tr::kProducerWarp && lane == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < Tr::kNumBufs; ++b) {
      mbar_init(&accum_full[b], 1);
      mbar_init(&accum_empty[b], static_cast<uint32_t>(active_warps));
    }
    mbar_init(drain_bar, 1);
    mbar_init(never_bar, 1);
    *abort_flag = 0;
    *ticket_flag = 0;
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
          tma_load_4d(w_map, &full_bar[slot], dst, 0, 0, kb0, tile, pol_w);
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
                        a_stage + (s * Tr::kMmaM + c * Tr::kRowsPerCopy) * kKBlock, 0, 0,
                        chunk * p.subs + s, pol_a);
      };
      // First ring pass: weights before the grid dependency resolves.
      const int first = n_units < stages ? n_units : stages;
      for (int i = 0; i < first; ++i) {
        mbar_arrive_expect_tx(&full_bar[i], tx_bytes);
        issue_weight(i);
      }
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
      if (p.flags & kFlagPdlTrigger) griddep_launch_dependents();
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
  } else if (warp == Tr::kMmaWarp) {
    // ============================================================= MMA ====
    if (lane == 0) {
      const uint32_t idesc = make_idesc_e4m3_f32(Tr::kMmaM, static_cast<uint32_t>(p.n_mma));
      const uint32_t w_sub_bytes = static_cast<uint32_t>(p.block_n) * kKBlock;
      const uint32_t a_sub_bytes = static_cast<uint32_t>(Tr::kMmaM) * kKBlock;
      const uint32_t w_base = smem_addr(w_region);
      const uint32_t a_base = smem_addr(a_region);
      bool any_issued = false;
      bool ok = true;
      if (p.flags & kFlagInjectTimeout) {
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
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * Tr::kBnMax);
          // A = activation rows (MMA M side), B = weight rows (MMA N side).
          const uint32_t a_addr = a_base + slot * p.a_stage_bytes + s * a_sub_bytes;
          const uint32_t b_addr = w_base + slot * p.w_stage_bytes + s * w_sub_bytes;
#pragma unroll
          for (int k = 0; k < kKBlock / 32; ++k) {
            mma_f8f6f4(d_tmem, make_desc_k_sw128(a_addr + 32u * k),
                       make_desc_k_sw128(b_addr + 32u * k), idesc, k > 0 ? 1u : 0u);
          }
          any_issued = true;
          mma_commit(&accum_full[buf]);
        }
        if (!ok) break;
        mma_commit(&empty_bar[slot]);
      }
      if (*abort_flag != 0 && any_issued) {
        mma_commit(drain_bar);
        if (!wait_for_completion(drain_bar, 0, timeout) && p.status != nullptr)
          atomicCAS(p.status, 0, kErrDrainMma);
      }
    }
    __syncwarp();
  } else {
    // ======================================================== EPILOGUE ====
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
#pragma unroll
            for (int ch = 0; ch < Tr::kColsPerWarp / 16; ++ch) {
              const int c_first = col0 + ch * 16;
              if (c_first < bn) {   // warp-uniform
                uint32_t raw[16];
                tmem_ld_x16(tmem_base + lane_addr + static_cast<uint32_t>(buf * Tr::kBnMax + c_first), raw);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int jj = ch * 16 + j;
                  const float c = jj < split ? c_lo : c_hi;
                  partial[jj] = fmaf(c, __uint_as_float(raw[j]), partial[jj]);
                }
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accum_empty[buf]);
          }
        }

        // ----------------------------------------------------- emit ------
        if (!waited) {
          griddep_wait();
          waited = true;
        }
        const long long c_first = cta_of_unit(tile_first, G, U);
        const long long c_last = cta_of_unit(tile_first + C - 1, G, U);
        const int contributors = static_cast<int>(c_last - c_first + 1);
        const int ncols = min(Tr::kColsPerWarp, min(bn - col0, N - n0));   // valid columns here
        if (contributors == 1) {
          if (row_ok && *abort_flag == 0)
            store_row_bf16<Tr::kColsPerWarp>(p.output + static_cast<size_t>(m) * N + n0, partial, ncols,
                                             (N & 7) == 0);
        } else {
          const int slab = static_cast<int>(cta - c_first);
          const size_t slab_stride = static_cast<size_t>(M) * N;
          if (row_ok)
            store_row_f32<Tr::kColsPerWarp>(p.ws + slab * slab_stride + static_cast<size_t>(m) * N + n0,
                                            partial, ncols, (N & 3) == 0);
          // Ticket: the CTA barrier orders every thread's workspace stores
          // before the leader's acquire-release increment (cumulative at GPU
          // scope), and the last arriver's increment acquires all earlier
          // contributors' stores; the second barrier hands that to the CTA.
          named_barrier_sync(1, epi_threads);
          if (leader) {
            int last = 0;
            if (*abort_flag == 0) {
              const int previous = atomic_add_acq_rel_gpu(p.sem + tile, 1);
              last = (previous == contributors - 1) ? 1 : 0;
            }
            *ticket_flag = last;
          }
          named_barrier_sync(1, epi_threads);
          if (*ticket_flag != 0) {
            // The tile's M x BN outputs are spread over all active epilogue
            // threads (consecutive threads -> consecutive columns, coalesced),
            // four elements per thread per pass with every slab load of the
            // pass in flight together; each element is summed over the slabs
            // in slab order 0, 1, ..., contributors-1 whatever the arrival
            // order, so the result is bit-identical run to run.
            const int bn_t = min(bn, N - tile * bn);
            const int total_el = M * bn_t;
            const int T = static_cast<int>(epi_threads);
            const float* base = p.ws + static_cast<size_t>(tile) * bn;
            __nv_bfloat16* obase = p.output + static_cast<size_t>(tile) * bn;
            for (int e0 = active_tid; e0 < total_el; e0 += 4 * T) {
              size_t off[4];
              bool ok_e[4];
              float total[4];
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const int e = e0 + q * T;
                ok_e[q] = e < total_el;
                const int ee = ok_e[q] ? e : e0;
                const int mm = ee / bn_t;
                off[q] = static_cast<size_t>(mm) * N + (ee - mm * bn_t);
                total[q] = 0.0f;
              }
              for (int s0 = 0; s0 < contributors; s0 += 8) {
                float v[4][8];
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                  for (int j = 0; j < 8; ++j)
                    v[q][j] = (s0 + j) < contributors ? __ldcg(base + (s0 + j) * slab_stride + off[q]) : 0.0f;
#pragma unroll
                for (int q = 0; q < 4; ++q)
#pragma unroll
                  for (int j = 0; j < 8; ++j)
                    if ((s0 + j) < contributors) total[q] = (s0 + j) == 0 ? v[q][j] : total[q] + v[q][j];
              }
#pragma unroll
              for (int q = 0; q < 4; ++q)
                if (ok_e[q]) obase[off[q]] = __float2bfloat16_rn(total[q]);
            }
            if (leader) store_relaxed_gpu(p.sem + tile, 0);
          }
        }
        u = seg_end;
      }
    }
  }

  // --------------------------------------------------------- teardown ----
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == Tr::kMmaWarp) tmem_dealloc(tmem_base, Tr::kTmemCols);
}

template <int MMA_M, int EPW>
__global__ void __launch_bounds__(KernelTraits<MMA_M, EPW>::kThreads, 1)
    dg_decode_gemm_kernel(const __grid_constant__ KernelParams p,
                          const __grid_constant__ CUtensorMap w_map,
                          const __grid_constant__ CUtensorMap a_map) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  decode_gemm_body<KernelTraits<MMA_M, EPW>>(p, &w_map, &a_map);
#else
  if (threadIdx.x == 0 && p.status != nullptr) atomicCAS(p.status, 0, kErrBadLaunchShape);
#endif
}

}  // namespace dg
