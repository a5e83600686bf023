// SPDX-License-Identifier: MIT
//
// dg_host.cuh -- host side of the B200 decode GEMM: configuration checking,
// the launch plan (grid, smem carve-up, stream-K ranges, workspace needs),
// tensor-map encoding and the launch itself.  Shared by the C-ABI library
// (dg_capi.cu) and the header-only C++ drop-in (include/decode_gemm.cuh).
//
// Mirrors the host half of the reference's kernels/decode_gemm.cuh
// (validate :319-346, make_weight_tma :413-447, make_activation_tma :449-468,
// make_launch_plan :1086-1096, ensure_smem_attribute :1100-1109,
// launch_with_maps :1113-1147) for the sm_100a kernel in dg_kernel.cuh.
//
// cuTensorMapEncodeTiled is resolved through cudaGetDriverEntryPoint, so
// libraries built from this header do not link libcuda and load on machines
// without a GPU driver (they then report cudaErrorInsufficientDriver or
// cudaErrorNoDevice at call time).

#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstring>

#include "dg_kernel.cuh"

namespace dg {

// Runtime configuration.  The reference's compile-time KernelConfig knobs map
// onto it (include/decode_gemm.cuh); grid_ctas selects the B200 stream-K
// schedule.
struct Config {
  int m_tile = 8;         // bound on M: 8, 16, 32, 64 (MMA M = 64) or 128 (MMA M = 128)
  int block_n = 256;      // BN: weight rows per tile; multiple of 8, <= 256
  int subs = 1;           // 128-K blocks per pipeline stage: 1, 2 or 4
  int stages = 0;         // smem ring depth; 0 = as many as fit
  int layout = kLayoutRaw;
  int pdl = 0;            // 1: trigger dependents + programmatic serialization
  int split_k = 1;        // reference S (grid_ctas == 0), or the cluster split
                          // (grid_ctas == kGridCluster; 1 = choose)
  int grid_ctas = 0;      // 0: grid = tiles x split_k; > 0: stream-K over this
                          // many CTAs; -1: stream-K over one CTA per SM;
                          // kGridCluster: cluster split-K
  int epi_warps = 0;      // informational; the tile width fixes the epilogue warps
  unsigned long long timeout_ns = 0;  // bounded-wait limit; 0 = 2 s
  int flags = 0;          // kFlagIndependentInputs, kFlagSwapAB, kFlagClassFromMTile (planning),
                          // kFlagInjectTimeout (a test hook)
  int pack_rows = 0;      // kLayoutPacked: rows per tile of the packed weights when a
                          // CTA tile spans several (block_n a multiple of it); 0 = block_n
};

// grid_ctas value selecting cluster split-K: grid (tiles, S), cluster
// (1, S, 1), the tile's S partials reduced through distributed shared memory.
constexpr int kGridCluster = -2;

// Clusters of S CTAs (one CTA per SM) a B200 holds at once, S = 0..16, as
// cudaOccupancyMaxActiveClusters reports on this pool's 148-SM parts: SMs
// come in GPCs that a cluster may not straddle, so the count falls faster
// than 148/S.  Used when no device can be asked.
constexpr int kB200ClusterOccupancy[kMaxClusterSplit + 1] = {0,  148, 74, 45, 33, 26, 22, 15, 15,
                                                             15, 11,  7,  7,  7,  7,  7,  7};

// The planner's cluster split for T tiles of C chunks, given occ[S] = the
// clusters of S CTAs that fit at once (every CTA gets a chunk, S <= C).  A
// grid that needs a second wave of clusters measured 40-70% slower, so only
// one-wave splits are taken:
//   dependent launches (each GEMM waits for the previous one before reading
//   its activation): a dependent GEMM streams at ~50 GB/s per SM, so its time
//   follows the chunks its busiest CTA streams, ceil(C/S): the smallest
//   one-wave S <= 16 that minimises ceil(C/S).  The non-portable sizes above
//   8 pay off where tiles are few (tensor-parallel shards: 896 x 16384 on
//   4 x 16 CTAs instead of 4 x 8 took 11.8 -> 9.4 us, 1792 x 16384 on 7 x 16
//   instead of 8 x 8 13.3 -> 11.2); a ragged split (16 chunks over 10 CTAs)
//   measured slower than the even one with the same busiest CTA (over 8);
//   Dependent grids also leave kSpareSms SMs free (at most SMs - 20 CTAs):
//   the kernel between two GEMMs of a layer chain (the quantiser) and the
//   next GEMM's early CTAs start there while this grid runs; 16384 x 7168 on
//   all 148 SMs (74 x 2 CTAs of 224 rows) took 25.4 us per layer of the
//   61-layer chain against 23.6 on 128 (64 x 2 of 256);
//   independent inputs (consecutive GEMMs may overlap): one CTA per tile
//   (no split, no reduction) when there are at least kIndependentTileCtas
//   tiles -- at C2 (28 tiles of 256 rows) about five GEMMs then stream side
//   by side, and against a split of 2 (56 CTAs) a GEMM took 15.6 / 15.9 /
//   17.3 / 19.1 / 20.3 us instead of 15.9 / 16.4 / 18.5 / 20.8 / 23.2 at
//   M = 1 / 16 / 32 / 64 / 128 over 1,000 launches, and 17.3 / 17.4 / 18.5 /
//   21.4 / 22.6 instead of 18.1 / 18.9 / 20.5 / 22.2 / 28.8 over 20; with
//   fewer tiles the smallest S <= 8 that still gives 32 CTAs.
// 1 (no split) when not even clusters of two fit in one wave.
constexpr int kSpareSms = 20;
constexpr int kIndependentTileCtas = 24;
__host__ __device__ inline int choose_cluster_split(int T, int C, bool independent, const int* occ,
                                                    int num_sms = 148) {
  if (independent) {
    if (T >= kIndependentTileCtas) return 1;
    const int s_max = C < 8 ? C : 8;
    for (int s = 2; s <= s_max; ++s)
      if (T <= occ[s] && static_cast<long long>(T) * s >= 32) return s;
    for (int s = s_max; s >= 2; --s)
      if (T <= occ[s]) return s;
    return 1;
  }
  const int s_max = C < kMaxClusterSplit ? C : kMaxClusterSplit;
  const long long max_ctas = (num_sms > 0 ? num_sms : 148) - kSpareSms;
  int best = 1;
  int best_chunks = C;
  for (int s = 2; s <= s_max; ++s) {
    const int chunks = (C + s - 1) / s;
    if (T <= occ[s] && static_cast<long long>(T) * s <= max_ctas && chunks < best_chunks) {
      best = s;
      best_chunks = chunks;
    }
  }
  return best;
}

struct Plan {
  KernelParams params{};
  dim3 grid{0, 0, 0};
  dim3 block{0, 0, 0};
  uint32_t smem_bytes = 0;
  int mma_m = 0;
  int copies = 0;           // batch copies along the MMA M side (1, 2 or 4)
  int epw = 0;              // epilogue warps per TMEM lane quarter (1, 2 or 4)
  int epi_warps = 0;
  int max_slabs = 1;        // workspace slabs needed (1 = no split tile)
  size_t ws_floats = 0;     // max_slabs * M * N when max_slabs > 1
  int sem_ints = 0;         // num_tiles when max_slabs > 1
  int padded_n = 0;
  int cluster = 1;          // CTAs per cluster along grid y (cluster split-K)
  bool swap = false;        // swap-AB class (SwapTraits)
  const char* error = nullptr;
};

// Kernel instantiation for a batch of M rows: the MMA M, the batch copies
// the activation tile holds along it, and the epilogue warps per TMEM lane
// quarter.  Every class keeps all four lane quarters busy in the epilogue:
//   M <= 16   MMA M  64, 4 copies of 16 rows, 4 warps x 64 columns
//   M <= 32   MMA M  64, 2 copies of 32 rows, 8 warps x 64 columns
//   M <= 64   MMA M 128, 2 copies of 64 rows, 8 warps x 64 columns
//   M <= 128  MMA M 128, 1 copy,             8 warps x 128 columns
// Up to M = 32 the MMA M of 64 keeps the activation stage at 64 rows (half
// of 128), which leaves shared memory for a third 56 KiB weight stage (its
// accumulator holds 16 batch rows per lane quarter, lanes 0-15): measured
// 0.5-2 us faster than MMA M 128 at M = 17..32.  One 64-row copy at M = 64
// halves the epilogue's active lanes and measured slower than two copies
// at MMA M 128.
// With kFlagSwapAB (M <= 16) the class is SwapTraits instead: the weights
// on the MMA's M side (two 128-row MMAs per tile of 136..256 rows), the
// batch padded to 16 on its N side, 4 epilogue warps and two MMA-issuing
// warps.
struct BatchClass {
  int mma_m;
  int copies;
  int epw;
  bool swap = false;
};

__host__ __device__ inline BatchClass batch_class_for(int M) {
  if (M <= 16) return {64, 4, 1};
  if (M <= 32) return {64, 2, 2};
  if (M <= 64) return {128, 2, 2};
  return {128, 1, 2};
}

__host__ __device__ inline int mma_m_for(int M) { return batch_class_for(M).mma_m; }

constexpr int kAccumBuffers = 2;

__host__ __device__ inline int padded_n(int n, int block_n) { return ((n + block_n - 1) / block_n) * block_n; }

inline size_t packed_weight_bytes(int n, int k, int block_n) {
  return static_cast<size_t>(padded_n(n, block_n)) * static_cast<size_t>(k);
}

__host__ __device__ constexpr uint32_t align1k(uint32_t v) { return (v + 1023u) & ~1023u; }

// Dynamic shared memory of a plan: 1 KiB alignment slack, the weight ring
// (stages x subs x block_n x 128 bytes, plus the MMA's read-ahead pad when
// block_n is not a multiple of 16), the activation ring (stages x subs x
// MMA-M rows x 128 bytes) and the barrier block.
// mma_rows: weight rows the MMA reads per 128-K block (0: block_n rounded up
// to 16; the swap-AB class reads two 128-row halves); the rows past block_n
// of the ring's last block come from a tail pad.  bufs: accumulator buffers
// (their barriers are in the block).
__host__ __device__ constexpr uint32_t pipeline_smem_bytes(int stages, int subs, int block_n, int mma_m,
                                                           int mma_rows = 0, int bufs = kAccumBuffers) {
  return 1024u +
         align1k(static_cast<uint32_t>(stages * subs * block_n * kKBlock +
                                       ((mma_rows > 0 ? mma_rows : ((block_n + 15) / 16) * 16) - block_n) * kKBlock)) +
         align1k(static_cast<uint32_t>(stages * subs * mma_m * kKBlock)) + SmemBarriers::bytes(stages, bufs);
}

// The shallowest ring whose drained buffers hold the fp32 partial of M rows
// that cluster split-K keeps in shared memory (rows of cluster_partial_stride
// floats); kMaxStages when none does.
__host__ __device__ constexpr int cluster_min_stages(int M, int subs, int block_n, int mma_m) {
  int s = 1;
  while (s < kMaxStages &&
         static_cast<uint64_t>(align1k(static_cast<uint32_t>(s * subs * block_n * kKBlock +
                                                             (((block_n + 15) / 16) * 16 - block_n) * kKBlock))) +
                 align1k(static_cast<uint32_t>(s * subs * mma_m * kKBlock)) <
             static_cast<uint64_t>(M) * cluster_partial_stride(block_n) * 4u)
    ++s;
  return s;
}

// The deepest ring up to `desired` stages (at least 1) that fits 227 KiB.
__host__ __device__ constexpr int fitted_stages(int desired, int subs, int block_n, int mma_m) {
  int s = desired > kMaxStages ? kMaxStages : (desired < 1 ? 1 : desired);
  while (s > 1 && pipeline_smem_bytes(s, subs, block_n, mma_m) > kMaxDynamicSmem) --s;
  return s;
}

// Static configuration checks (no shape).
__host__ __device__ inline const char* check_config(const Config& c) {
  if (!(c.m_tile == 8 || c.m_tile == 16 || c.m_tile == 32 || c.m_tile == 64 || c.m_tile == 128))
    return "m_tile must be 8, 16, 32, 64 or 128";
  if (c.block_n < 8 || c.block_n > 256 || c.block_n % 8 != 0)
    return "block_n (BN) must be a multiple of 8 in [8, 256]";
  if (!(c.subs == 1 || c.subs == 2 || c.subs == 4)) return "subs must be 1, 2 or 4";
  if (c.stages < 0 || c.stages > kMaxStages) return "stages must be in [0, 16]";
  if (c.layout < kLayoutRaw || c.layout > kLayoutPackedSwizzled) return "unknown weight layout";
  if (c.split_k < 1) return "split_k must be >= 1";
  if (c.epi_warps != 0) return "epi_warps is chosen by the planner; leave it 0";
  if (c.pack_rows != 0 && c.pack_rows != c.block_n) {
    if (c.layout != kLayoutPacked) return "pack_rows applies to the packed layout only";
    if (c.pack_rows < 8 || c.pack_rows % 8 != 0 || c.block_n % c.pack_rows != 0)
      return "pack_rows must be a multiple of 8 that divides block_n";
  }
  return nullptr;
}

// Full plan for one (M, N, K); `num_sms` sizes the stream-K grid when
// grid_ctas < 0; `cluster_occupancy` (clusters of S CTAs that fit at once,
// S = 0..16) chooses the cluster split when split_k <= 1 -- null: the
// measured B200 table on the host (device code must give split_k).  Host
// and device code compute the same plan (the header-only kernel entry
// rebuilds it on the device).  On failure plan.error names the violated
// rule.
__host__ __device__ inline Plan make_plan(const Config& c, int M, int N, int K, int num_sms,
                                          const int* cluster_occupancy = nullptr) {
  Plan plan;
  if ((plan.error = check_config(c)) != nullptr) return plan;
  if (M < 1 || M > c.m_tile) return plan.error = "M out of [1, m_tile]", plan;
  if (N < 1) return plan.error = "N must be positive", plan;
  if (K < kKBlock || K % kKBlock != 0) return plan.error = "K must be a positive multiple of 128", plan;
  const int num_kb = K / kKBlock;
  if (num_kb % c.subs != 0) return plan.error = "K/128 must be a multiple of subs", plan;
  const int C = num_kb / c.subs;
  const int T = (N + c.block_n - 1) / c.block_n;
  const long long U = static_cast<long long>(T) * C;
  if (U > (1ll << 40)) return plan.error = "problem too large", plan;

  // kFlagClassFromMTile: the class of m_tile rather than of M (the C++
  // header's kernel entry is compiled for its KernelConfig's M_TILE).
  BatchClass bc = batch_class_for((c.flags & kFlagClassFromMTile) ? c.m_tile : M);
  if (c.flags & kFlagSwapAB) {
    if (((c.flags & kFlagClassFromMTile) ? c.m_tile : M) > SwapTraits::kMmaN)
      return plan.error = "swap-AB: M must be <= 16", plan;
    if (c.block_n <= SwapTraits::kMmaM) return plan.error = "swap-AB: block_n must be in [136, 256]", plan;
    if (c.grid_ctas != kGridCluster && !(c.grid_ctas == 0 && c.split_k == 1))
      return plan.error = "swap-AB: cluster split-K or one CTA per tile (grid_ctas 0, split_k 1)", plan;
    bc = {SwapTraits::kMmaM, 1, 1, true};
  }
  const int mma_m = bc.mma_m;
  const int epw = bc.epw;
  const int copies = bc.copies;
  // Activation rows per 128-K block in shared memory: the MMA M (batch
  // copies included), or the swap class's 16-row MMA N.
  const int act_rows = bc.swap ? SwapTraits::kActRows : mma_m;
  const int n_mma = bc.swap ? SwapTraits::kMmaN : ((c.block_n + 15) / 16) * 16;
  const int a_rows = ((M + 7) / 8) * 8;
  if (a_rows > act_rows / copies) return plan.error = "batch does not fit its activation copy", plan;
  const int bufs = kAccumBuffers;
  const uint32_t w_stage = static_cast<uint32_t>(c.subs * c.block_n * kKBlock);
  const uint32_t a_stage = static_cast<uint32_t>(c.subs * act_rows * kKBlock);
  const uint32_t a_tx = static_cast<uint32_t>(c.subs * copies * a_rows * kKBlock);
  // The MMA reads n_mma weight rows from each 128-K block (the swap class:
  // two 128-row halves, 256 rows); rows past those loaded come from the next
  // block or this tail pad and only feed output columns that are never
  // stored.
  const int mma_rows = bc.swap ? 2 * SwapTraits::kMmaM : n_mma;
  const uint32_t w_pad = static_cast<uint32_t>((mma_rows - c.block_n) * kKBlock);
  (void)bufs;
  auto smem_for = [&](int stages) -> uint32_t {
    return pipeline_smem_bytes(stages, c.subs, c.block_n, act_rows, mma_rows,
                               bc.swap ? SwapTraits::kNumBufs : kAccumBuffers);
  };
  int stages = c.stages;
  if (stages == 0) {
    stages = 1;
    while (stages < kMaxStages && smem_for(stages + 1) <= kMaxDynamicSmem) ++stages;
  }
  if (smem_for(stages) > kMaxDynamicSmem) return plan.error = "dynamic shared memory exceeds 227 KiB", plan;

  long long G;
  int cluster = 1;
  if (c.grid_ctas == kGridCluster) {
#if defined(__CUDA_ARCH__)
    const int* occ = cluster_occupancy;
#else
    const int* occ = cluster_occupancy != nullptr ? cluster_occupancy : kB200ClusterOccupancy;
#endif
    if (c.split_k <= 1 && occ == nullptr) return plan.error = "cluster split: give split_k", plan;
    const int S = c.split_k > 1 ? c.split_k
                                : choose_cluster_split(T, C, (c.flags & kFlagIndependentInputs) != 0, occ, num_sms);
    if (S > kMaxClusterSplit) return plan.error = "cluster split: split_k must be <= 16", plan;
    // A given split may exceed the chunks of a tile: the CTAs left without a
    // chunk contribute zero partials.
    // The fp32 partial [M][block_n] (rows padded to a multiple of 32 floats)
    // goes to the drained pipeline ring.
    if (S > 1 && static_cast<uint64_t>(M) * cluster_partial_stride(c.block_n) * 4u >
                     static_cast<uint64_t>(align1k(stages * w_stage + w_pad)) + align1k(stages * a_stage))
      return plan.error = "cluster split: the M x block_n fp32 partial exceeds the pipeline's shared memory", plan;
    G = static_cast<long long>(T) * S;
    if (T > 0x7fffffff) return plan.error = "grid too large", plan;
    plan.grid = dim3(static_cast<unsigned>(T), static_cast<unsigned>(S), 1u);
    cluster = S;
  } else if (c.grid_ctas > 0) {
    G = c.grid_ctas < U ? c.grid_ctas : U;
    plan.grid = dim3(static_cast<unsigned>(G), 1u, 1u);
  } else if (c.grid_ctas < 0) {
    const long long sms = num_sms > 0 ? num_sms : 148;
    G = sms < U ? sms : U;
    plan.grid = dim3(static_cast<unsigned>(G), 1u, 1u);
  } else {
    if (C % c.split_k != 0) return plan.error = "split-K: (K/128)/subs must be a multiple of split_k", plan;
    G = static_cast<long long>(T) * c.split_k;
    if (T > 0x7fffffff || c.split_k > 65535) return plan.error = "grid too large", plan;
    plan.grid = dim3(static_cast<unsigned>(T), static_cast<unsigned>(c.split_k), 1u);
  }
  // Slabs of a split tile: the reference schedule gives every tile exactly
  // split_k contributors (C % split_k == 0); stream-K counts them.
  int max_slabs = (cluster == 1 && c.grid_ctas == 0) ? c.split_k : 1;
  for (int t = 0; cluster == 1 && c.grid_ctas != 0 && t < T; ++t) {
    const long long first = cta_of_unit(static_cast<long long>(t) * C, G, U);
    const long long last = cta_of_unit(static_cast<long long>(t) * C + C - 1, G, U);
    max_slabs = max_slabs > static_cast<int>(last - first + 1) ? max_slabs : static_cast<int>(last - first + 1);
  }
  if (max_slabs > kMaxContributors) return plan.error = "split too fine: more than 1023 CTAs share one tile", plan;

  KernelParams& p = plan.params;
  p.M = M;
  p.N = N;
  p.K = K;
  p.block_n = c.block_n;
  p.pack_rows = (c.layout == kLayoutPacked && c.pack_rows != 0) ? c.pack_rows : c.block_n;
  p.pack_tiles = c.block_n / p.pack_rows;
  p.n_mma = n_mma;
  p.a_rows = a_rows;
  p.subs = c.subs;
  p.stages = stages;
  p.layout = c.layout;
  p.num_tiles = T;
  p.chunks_per_tile = C;
  p.num_kb = num_kb;
  p.num_ctas = static_cast<int>(G);
  // Contributors of a split tile may wait (bounded) for one another only when
  // the whole grid fits on the device at once: one CTA per SM always fits.
  const bool coop = num_sms > 0 && G <= num_sms;
  p.flags = (c.pdl ? kFlagPdlTrigger : 0) | (coop ? kFlagCoopReduce : 0) | (cluster > 1 ? kFlagCluster : 0) |
            (c.flags & ~(kFlagPdlTrigger | kFlagCoopReduce | kFlagCluster));
  p.total_units = U;
  p.w_stage_bytes = w_stage;
  p.a_stage_bytes = a_stage;
  p.a_tx_bytes = a_tx;
  p.w_region_bytes = align1k(stages * w_stage + w_pad);
  p.a_region_bytes = align1k(stages * a_stage);
  p.smem_bytes = smem_for(stages);
  p.timeout_ns = c.timeout_ns ? c.timeout_ns : kDefaultTimeoutNs;
  p.ldo = N;
  p.n_outs = 1;
  p.world = 1;
  p.rank = 0;

  plan.epi_warps = 4 * epw;
  plan.block = dim3(static_cast<unsigned>(bc.swap ? SwapTraits::kThreads : block_threads(copies, epw)), 1u, 1u);
  plan.swap = bc.swap;
  plan.smem_bytes = p.smem_bytes;
  plan.mma_m = mma_m;
  plan.copies = copies;
  plan.epw = epw;
  plan.max_slabs = max_slabs;
  plan.ws_floats = max_slabs > 1 ? static_cast<size_t>(max_slabs) * M * static_cast<size_t>(N) : 0;
  plan.sem_ints = max_slabs > 1 ? T : 0;
  plan.padded_n = padded_n(N, p.pack_rows);
  plan.cluster = cluster;
  return plan;
}

// ----------------------------------------------------------- tensor maps ---
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_tiled_fn() {
  static std::atomic<EncodeTiledFn> cached{nullptr};
  EncodeTiledFn fn = cached.load(std::memory_order_acquire);
  if (fn != nullptr) return fn;
  void* sym = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &sym, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || sym == nullptr)
    return nullptr;
  fn = reinterpret_cast<EncodeTiledFn>(sym);
  cached.store(fn, std::memory_order_release);
  return fn;
}

// Weight map.  Both TMA layouts use a rank-4 map so that one copy lands
// subs*BM*128 bytes in [subs][BM][128] order with the 128-byte swizzle the
// MMA descriptors expect:
//   raw    dims {128, N, K/128, 1}, byte strides {K, 128, N*K}, box {128, BM,
//          subs, 1}: dim 0 and 2 walk K in 128-byte blocks, dim 1 walks rows
//          (the K-block split keeps the inner box at the 128-byte swizzle
//          span);
//   packed dims {128, R, tiles, K/128} (R = pack_rows, the packed tile
//          height), strides {128, (K/128)*R*128, R*128}, box {128, R, BM/R,
//          subs}.
// The swizzled-packed layout is read with bulk copies and needs no map.
inline cudaError_t make_weight_map(CUtensorMap* map, const Config& c, const void* weight, int N, int K) {
  std::memset(map, 0, sizeof(*map));
  if (c.layout == kLayoutPackedSwizzled) return cudaSuccess;
  EncodeTiledFn encode = encode_tiled_fn();
  if (encode == nullptr) return cudaErrorInsufficientDriver;
  const cuuint64_t kb = static_cast<cuuint64_t>(K / kKBlock);
  cuuint64_t dims[4];
  cuuint64_t strides[3];
  if (c.layout == kLayoutRaw) {
    dims[0] = kKBlock;
    dims[1] = static_cast<cuuint64_t>(N);
    dims[2] = kb;
    dims[3] = 1;
    strides[0] = static_cast<cuuint64_t>(K);
    strides[1] = kKBlock;
    strides[2] = static_cast<cuuint64_t>(N) * static_cast<cuuint64_t>(K);
  } else {
    // Packed [tile][kb][rows][128] with the tile dimension ahead of the K
    // blocks (strides need not grow with the dimension): box {128, rows,
    // block_n / rows, subs} lands [sub][block_n rows][128 B], the MMA's
    // operand order, also when one CTA tile spans several packed tiles.
    const cuuint64_t rows = static_cast<cuuint64_t>(c.pack_rows != 0 ? c.pack_rows : c.block_n);
    const cuuint64_t tiles = (static_cast<cuuint64_t>(N) + rows - 1) / rows;
    dims[0] = kKBlock;
    dims[1] = rows;
    dims[2] = tiles;
    dims[3] = kb;
    strides[0] = kKBlock;
    strides[1] = kb * rows * kKBlock;
    strides[2] = rows * kKBlock;
  }
  const bool packed = c.layout == kLayoutPacked;
  const cuuint32_t rows_box = static_cast<cuuint32_t>(packed && c.pack_rows != 0 ? c.pack_rows : c.block_n);
  const cuuint32_t box[4] = {kKBlock, rows_box,
                             static_cast<cuuint32_t>(packed ? c.block_n / rows_box : c.subs),
                             static_cast<cuuint32_t>(packed ? c.subs : 1)};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(weight), dims, strides,
                            box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Activation map: dims {128, M, K/128}, strides {K, 128}, box {128, a_rows, 1}
// with a_rows = M rounded up to 8 (rows M..a_rows-1 land as zeros); the
// producer issues one box per 128-K block and batch copy.  The map does not
// depend on the configuration (kept in the signature beside the weight map's).
inline cudaError_t make_activation_map(CUtensorMap* map, const Config& /*c*/, const void* act, int M, int K) {
  std::memset(map, 0, sizeof(*map));
  EncodeTiledFn encode = encode_tiled_fn();
  if (encode == nullptr) return cudaErrorInsufficientDriver;
  const cuuint64_t dims[3] = {kKBlock, static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(K / kKBlock)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(K), kKBlock};
  const cuuint32_t box[3] = {kKBlock, static_cast<cuuint32_t>(((M + 7) / 8) * 8), 1u};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(act), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// ---------------------------------------------------------------- launch ---
using KernelFn = void (*)(KernelParams, CUtensorMap, CUtensorMap);

template <int MMA_M, int COPIES, int EPW>
inline KernelFn kernel_ptr() {
  return reinterpret_cast<KernelFn>(&dg_decode_gemm_kernel<MMA_M, COPIES, EPW>);
}

inline KernelFn swap_kernel_ptr() { return reinterpret_cast<KernelFn>(&dg_decode_gemm_swap_kernel<SwapTraits>); }

// A kernel that reallocates registers (setmaxnreg) needs a launch register
// pool, threads x registers per thread at launch, that covers the split;
// setmaxnreg.inc would otherwise wait forever.  Checked once per kernel.
inline cudaError_t check_register_pool(const void* fn, int copies, int epw) {
  if (!uses_reg_realloc(copies, epw)) return cudaSuccess;
  cudaFuncAttributes attr{};
  const cudaError_t err = cudaFuncGetAttributes(&attr, fn);
  if (err != cudaSuccess) return err;
  const long long pool = static_cast<long long>(attr.numRegs) * block_threads(copies, epw);
  const long long need = static_cast<long long>(kEpiRegs) * 32 * 4 * epw +
                         static_cast<long long>(kCtrlRegs) * 32 * ctrl_warps(copies, epw);
  return pool >= need ? cudaSuccess : cudaErrorInvalidConfiguration;
}

// Raises the dynamic-smem limit of `fn` once per (kernel, size).  Unlike the
// reference's single cached value per Cfg (kernels/decode_gemm.cuh:1100-1109)
// this keeps the largest size set so far per kernel, so interleaved callers
// with different M never lower it under each other.
// Function attributes belong to the current device's context, so a cache of
// "already set" keeps one bit per device id below 64 (devices from 64 on set
// the attribute on every call).
inline unsigned long long current_device_bit() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return 0ull;
  }
  return (dev >= 0 && dev < 64) ? (1ull << dev) : 0ull;
}

inline bool func_attribute_done(const std::atomic<unsigned long long>* done) {
  const unsigned long long bit = current_device_bit();
  return bit != 0ull && (done->load(std::memory_order_acquire) & bit) != 0ull;
}

// Sets `attr` = `value` on `fn` for the current device unless `done` says it
// was set there already.
inline cudaError_t set_func_attribute_once(const void* fn, cudaFuncAttribute attr, int value,
                                           std::atomic<unsigned long long>* done) {
  const unsigned long long bit = current_device_bit();
  if (bit != 0ull && (done->load(std::memory_order_acquire) & bit) != 0ull) return cudaSuccess;
  const cudaError_t err = cudaFuncSetAttribute(fn, attr, value);
  if (err == cudaSuccess && bit != 0ull) done->fetch_or(bit, std::memory_order_acq_rel);
  return err;
}

// Raises the kernel's dynamic shared memory limit to the sm_100 maximum (once
// per device); every plan's smem_bytes is at most that.
inline cudaError_t ensure_smem(const void* fn, std::atomic<unsigned long long>* done) {
  return set_func_attribute_once(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(kMaxDynamicSmem), done);
}

// Checks the pointers a plan needs before anything is enqueued.
inline cudaError_t check_buffers(const Plan& plan, const KernelParams& p) {
  if (p.output == nullptr || p.w_scales == nullptr || p.a_scales == nullptr) return cudaErrorInvalidValue;
  if (plan.max_slabs > 1 && (p.ws == nullptr || p.sem == nullptr)) return cudaErrorInvalidValue;
  if (p.layout == kLayoutPackedSwizzled &&
      (p.weight == nullptr || (reinterpret_cast<uintptr_t>(p.weight) & 15u) != 0))
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

inline cudaError_t launch_kernel(KernelFn fn, const Plan& plan, const KernelParams& p, const CUtensorMap& w,
                                 const CUtensorMap& a, cudaStream_t stream, bool pdl_attr) {
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[2]{};
  cfg.gridDim = plan.grid;
  cfg.blockDim = plan.block;
  cfg.dynamicSmemBytes = plan.smem_bytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (pdl_attr) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
    ++cfg.numAttrs;
  }
  if (plan.cluster > 1) {
    attr[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
    attr[cfg.numAttrs].val.clusterDim.x = 1;
    attr[cfg.numAttrs].val.clusterDim.y = static_cast<unsigned>(plan.cluster);
    attr[cfg.numAttrs].val.clusterDim.z = 1;
    ++cfg.numAttrs;
  }
  return cudaLaunchKernelEx(&cfg, fn, p, w, a);
}

}  // namespace dg
