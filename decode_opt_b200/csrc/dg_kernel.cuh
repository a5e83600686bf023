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
// (kernels/decode_gemm.cuh:574-1081).  It is a new design for Blackwell:
//
// Swap-AB on tcgen05.  A weight tile of BM output rows is the MMA's M side
// (M=128 when BM>64, else M=64) and the batch (M=1..128 decode rows) is the
// narrow N side, rounded up to 16.  One `tcgen05.mma.kind::f8f6f4` covers
// K=32, four cover one 128-wide scale block.  Each scale block accumulates into
// its own TMEM buffer (fresh: the first of the four MMAs does not accumulate),
// so the per-block dequantisation stays exact:
//     partial[m] = fmaf(w_s * a_s[m], raw_kb[m], partial[m])     (fp32)
// which is the reference's numerical path (kernels/decode_gemm.cuh:897-946).
//
// Warp roles (one CTA per SM, 2 + EPI_WARPS warps):
//   warp 0       TMA producer: weight + activation tiles for one pipeline
//                stage per (tile, chunk) unit into a ring of `stages` slots;
//   warp 1       MMA issuer and TMEM owner: one elected lane issues the
//                tcgen05.mma chain, tcgen05.commit frees smem slots and
//                publishes finished accumulators;
//   warps 2..    epilogue: TMEM -> registers (tcgen05.ld), scale fold into
//                fp32 partials held in registers, then bf16 store or the
//                split reduction.  Warp w reads TMEM lane quarter (w % 4).
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
// come after it.  The producer issues griddepcontrol.launch_dependents after
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
constexpr int kMaxAccumBuffers = 16;
constexpr uint64_t kDefaultTimeoutNs = 2000000000ull;  // 2 s

enum Layout : int {
  kLayoutRaw = 0,             // W[N,K], K contiguous
  kLayoutPacked = 1,          // [tile][kb][BM rows][128 B] (reference prepack)
  kLayoutPackedSwizzled = 2,  // same order, bytes pre-swizzled for SWIZZLE_128B
};

enum Flags : int {
  kFlagPdlTrigger = 1,     // producer issues griddepcontrol.launch_dependents
  kFlagInjectTimeout = 2,  // test hook: the MMA warp waits on a barrier nobody arrives on
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
  int block_n;          // BM: output rows per tile
  int subs;             // 128-K blocks per pipeline stage
  int stages;           // smem ring depth
  int layout;           // Layout
  int n_mma;            // MMA N = activation rows per box (M rounded up to 16)
  int num_tiles;        // ceil(N / BM)
  int chunks_per_tile;  // (K/128) / subs
  int num_kb;           // K/128
  int num_scale_rows;   // ceil(N/128)
  int num_ctas;         // G
  int flags;
  long long total_units;     // num_tiles * chunks_per_tile
  uint32_t w_stage_bytes;    // subs * BM * 128
  uint32_t a_stage_bytes;    // subs * n_mma * 128
  uint32_t w_region_bytes;   // stages * w_stage_bytes + tail pad, 1 KiB aligned
  uint32_t a_region_bytes;   // stages * a_stage_bytes
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

// Compile-time geometry of one kernel instantiation.
template <int MMA_M_, int M_TILE_, int EPI_WARPS_>
struct KernelTraits {
  static constexpr int kMmaM = MMA_M_;
  static constexpr int kMTile = M_TILE_;
  static constexpr int kEpiWarps = EPI_WARPS_;
  static_assert(kMmaM == 64 || kMmaM == 128, "tcgen05 cta_group::1 M is 64 or 128");
  static_assert(kMTile == 8 || kMTile == 16 || kMTile == 32 || kMTile == 64 || kMTile == 128,
                "M_TILE must be 8/16/32/64/128");
  static_assert(kEpiWarps == 4 || kEpiWarps == 8, "4 or 8 epilogue warps");
  static constexpr int kThreads = (2 + kEpiWarps) * 32;
  static constexpr int kEpiThreads = kEpiWarps * 32;
  // TMEM columns of one accumulator buffer (fp32: one column per batch row).
  static constexpr int kColsPerBuf = kMTile < 16 ? 16 : kMTile;
  static constexpr int kNumBufs =
      (512 / kColsPerBuf) < kMaxAccumBuffers ? (512 / kColsPerBuf) : kMaxAccumBuffers;
  static constexpr int kTmemColsRaw = kNumBufs * kColsPerBuf;
  static constexpr uint32_t kTmemCols =
      kTmemColsRaw <= 32 ? 32u : kTmemColsRaw <= 64 ? 64u : kTmemColsRaw <= 128 ? 128u
      : kTmemColsRaw <= 256 ? 256u : 512u;
  // Batch columns owned by one epilogue thread (8 warps split them in halves).
  static constexpr int kColGroups = kEpiWarps / 4;
  static constexpr int kPartial = kMTile / kColGroups;
  static constexpr int kLoadWidth = kPartial < 16 ? kPartial : 16;
  static constexpr int kLoads = kPartial / kLoadWidth;
  static_assert(kPartial % kLoadWidth == 0, "column split");
  // Rows of the MMA tile one epilogue warp owns in its TMEM lane quarter.
  static constexpr int kRowsPerWarp = kMmaM / 4;
};

// Shared-memory carve-up that follows the 1 KiB-aligned operand regions.
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

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < Tr::kNumBufs; ++b) {
      mbar_init(&accum_full[b], 1);
      mbar_init(&accum_empty[b], Tr::kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    mbar_init(never_bar, 1);
    *abort_flag = 0;
    *ticket_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Tr::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ======================================================== PRODUCER ====
    if (lane == 0) {
      const bool swizzled_bulk = (p.layout == kLayoutPackedSwizzled);
      if (!swizzled_bulk) prefetch_tensor_map(w_map);
      prefetch_tensor_map(a_map);
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_a = policy_evict_last();
      const uint32_t tx_bytes = p.w_stage_bytes + p.a_stage_bytes;
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
        tma_load_3d(a_map, &full_bar[slot], a_region + static_cast<size_t>(slot) * p.a_stage_bytes,
                    0, 0, chunk * p.subs, pol_a);
      };
      // First ring pass: weights before the grid dependency resolves.
      const int first = n_units < stages ? n_units : stages;
      for (int i = 0; i < first; ++i) {
        mbar_arrive_expect_tx(&full_bar[i], tx_bytes);
        issue_weight(i);
      }
      griddep_wait();
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
      // Drain: nothing may still be landing in smem when the CTA exits.  In
      // the normal path the MMA warp has consumed every stage, so these
      // waits return at once; after an abort they bound the wait for the
      // copies this thread started.
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
  } else if (warp == 1) {
    // ============================================================= MMA ====
    if (lane == 0) {
      const uint32_t idesc = make_idesc_e4m3_f32(Tr::kMmaM, static_cast<uint32_t>(p.n_mma));
      const uint32_t w_sub_bytes = static_cast<uint32_t>(p.block_n) * kKBlock;
      const uint32_t a_sub_bytes = static_cast<uint32_t>(p.n_mma) * kKBlock;
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
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * Tr::kColsPerBuf);
          const uint32_t a_addr = w_base + slot * p.w_stage_bytes + s * w_sub_bytes;
          const uint32_t b_addr = a_base + slot * p.a_stage_bytes + s * a_sub_bytes;
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
    const int e = static_cast<int>(warp) - 2;           // 0 .. kEpiWarps-1
    const int quarter = static_cast<int>(warp & 3u);    // TMEM lane quarter
    const int col0 = (e / 4) * Tr::kPartial;            // first batch column owned
    const int row = quarter * Tr::kRowsPerWarp + static_cast<int>(lane);
    const bool lane_has_row = (Tr::kMmaM == 128) || (lane < 16u);
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int M = p.M;
    const int N = p.N;
    const int KB = p.num_kb;
    const bool leader = (e == 0 && lane == 0);

    griddep_wait();   // activation scales, output and workspace come after the producer grid

    int acc = 0;
    long long u = u_begin;
    while (u < u_end) {
      const int tile = static_cast<int>(u / C);
      const long long tile_first = static_cast<long long>(tile) * C;
      const long long seg_end = (tile_first + C) < u_end ? (tile_first + C) : u_end;
      const int n = tile * p.block_n + row;
      const bool row_ok = lane_has_row && row < p.block_n && n < N;
      const int g = (n < N ? n : N - 1) / kKBlock;
      const float* w_s_row = p.w_scales + static_cast<size_t>(g) * KB;

      float partial[Tr::kPartial];
#pragma unroll
      for (int j = 0; j < Tr::kPartial; ++j) partial[j] = 0.0f;

      for (long long uu = u; uu < seg_end; ++uu) {
        const int chunk = static_cast<int>(uu - tile_first);
        for (int s = 0; s < p.subs; ++s, ++acc) {
          const int kb = chunk * p.subs + s;
          const int buf = acc % Tr::kNumBufs;
          const float w_s = __ldg(w_s_row + kb);
          int ready = 0;
          if (lane == 0) {
            ready = mbar_wait_bounded(&accum_full[buf], static_cast<uint32_t>((acc / Tr::kNumBufs) & 1),
                                      abort_flag, p.status, kErrEpilogueAccumWait, timeout)
                        ? 1
                        : 0;
          }
          ready = __shfl_sync(0xffffffffu, ready, 0);
          if (ready) {
            tc_fence_after();
#pragma unroll
            for (int ld = 0; ld < Tr::kLoads; ++ld) {
              const int c_first = col0 + ld * Tr::kLoadWidth;
              if (c_first < M) {   // warp-uniform
                uint32_t raw[Tr::kLoadWidth];
                const uint32_t taddr = tmem_base + lane_addr +
                                       static_cast<uint32_t>(buf * Tr::kColsPerBuf + c_first);
                if constexpr (Tr::kLoadWidth == 16) {
                  tmem_ld_x16(taddr, reinterpret_cast<uint32_t(&)[16]>(raw));
                } else {
                  tmem_ld_x8(taddr, reinterpret_cast<uint32_t(&)[8]>(raw));
                }
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < Tr::kLoadWidth; ++j) {
                  const int m = c_first + j;
                  if (m < M) {
                    const float a_s = __ldg(p.a_scales + static_cast<size_t>(m) * KB + kb);
                    partial[ld * Tr::kLoadWidth + j] =
                        fmaf(w_s * a_s, __uint_as_float(raw[j]), partial[ld * Tr::kLoadWidth + j]);
                  }
                }
              }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&accum_empty[buf]);
          }
        }
      }

      // ------------------------------------------------------- emit ------
      const long long c_first = cta_of_unit(tile_first, G, U);
      const long long c_last = cta_of_unit(tile_first + C - 1, G, U);
      const int contributors = static_cast<int>(c_last - c_first + 1);
      if (contributors == 1) {
        if (row_ok && *abort_flag == 0) {
#pragma unroll
          for (int j = 0; j < Tr::kPartial; ++j) {
            const int m = col0 + j;
            if (m < M) p.output[static_cast<size_t>(m) * N + n] = __float2bfloat16_rn(partial[j]);
          }
        }
      } else {
        const int slab = static_cast<int>(cta - c_first);
        const size_t slab_stride = static_cast<size_t>(M) * N;
        if (row_ok) {
          float* dst = p.ws + slab * slab_stride + n;
#pragma unroll
          for (int j = 0; j < Tr::kPartial; ++j) {
            const int m = col0 + j;
            if (m < M) __stcg(dst + static_cast<size_t>(m) * N, partial[j]);
          }
        }
        __threadfence();
        named_barrier_sync(1, Tr::kEpiThreads);
        if (leader) {
          int last = 0;
          if (*abort_flag == 0) {
            const int previous = atomicAdd(p.sem + tile, 1);
            last = (previous == contributors - 1) ? 1 : 0;
          }
          *ticket_flag = last;
        }
        named_barrier_sync(1, Tr::kEpiThreads);
        if (*ticket_flag != 0) {
          __threadfence();
          if (row_ok) {
            const float* src = p.ws + n;
#pragma unroll
            for (int j = 0; j < Tr::kPartial; ++j) {
              const int m = col0 + j;
              if (m < M) {
                const size_t off = static_cast<size_t>(m) * N;
                float total = __ldcg(src + off);
                for (int sl = 1; sl < contributors; ++sl) total += __ldcg(src + sl * slab_stride + off);
                p.output[off + n] = __float2bfloat16_rn(total);
              }
            }
          }
          if (leader) atomicExch(p.sem + tile, 0);
        }
      }
      u = seg_end;
    }
  }

  // --------------------------------------------------------- teardown ----
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, Tr::kTmemCols);
}

template <int MMA_M, int M_TILE, int EPI_WARPS>
__global__ void __launch_bounds__((2 + EPI_WARPS) * 32, 1)
    dg_decode_gemm_kernel(const __grid_constant__ KernelParams p,
                          const __grid_constant__ CUtensorMap w_map,
                          const __grid_constant__ CUtensorMap a_map) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  decode_gemm_body<KernelTraits<MMA_M, M_TILE, EPI_WARPS>>(p, &w_map, &a_map);
#else
  if (threadIdx.x == 0 && p.status != nullptr) atomicCAS(p.status, 0, kErrBadLaunchShape);
#endif
}

}  // namespace dg
