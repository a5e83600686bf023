// SPDX-License-Identifier: MIT
//
// decode_gemm.cuh -- the C++ face of the B200 decode GEMM: the reference's
// `namespace decode_gemm` interface (kernels/decode_gemm.cuh of the reference:
// KernelConfig :147-347, Problem / GemmRuntime / LaunchPlan :352-380,
// make_weight_tma / make_activation_tma :413-468, make_launch_plan /
// ensure_smem_attribute / launch_with_maps / launch :1086-1159, and the
// __global__ fp8_decode_gemm<Cfg> that its bench launches itself), so that
// code written against that header -- bench/kernel_api.h includes
// "decode_gemm.cuh" and "weight_prepack.cuh" -- builds against this one.
//
// Build: -I <repo>/include -I <repo>/decode_opt_b200/csrc, nvcc -std=c++17
// -gencode arch=compute_100a,code=sm_100a; link -L <repo>/decode_opt_b200
// -ldecode_gemm_b200 -lcuda.
//
// Host calls go through the library's C ABI (decode_gemm_b200.h): dg_plan
// for the launch plan, dg_make_*_map for the tensor maps, dg_launch_with_maps
// for launch / launch_with_maps.  fp8_decode_gemm<Cfg> is the same sm_100a
// kernel compiled in the caller's translation unit for Cfg's batch class:
// it rebuilds the library's plan on the device from Cfg and the GemmRuntime
// (dg::make_plan runs on host and device) and runs the kernel body, so a
// caller that launches it itself with make_launch_plan's grid, block and
// shared memory gets the C ABI's results bit for bit.
//
// Mapping of the reference's configuration (B200 semantics):
//   M_TILE              batch class of the kernel (MMA M 64 up to 32, else 128)
//   OUTPUT_ROWS_PER_CTA BM: rows per tile of the weight layout (the packed
//                       layout's tile height, multiple of 8 in [8, 256]).  A CTA
//                       takes T = floor(256 / BM) consecutive BM-row tiles --
//                       the reference's TILES_PER_CTA idea, sized for the
//                       tcgen05 N side: kBlockN = T * BM weight rows (224-256
//                       for BM 32..64) per MMA, 7-8 KiB of weights per
//                       instruction instead of BM * 128 bytes.  Packed weights
//                       are read in the reference's layout as they are: one
//                       TMA box {128, BM, 1, T} per 128-K block lands the T
//                       tiles as one MMA operand.
//   SUBS_PER_STAGE      128-K blocks per pipeline stage: 1, 2 or 4
//   NUM_MATH_WG x STAGES_PER_WG  ring depth, raised to hold the cluster
//                       split's partial and reduced to what fits 227 KiB
//   PREPACK             packed (prepack) weight layout instead of raw [N][K]
//   PDL, EPI_OVERLAP    griddepcontrol.launch_dependents (either); PDL also
//                       sets programmatic stream serialization in launch*
//   SPLIT_K_CTA, SPLITK_FACTOR  the split of every tile's K range, S =
//                       max(factor, 4) (the reference's factor split BM-row
//                       tiles; a CTA tile here spans T of them): grid (tiles, S) as
//                       one thread-block cluster per tile, the S partials
//                       reduced through distributed shared memory in rank
//                       order (deterministic; no workspace or semaphore is
//                       touched, so splitk_sem stays zero).  S is a
//                       compile-time constant of Cfg, so fp8_decode_gemm<Cfg>
//                       carries it as __cluster_dims__ and a caller's own
//                       launch with make_launch_plan's grid forms the clusters.
//   MATH_REGS, PROD_REGS, SINGLE_PRODUCER_WARP, PRELOAD_ACT, SCALE_IN_SMEM,
//   TILES_PER_CTA       range-checked as the reference checks them; the
//                       sm_100a kernel's warp roles are fixed.
// The weight scales need ceil(N/128) rows; the activation map's box is
// round_up(M, 8) rows (rows >= M read as zeros).  Errors follow the
// reference: cudaError_t from launches, a reason string from validate() /
// LaunchPlan::error, std::runtime_error from a failed tensor-map encode.

#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "decode_gemm_b200.h"
#include "dg_host.cuh"
#include "weight_prepack.cuh"

namespace decode_gemm {

inline constexpr uint32_t kKBlock = 128;
inline constexpr uint32_t kMaxDynamicSmemBytes = 227u * 1024u;
inline constexpr uint32_t kRegisterFileSize = 65536;

namespace detail {

// Kernel traits of the batch class of M_TILE.
template <int M_TILE> struct ClassOf;
template <> struct ClassOf<8> { using type = dg::KernelTraits<64, 4, 1>; };
template <> struct ClassOf<16> { using type = dg::KernelTraits<64, 4, 1>; };
template <> struct ClassOf<32> { using type = dg::KernelTraits<64, 2, 2>; };
template <> struct ClassOf<64> { using type = dg::KernelTraits<128, 2, 2>; };
template <> struct ClassOf<128> { using type = dg::KernelTraits<128, 1, 2>; };

}  // namespace detail

template <int M_TILE_, int OUTPUT_ROWS_PER_CTA_, int NUM_MATH_WG_, int MATH_REGS_, int STAGES_PER_WG_,
          int TILES_PER_CTA_, int SUBS_PER_STAGE_, bool PREPACK_, bool PDL_, bool EPI_OVERLAP_, bool SPLIT_K_CTA_,
          int PROD_REGS_ = 32, bool SINGLE_PRODUCER_WARP_ = false, bool PRELOAD_ACT_ = false,
          bool SCALE_IN_SMEM_ = (M_TILE_ <= 16), int SPLITK_FACTOR_ = 0>
struct KernelConfig {
  static_assert(M_TILE_ == 8 || M_TILE_ == 16 || M_TILE_ == 32 || M_TILE_ == 64 || M_TILE_ == 128,
                "M_TILE must be one of 8/16/32/64/128");
  static_assert(OUTPUT_ROWS_PER_CTA_ > 0 && OUTPUT_ROWS_PER_CTA_ <= 256 && OUTPUT_ROWS_PER_CTA_ % 8 == 0,
                "OUTPUT_ROWS_PER_CTA (BM) must be a multiple of 8 in (0, 256]");
  static_assert(NUM_MATH_WG_ == 1 || NUM_MATH_WG_ == 2 || NUM_MATH_WG_ == 4, "NUM_MATH_WG must be 1, 2 or 4");
  static_assert(TILES_PER_CTA_ > 0 && NUM_MATH_WG_ % TILES_PER_CTA_ == 0,
                "NUM_MATH_WG must be divisible by TILES_PER_CTA");
  static_assert(STAGES_PER_WG_ > 0, "STAGES_PER_WG must be positive");
  static_assert(SUBS_PER_STAGE_ == 1 || SUBS_PER_STAGE_ == 2 || SUBS_PER_STAGE_ == 4,
                "SUBS_PER_STAGE must be 1, 2 or 4 on sm_100a");
  static_assert(MATH_REGS_ >= 24 && MATH_REGS_ <= 256 && MATH_REGS_ % 8 == 0,
                "MATH_REGS must be a multiple of 8 in the PTX range [24, 256]");
  static_assert(PROD_REGS_ >= 24 && PROD_REGS_ <= 256 && PROD_REGS_ % 8 == 0,
                "PROD_REGS must be a multiple of 8 in the PTX range [24, 256]");
  static_assert((NUM_MATH_WG_ * MATH_REGS_ + PROD_REGS_) * 128 <= static_cast<int>(kRegisterFileSize),
                "register budget exceeded: (WG*MATH_REGS + PROD_REGS)*128 <= 65536");
  static_assert(!PRELOAD_ACT_ || (M_TILE_ == 8 && PREPACK_),
                "PRELOAD_ACT is only allowed for M_TILE=8 + PREPACK");
  static_assert(SPLITK_FACTOR_ == 0 || SPLITK_FACTOR_ == 1 || SPLITK_FACTOR_ == 2 || SPLITK_FACTOR_ == 4 ||
                    SPLITK_FACTOR_ == 8,
                "SPLITK_FACTOR must be 0 (legacy: follow SPLIT_K_CTA), 1 (off), 2, 4 or 8");
  static_assert(SPLITK_FACTOR_ != 1 || !SPLIT_K_CTA_,
                "SPLITK_FACTOR=1 means split-K off and contradicts SPLIT_K_CTA=true");

  static constexpr uint32_t kMTile = static_cast<uint32_t>(M_TILE_);
  static constexpr uint32_t kOutputRows = static_cast<uint32_t>(OUTPUT_ROWS_PER_CTA_);
  static constexpr uint32_t kNumMathWgs = static_cast<uint32_t>(NUM_MATH_WG_);
  static constexpr uint32_t kMathRegisters = static_cast<uint32_t>(MATH_REGS_);
  static constexpr uint32_t kProducerRegs = static_cast<uint32_t>(PROD_REGS_);
  static constexpr uint32_t kStagesPerMathWg = static_cast<uint32_t>(STAGES_PER_WG_);
  static constexpr uint32_t kOutputTilesPerCta = static_cast<uint32_t>(TILES_PER_CTA_);
  static constexpr uint32_t kSubsPerStage = static_cast<uint32_t>(SUBS_PER_STAGE_);
  static constexpr bool kPrepack = PREPACK_;
  static constexpr bool kPdl = PDL_;
  static constexpr bool kEpiOverlap = EPI_OVERLAP_;
  static constexpr uint32_t kSplitKFactor =
      (SPLITK_FACTOR_ >= 2) ? static_cast<uint32_t>(SPLITK_FACTOR_) : ((SPLITK_FACTOR_ == 1 || !SPLIT_K_CTA_) ? 1u : 2u);
  static constexpr bool kSplitKCta = kSplitKFactor > 1u;
  static constexpr bool kSingleProducerWarp = SINGLE_PRODUCER_WARP_;
  static constexpr bool kPreloadActivation = PRELOAD_ACT_;
  static constexpr bool kScaleInSmem = SCALE_IN_SMEM_;
  static constexpr uint32_t kWgsPerOutputTile = kNumMathWgs / kOutputTilesPerCta;
  static constexpr uint32_t kStages = kNumMathWgs * kStagesPerMathWg;

  // ---- the sm_100a kernel of this configuration
  using Traits = typename detail::ClassOf<M_TILE_>::type;
  static constexpr uint32_t kNumThreads = static_cast<uint32_t>(Traits::kThreads);
  static constexpr int kMmaM = Traits::kMmaM;
  // BM-row tiles per CTA tile and the CTA tile's weight rows (the MMA N).
  static constexpr int kPackTiles = OUTPUT_ROWS_PER_CTA_ <= 128 ? 256 / OUTPUT_ROWS_PER_CTA_ : 1;
  static constexpr int kBlockN = OUTPUT_ROWS_PER_CTA_ * kPackTiles;
  // CTAs per tile: one cluster, split along K -- at least 4 (the split the
  // B200 planner takes for 224-256-row tiles of the reference's shapes in a
  // dependent chain), SPLITK_FACTOR when that asks for more.  The
  // reference's factor split BM-row tiles; a CTA tile here is T of them.
  static constexpr int kClusterSplit = kSplitKFactor > 4u ? static_cast<int>(kSplitKFactor) : 4;
  // Ring depth the kernel runs with: NUM_MATH_WG x STAGES_PER_WG, at least
  // what holds the cluster partial of M_TILE rows, at most what fits 227 KiB.
  static constexpr int kMinStages = dg::cluster_min_stages(M_TILE_, SUBS_PER_STAGE_, kBlockN, Traits::kMmaM);
  static constexpr int kRingStages =
      dg::fitted_stages(static_cast<int>(kStages) > kMinStages ? static_cast<int>(kStages) : kMinStages,
                        SUBS_PER_STAGE_, kBlockN, Traits::kMmaM);
  static constexpr uint32_t kFixedSmemBytes =
      dg::pipeline_smem_bytes(kRingStages, SUBS_PER_STAGE_, kBlockN, Traits::kMmaM);

  // The planner's configuration (host and device).
  static __host__ __device__ constexpr dg::Config b200_config() {
    dg::Config c{};
    c.m_tile = M_TILE_;
    c.block_n = kBlockN;
    c.pack_rows = (PREPACK_ && kPackTiles > 1) ? OUTPUT_ROWS_PER_CTA_ : 0;
    c.subs = SUBS_PER_STAGE_;
    c.stages = kRingStages;
    c.layout = PREPACK_ ? dg::kLayoutPacked : dg::kLayoutRaw;
    c.pdl = (PDL_ || EPI_OVERLAP_) ? 1 : 0;
    c.split_k = kClusterSplit;
    c.grid_ctas = dg::kGridCluster;
    c.epi_warps = 0;
    c.timeout_ns = 0;
    c.flags = dg::kFlagClassFromMTile;
    return c;
  }
  static dg_config c_config() {
    const dg::Config b = b200_config();
    dg_config c{};
    c.m_tile = b.m_tile;
    c.block_n = b.block_n;
    c.subs = b.subs;
    c.stages = b.stages;
    c.layout = b.layout;
    c.pdl = b.pdl;
    c.split_k = b.split_k;
    c.grid_ctas = b.grid_ctas;
    c.epi_warps = 0;
    c.flags = b.flags;
    c.timeout_ns = 0;
    c.pack_rows = b.pack_rows;
    return c;
  }

  // ---- geometry: num_output_tiles counts BM-row tiles as the reference does
  // (the packed layout's tiles; splitk_sem needs no more ints); the grid is
  // (ceil(N / kBlockN), kClusterSplit).
  static __host__ __device__ constexpr uint32_t num_output_tiles(int n) {
    return (static_cast<uint32_t>(n) + kOutputRows - 1) / kOutputRows;
  }
  static __host__ __device__ constexpr uint32_t num_ctas_x(int n) {
    return (static_cast<uint32_t>(n) + kBlockN - 1) / kBlockN;
  }
  static __host__ __device__ constexpr uint32_t num_ctas(int n) {
    return num_ctas_x(n) * static_cast<uint32_t>(kClusterSplit);
  }
  // Dynamic shared memory of a launch for M = m: the plan's (N does not
  // enter it).
  static __host__ __device__ uint32_t dynamic_smem_bytes(int m, int k) {
    const dg::Plan pl = dg::make_plan(b200_config(), m, kBlockN, k, 0);
    return pl.error == nullptr ? pl.smem_bytes : kFixedSmemBytes;
  }
  template <uint32_t K>
  static constexpr bool k_ok_for_splitk() {
    return (K % (kKBlock * kSubsPerStage * kWgsPerOutputTile * kSplitKFactor)) == 0;
  }

  // The reference's shape rules, same messages, then the sm_100a plan's.
  static const char* validate(int m, int n, int k) {
    if (m < 1 || static_cast<uint32_t>(m) > kMTile) return "M out of [1, M_TILE]";
    if (n < 1) return "N must be positive";
    if (k % kKBlock != 0) return "K must be a multiple of 128";
    const uint32_t num_k_blocks = static_cast<uint32_t>(k) / kKBlock;
    if (num_k_blocks % kSubsPerStage != 0) return "K/128 must be a multiple of SUBS_PER_STAGE";
    const uint32_t num_k_chunks = num_k_blocks / kSubsPerStage;
    if (num_k_chunks % kWgsPerOutputTile != 0) return "K/(128*SUBS) must be a multiple of WGsPerOutputTile";
    if (kSplitKCta) {
      if (num_k_chunks % kSplitKFactor != 0) return "SPLIT_K: K/(128*SUBS) must be a multiple of SPLITK_FACTOR";
      if ((num_k_chunks / kSplitKFactor) % kWgsPerOutputTile != 0)
        return "SPLIT_K: (K/S)/(128*SUBS) must be a multiple of WGsPerOutputTile";
      if ((num_k_chunks / kSplitKFactor) < kWgsPerOutputTile) return "SPLIT_K: not even one k group per warp group";
    }
    return dg::make_plan(b200_config(), m, n, k, 0).error;
  }
};

// ---------------------------------------------------------------------------
// Runtime problem (host) / kernel argument (device) -- the reference's types
// ---------------------------------------------------------------------------
struct Problem {
  int M = 0;
  int N = 0;
  int K = 0;
  const __nv_fp8_e4m3* activation = nullptr;   // [M, K], K contiguous
  const __nv_fp8_e4m3* weight = nullptr;       // PREPACK ? packed : [N, K]
  const float* weight_scales = nullptr;        // [ceil(N/128), K/128]
  const float* activation_scales = nullptr;    // [M, K/128]
  __nv_bfloat16* output = nullptr;             // [M, N]
  float* splitk_ws = nullptr;                  // split-K: [S][M][N] fp32
  int* splitk_sem = nullptr;                   // split-K: >= num_output_tiles int32, zeroed once
};

struct GemmRuntime {
  int M = 0;
  int N = 0;
  int K = 0;
  float* splitk_ws = nullptr;
  int* splitk_sem = nullptr;
};

struct LaunchPlan {
  dim3 grid{0, 0, 0};
  dim3 block{0, 0, 0};
  uint32_t smem_bytes = 0;
  int num_output_tiles = 0;
  int padded_n = 0;
  const char* error = nullptr;   // nullptr == usable
};

// ---------------------------------------------------------------------------
// The kernel entry (launched by launch_with_maps's callers themselves)
// ---------------------------------------------------------------------------
template <typename Cfg>
__global__ void __launch_bounds__(Cfg::kNumThreads, 1) __cluster_dims__(1, Cfg::kClusterSplit, 1)
    fp8_decode_gemm(__nv_bfloat16* output, const float* weight_scales, const float* activation_scales,
                    const __grid_constant__ CUtensorMap w_tma, const __grid_constant__ CUtensorMap a_tma,
                    GemmRuntime rt) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  dg::Plan plan = dg::make_plan(Cfg::b200_config(), rt.M, rt.N, rt.K, 0);
  if (plan.error != nullptr) return;
  dg::KernelParams& p = plan.params;
  p.output = output;
  p.outs[0] = output;
  p.w_scales = weight_scales;
  p.a_scales = activation_scales;
  p.ws = rt.splitk_ws;
  p.sem = rt.splitk_sem;
  p.status = nullptr;
  p.weight = nullptr;
  dg::decode_gemm_body<typename Cfg::Traits>(p, &w_tma, &a_tma);
#endif
}

namespace detail {

inline dg_problem c_problem(const Problem& p) {
  dg_problem q{};
  q.M = p.M;
  q.N = p.N;
  q.K = p.K;
  q.activation = p.activation;
  q.weight = p.weight;
  q.weight_scales = p.weight_scales;
  q.activation_scales = p.activation_scales;
  q.output = p.output;
  q.splitk_ws = p.splitk_ws;
  q.splitk_sem = p.splitk_sem;
  q.status = nullptr;
  return q;
}

// Per-thread copy of the planner's message (LaunchPlan::error points at it).
inline const char* keep_message(const char* msg) {
  thread_local char buf[96];
  std::snprintf(buf, sizeof(buf), "%s", msg);
  return buf;
}

}  // namespace detail

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <typename Cfg>
inline CUtensorMap make_weight_tma(const Problem& p) {
  CUtensorMap map{};
  const dg_config c = Cfg::c_config();
  const int rc = dg_make_weight_map(&c, p.weight, p.N, p.K, &map);
  if (rc != 0) throw std::runtime_error("cuTensorMapEncodeTiled(weight) failed: cudaError " + std::to_string(rc));
  return map;
}

template <typename Cfg>
inline CUtensorMap make_activation_tma(const Problem& p) {
  CUtensorMap map{};
  const dg_config c = Cfg::c_config();
  const int rc = dg_make_activation_map(&c, p.activation, p.M, p.K, &map);
  if (rc != 0)
    throw std::runtime_error("cuTensorMapEncodeTiled(activation) failed: cudaError " + std::to_string(rc));
  return map;
}

template <typename Cfg>
inline LaunchPlan make_launch_plan(const Problem& p) {
  LaunchPlan plan;
  plan.error = Cfg::validate(p.M, p.N, p.K);
  const dg_config c = Cfg::c_config();
  dg_plan_info info{};
  const int rc = dg_plan(&c, p.M, p.N, p.K, &info);
  if (rc == 0) {
    plan.grid = dim3(info.grid_x, info.grid_y, info.grid_z);
    plan.block = dim3(info.block_x, 1u, 1u);
    plan.smem_bytes = info.smem_bytes;
    plan.num_output_tiles = static_cast<int>(Cfg::num_output_tiles(p.N));
    plan.padded_n = prepack::padded_n(p.N, static_cast<int>(Cfg::kOutputRows));
  } else if (plan.error == nullptr) {
    plan.error = detail::keep_message(info.error[0] ? info.error : "the sm_100a planner rejects this shape");
  }
  return plan;
}

// Raises the dynamic shared-memory limit of fp8_decode_gemm<Cfg> (kept at the
// largest size requested so far) and checks that its launch register pool
// covers the kernel's register split (setmaxnreg) before anything launches it.
template <typename Cfg>
inline cudaError_t ensure_smem_attribute(uint32_t smem_bytes) {
  // Raised once per device to the sm_100 maximum (function attributes belong
  // to the device's context; the reference caches one value per process).
  static std::atomic<unsigned long long> done{0};
  if (smem_bytes > kMaxDynamicSmemBytes) return cudaErrorInvalidValue;
  if (dg::func_attribute_done(&done)) return cudaSuccess;
  const void* fn = reinterpret_cast<const void*>(&fp8_decode_gemm<Cfg>);
  const cudaError_t pool = dg::check_register_pool(fn, Cfg::Traits::kCopies, Cfg::Traits::kEpw);
  if (pool != cudaSuccess) return pool;
  return dg::set_func_attribute_once(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(kMaxDynamicSmemBytes), &done);
}

// Launch with pre-built tensor maps (keep map encoding out of timed loops).
template <typename Cfg>
inline cudaError_t launch_with_maps(const Problem& p, const CUtensorMap& w_tma, const CUtensorMap& a_tma,
                                    cudaStream_t stream) {
  if (Cfg::validate(p.M, p.N, p.K) != nullptr) return cudaErrorInvalidValue;
  if (Cfg::kSplitKCta && (p.splitk_ws == nullptr || p.splitk_sem == nullptr)) return cudaErrorInvalidValue;
  const dg_config c = Cfg::c_config();
  const dg_problem q = detail::c_problem(p);
  return static_cast<cudaError_t>(dg_launch_with_maps(&c, &q, &w_tma, &a_tma, stream, Cfg::kPdl ? 1 : 0));
}

// Encode both tensor maps, then launch.
template <typename Cfg>
inline cudaError_t launch(const Problem& p, cudaStream_t stream = nullptr) {
  if (Cfg::validate(p.M, p.N, p.K) != nullptr) return cudaErrorInvalidValue;
  if (Cfg::kSplitKCta && (p.splitk_ws == nullptr || p.splitk_sem == nullptr)) return cudaErrorInvalidValue;
  const CUtensorMap w_tma = make_weight_tma<Cfg>(p);
  const CUtensorMap a_tma = make_activation_tma<Cfg>(p);
  return launch_with_maps<Cfg>(p, w_tma, a_tma, stream);
}

}  // namespace decode_gemm
