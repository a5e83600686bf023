// SPDX-License-Identifier: MIT
//
// oracle/oracle.cpp -- CPU restatement of the reference's FP8 decode-GEMM
// numerics.  TEST INFRASTRUCTURE ONLY: the product (decode_opt_b200/) never
// links, loads or calls this file.  Only tests/, __graft_entry__.smoke() and
// bench.py's CPU-baseline leg use it, and only as the checker.
//
// Parity is pinned: tests/test_oracle.py checks every generator and the
// reference GEMM here bit-for-bit against (a) golden fixtures produced by the
// reference's own smoke_test.cu host code (tests/golden/make_golden.py, via
// oracle/ref_shim.cu) and (b) that same reference build when it is present
// (oracle/_ref/libref_oracle.so).
//
// Each function cites the reference function it restates.  The random streams
// must come from the same libstdc++ `std::mt19937_64` +
// `std::normal_distribution<float>` as the reference, because the C++
// standard leaves normal_distribution's algorithm to the implementation.
//
// Exported C ABI (all host pointers, caller-allocated):
//   orc_fp8_lut                      256-entry e4m3 -> float table
//   orc_bf16_round                   round-to-nearest-even to bf16, as float
//   orc_quant_e4m3                   float -> e4m3 byte (CUDA header conversion)
//   orc_gen_weight_smoke             smoke_test.cu generate_weight
//   orc_gen_activation_smoke         smoke_test.cu generate_activation
//   orc_gen_weight_bench             bench_decode.cu make_weights
//   orc_gen_activation_bench         bench_decode.cu make_activation
//   orc_quantize_rows                bench_decode.cu:459-467, the block quantisation
//                                    of make_activation, on given rows
//   orc_gen_pertensor                per-tensor-scaled N(0,1) inputs (BASELINE mode)
//   orc_compute_reference            smoke_test.cu compute_reference
//   orc_compute_reference_mt         same, N split over threads (bit-identical)
//   orc_prepack                      weight_prepack.cuh packed layout, on the CPU
//   orc_prepack_swizzled             the B200 descriptor-ready packed layout

#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <random>
#include <thread>
#include <vector>

namespace {

constexpr float kFp8Max = 448.0f;           // kernels/smoke_test.cu:45
constexpr float kQuantEps = 1.0e-4f;        // kernels/smoke_test.cu:46
constexpr int kKBlock = 128;                // kernels/decode_gemm.cuh:77

float g_lut[256];
bool g_lut_ready = false;

// kernels/smoke_test.cu:60-69 -- e4m3 byte -> float, non-finite mapped to 0.
void init_lut() {
  if (g_lut_ready) return;
  for (int i = 0; i < 256; ++i) {
    __nv_fp8_e4m3 v;
    v.__x = static_cast<uint8_t>(i);
    const float f = static_cast<float>(v);
    g_lut[i] = std::isfinite(f) ? f : 0.0f;
  }
  g_lut_ready = true;
}

// kernels/smoke_test.cu:100
inline float bf16_round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// kernels/smoke_test.cu:133 / bench/bench_decode.cu:397-401: clamp to +-448
// then convert with the CUDA header's round-to-nearest e4m3 conversion.
inline uint8_t quant(float v, float scale) {
  const float q = std::min(std::max(v / scale, -kFp8Max), kFp8Max);
  return __nv_fp8_e4m3(q).__x;
}

// splitmix64: derives independent per-block seeds for the per-tensor
// generator (no reference counterpart; see orc_gen_pertensor).
inline uint64_t splitmix64(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

}  // namespace

extern "C" {

void orc_fp8_lut(float* out256) {
  init_lut();
  std::memcpy(out256, g_lut, sizeof(g_lut));
}

float orc_bf16_round(float v) { return bf16_round(v); }

uint8_t orc_quant_e4m3(float v) { return __nv_fp8_e4m3(v).__x; }

// Restates kernels/smoke_test.cu:102-140 (generate_weight).  weight: [N,K]
// bytes; scales: [ceil(N/128), K/128].  Values are N(0,1)/sqrt(K) rounded to
// bf16, drawn for a full 128x128 block even when the last block has fewer than
// 128 real rows, then quantised per 128x128 block with scale =
// max(amax, 1e-4)/448.
void orc_gen_weight_smoke(int N, int K, uint64_t seed, uint8_t* weight, float* scales) {
  const int kb_count = K / kKBlock;
  const int scale_rows = (N + kKBlock - 1) / kKBlock;
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  const float inv_sqrt_k = 1.0f / std::sqrt(static_cast<float>(K));
  std::vector<float> block(kKBlock * kKBlock);
  for (int nb = 0; nb < scale_rows; ++nb) {
    for (int kb = 0; kb < kb_count; ++kb) {
      float amax = 0.0f;
      for (int i = 0; i < kKBlock * kKBlock; ++i) {
        block[i] = bf16_round(normal(rng) * inv_sqrt_k);
        amax = std::max(amax, std::fabs(block[i]));
      }
      const float scale = std::max(amax, kQuantEps) / kFp8Max;
      scales[static_cast<size_t>(nb) * kb_count + kb] = scale;
      const int rows = std::min(kKBlock, N - nb * kKBlock);
      for (int r = 0; r < rows; ++r) {
        uint8_t* dst = weight + static_cast<size_t>(nb * kKBlock + r) * K +
                       static_cast<size_t>(kb) * kKBlock;
        const float* src = &block[static_cast<size_t>(r) * kKBlock];
        for (int c = 0; c < kKBlock; ++c) dst[c] = quant(src[c], scale);
      }
    }
  }
}

// Restates kernels/smoke_test.cu:142-168 (generate_activation).  act: [M,K]
// bytes; scales: [M, K/128].  Row by row, 128 bf16-rounded N(0,1)/sqrt(K)
// draws per k_block, quantised per 1x128 block.  The smoke test seeds this
// with seed ^ (0x9e3779b97f4a7c15 * M) (kernels/smoke_test.cu:523); the
// caller passes the already-mixed seed.
void orc_gen_activation_smoke(int M, int K, uint64_t seed, uint8_t* act, float* scales) {
  const int kb_count = K / kKBlock;
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  const float inv_sqrt_k = 1.0f / std::sqrt(static_cast<float>(K));
  float values[kKBlock];
  for (int m = 0; m < M; ++m) {
    for (int kb = 0; kb < kb_count; ++kb) {
      float amax = 0.0f;
      for (int c = 0; c < kKBlock; ++c) {
        values[c] = bf16_round(normal(rng) * inv_sqrt_k);
        amax = std::max(amax, std::fabs(values[c]));
      }
      const float scale = std::max(amax, kQuantEps) / kFp8Max;
      scales[static_cast<size_t>(m) * kb_count + kb] = scale;
      uint8_t* dst = act + static_cast<size_t>(m) * K + static_cast<size_t>(kb) * kKBlock;
      for (int c = 0; c < kKBlock; ++c) dst[c] = quant(values[c], scale);
    }
  }
}

// Restates bench/bench_decode.cu:404-444 (make_weights).  n_ker =
// ceil(n_log/128)*128 rows are produced; rows >= n_log are exact zeros but
// still consume draws only for rows < n_log.  scales has nb+1 rows, the last
// one zero (the bench's out-of-bounds guard row).  No bf16 rounding here.
void orc_gen_weight_bench(int n_log, int K, uint64_t seed, uint8_t* weight, float* scales) {
  const int n_ker = ((n_log + 127) / 128) * 128;
  const int kb = K / kKBlock;
  const int nb = n_ker / 128;
  std::memset(scales, 0, sizeof(float) * static_cast<size_t>(nb + 1) * kb);
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  const float inv_sqrt_k = 1.0f / std::sqrt(static_cast<float>(K));
  std::vector<float> block(128 * 128);
  for (int nbi = 0; nbi < nb; ++nbi) {
    for (int kbi = 0; kbi < kb; ++kbi) {
      float amax = 0.0f;
      for (int r = 0; r < 128; ++r) {
        const int n = nbi * 128 + r;
        for (int c = 0; c < 128; ++c) {
          const float v = (n < n_log) ? static_cast<float>(normal(rng) * inv_sqrt_k) : 0.0f;
          block[r * 128 + c] = v;
          amax = std::max(amax, std::abs(v));
        }
      }
      const float scale = std::max(amax, kQuantEps) / kFp8Max;
      scales[static_cast<size_t>(nbi) * kb + kbi] = scale;
      for (int r = 0; r < 128; ++r) {
        const int n = nbi * 128 + r;
        uint8_t* dst = weight + static_cast<size_t>(n) * K + static_cast<size_t>(kbi) * 128;
        for (int c = 0; c < 128; ++c) dst[c] = quant(block[r * 128 + c], scale);
      }
    }
  }
}

// Restates bench/bench_decode.cu:446-470 (make_activation): a full row of K
// draws first, then per-1x128 quantisation of that row.
void orc_gen_activation_bench(int rows, int K, uint64_t seed, uint8_t* act, float* scales) {
  const int kb = K / kKBlock;
  std::mt19937_64 rng(seed);
  std::normal_distribution<float> normal(0.0f, 1.0f);
  const float inv_sqrt_k = 1.0f / std::sqrt(static_cast<float>(K));
  std::vector<float> row(static_cast<size_t>(K));
  for (int m = 0; m < rows; ++m) {
    for (int k = 0; k < K; ++k) row[k] = static_cast<float>(normal(rng) * inv_sqrt_k);
    for (int kbi = 0; kbi < kb; ++kbi) {
      float amax = 0.0f;
      for (int c = 0; c < 128; ++c) amax = std::max(amax, std::abs(row[kbi * 128 + c]));
      const float scale = std::max(amax, kQuantEps) / kFp8Max;
      scales[static_cast<size_t>(m) * kb + kbi] = scale;
      uint8_t* dst = act + static_cast<size_t>(m) * K + static_cast<size_t>(kbi) * 128;
      for (int c = 0; c < 128; ++c) dst[c] = quant(row[kbi * 128 + c], scale);
    }
  }
}

// The block quantisation of make_activation (bench/bench_decode.cu:459-467)
// applied to given fp32 rows (row stride ldx): per row and 128-column block,
// amax = max |v| (std::max order), scale = max(amax, 1e-4) / 448,
// q = e4m3(clamp(v / scale, +-448)).  The GPU activation quantiser is checked
// against it.
void orc_quantize_rows(int rows, int K, const float* x, int ldx, uint8_t* q, float* scales) {
  const int kb = K / kKBlock;
  for (int m = 0; m < rows; ++m) {
    const float* row = x + static_cast<size_t>(m) * ldx;
    for (int kbi = 0; kbi < kb; ++kbi) {
      float amax = 0.0f;
      for (int c = 0; c < 128; ++c) amax = std::max(amax, std::abs(row[kbi * 128 + c]));
      const float scale = std::max(amax, kQuantEps) / kFp8Max;
      scales[static_cast<size_t>(m) * kb + kbi] = scale;
      uint8_t* dst = q + static_cast<size_t>(m) * K + static_cast<size_t>(kbi) * 128;
      for (int c = 0; c < 128; ++c) dst[c] = quant(row[kbi * 128 + c], scale);
    }
  }
}

// Per-tensor-scaled inputs (the BASELINE configs' data mode; the reference
// has no generator for it).  rows x K values ~ N(0,1); one fp32 scale
// s = amax/448 for the whole tensor; q = clamp(v/s, +-448) -> e4m3.  Every
// entry of the block-scale array (scale_rows x K/128) is set to s, so the
// block-scale kernel computes the per-tensor GEMM exactly.  Each 128-row block
// draws from its own mt19937_64 seeded with splitmix64(seed ^ block), so the
// result does not depend on `threads`.  Returns s.
float orc_gen_pertensor(int rows, int K, uint64_t seed, uint8_t* out, float* scales,
                        int scale_rows, int threads) {
  const int nblocks = (rows + 127) / 128;
  if (threads < 1) threads = 1;
  std::vector<float> block_amax(static_cast<size_t>(nblocks), 0.0f);
  auto draw_block = [&](int b, float* dst_vals) {
    std::mt19937_64 rng(splitmix64(seed ^ static_cast<uint64_t>(b)));
    std::normal_distribution<float> normal(0.0f, 1.0f);
    const int r_end = std::min(rows, (b + 1) * 128);
    const size_t count = static_cast<size_t>(r_end - b * 128) * K;
    for (size_t i = 0; i < count; ++i) dst_vals[i] = normal(rng);
    return count;
  };
  // Pass 1: amax per block (values regenerated in pass 2 to bound memory).
  auto pass1 = [&](int t) {
    std::vector<float> vals(static_cast<size_t>(128) * K);
    for (int b = t; b < nblocks; b += threads) {
      const size_t count = draw_block(b, vals.data());
      float a = 0.0f;
      for (size_t i = 0; i < count; ++i) a = std::max(a, std::fabs(vals[i]));
      block_amax[b] = a;
    }
  };
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) pool.emplace_back(pass1, t);
  for (auto& th : pool) th.join();
  pool.clear();
  float amax = 0.0f;
  for (float a : block_amax) amax = std::max(amax, a);
  const float scale = std::max(amax, kQuantEps) / kFp8Max;
  auto pass2 = [&](int t) {
    std::vector<float> vals(static_cast<size_t>(128) * K);
    for (int b = t; b < nblocks; b += threads) {
      const size_t count = draw_block(b, vals.data());
      uint8_t* dst = out + static_cast<size_t>(b) * 128 * K;
      for (size_t i = 0; i < count; ++i) dst[i] = quant(vals[i], scale);
    }
  };
  for (int t = 0; t < threads; ++t) pool.emplace_back(pass2, t);
  for (auto& th : pool) th.join();
  const size_t n_scales = static_cast<size_t>(scale_rows) * (K / kKBlock);
  for (size_t i = 0; i < n_scales; ++i) scales[i] = scale;
  return scale;
}

// Restates kernels/smoke_test.cu:173-207 (compute_reference) on output rows
// [n_begin, n_end): per k_block, dequantise through the LUT, four strided
// partial sums combined as (r0+r1)+(r2+r3), then
// acc = fma(w_scale*a_scale, raw, acc); finally every output is rounded to
// bf16.  out: [M,N] fp32 (bf16-representable values).
static void reference_rows(int M, int N, int K, const uint8_t* act, const float* a_scales,
                           const uint8_t* weight, const float* w_scales, float* out,
                           int n_begin, int n_end) {
  init_lut();
  const int kb_count = K / kKBlock;
  for (int m = 0; m < M; ++m)
    for (int n = n_begin; n < n_end; ++n) out[static_cast<size_t>(m) * N + n] = 0.0f;
  std::vector<float> w_row(kKBlock);
  std::vector<float> act_block(static_cast<size_t>(M) * kKBlock);
  for (int kb = 0; kb < kb_count; ++kb) {
    for (int m = 0; m < M; ++m) {
      const uint8_t* a = act + static_cast<size_t>(m) * K + static_cast<size_t>(kb) * kKBlock;
      float* dst = &act_block[static_cast<size_t>(m) * kKBlock];
      for (int j = 0; j < kKBlock; ++j) dst[j] = g_lut[a[j]];
    }
    for (int n = n_begin; n < n_end; ++n) {
      const uint8_t* w = weight + static_cast<size_t>(n) * K + static_cast<size_t>(kb) * kKBlock;
      for (int j = 0; j < kKBlock; ++j) w_row[j] = g_lut[w[j]];
      const float ws = w_scales[static_cast<size_t>(n / kKBlock) * kb_count + kb];
      for (int m = 0; m < M; ++m) {
        const float* a = &act_block[static_cast<size_t>(m) * kKBlock];
        float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
        for (int j = 0; j < kKBlock; j += 4) {
          r0 += w_row[j] * a[j];
          r1 += w_row[j + 1] * a[j + 1];
          r2 += w_row[j + 2] * a[j + 2];
          r3 += w_row[j + 3] * a[j + 3];
        }
        const float raw = (r0 + r1) + (r2 + r3);
        const float combined = ws * a_scales[static_cast<size_t>(m) * kb_count + kb];
        float* acc = &out[static_cast<size_t>(m) * N + n];
        *acc = std::fma(combined, raw, *acc);
      }
    }
  }
  for (int m = 0; m < M; ++m)
    for (int n = n_begin; n < n_end; ++n) {
      float& v = out[static_cast<size_t>(m) * N + n];
      v = bf16_round(v);
    }
}

void orc_compute_reference(int M, int N, int K, const uint8_t* act, const float* a_scales,
                           const uint8_t* weight, const float* w_scales, float* out) {
  reference_rows(M, N, K, act, a_scales, weight, w_scales, out, 0, N);
}

// Same arithmetic, output rows split over `threads` workers.  Every output
// element is computed by exactly the code above, so the result is
// bit-identical to orc_compute_reference for any thread count.
void orc_compute_reference_mt(int M, int N, int K, const uint8_t* act, const float* a_scales,
                              const uint8_t* weight, const float* w_scales, float* out,
                              int threads) {
  init_lut();
  if (threads <= 1 || N < 2) {
    reference_rows(M, N, K, act, a_scales, weight, w_scales, out, 0, N);
    return;
  }
  threads = std::min(threads, N);
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    const int b = static_cast<int>(static_cast<int64_t>(N) * t / threads);
    const int e = static_cast<int>(static_cast<int64_t>(N) * (t + 1) / threads);
    pool.emplace_back(reference_rows, M, N, K, act, a_scales, weight, w_scales, out, b, e);
  }
  for (auto& th : pool) th.join();
}

// Restates kernels/weight_prepack.cuh:13-19,55-97: packed[((tile*KB + kb)*BM
// + row)*128 + k%128] = W[tile*BM + row][k], rows >= N zero.  dst holds
// ceil(N/BM)*BM*K bytes.
void orc_prepack(const uint8_t* src, uint8_t* dst, int N, int K, int BM) {
  const int tiles = (N + BM - 1) / BM;
  const int kb_count = K / kKBlock;
  for (int t = 0; t < tiles; ++t)
    for (int kb = 0; kb < kb_count; ++kb)
      for (int r = 0; r < BM; ++r) {
        uint8_t* d = dst + ((static_cast<size_t>(t) * kb_count + kb) * BM + r) * kKBlock;
        const int n = t * BM + r;
        if (n < N)
          std::memcpy(d, src + static_cast<size_t>(n) * K + static_cast<size_t>(kb) * kKBlock,
                      kKBlock);
        else
          std::memset(d, 0, kKBlock);
      }
}

// The B200 descriptor-ready layout (no reference counterpart): the same
// [tile][kb][row][128] order as orc_prepack, but inside every 1024-byte group
// of 8 rows the 16-byte chunk c of row r is stored at chunk (c ^ (r % 8)) --
// the 128-byte swizzle that tcgen05 K-major SWIZZLE_128B operands use -- so a
// plain bulk copy lands bytes exactly where the MMA descriptor reads them.
void orc_prepack_swizzled(const uint8_t* src, uint8_t* dst, int N, int K, int BM) {
  const int tiles = (N + BM - 1) / BM;
  const int kb_count = K / kKBlock;
  for (int t = 0; t < tiles; ++t)
    for (int kb = 0; kb < kb_count; ++kb)
      for (int r = 0; r < BM; ++r) {
        uint8_t* d = dst + ((static_cast<size_t>(t) * kb_count + kb) * BM + r) * kKBlock;
        const int n = t * BM + r;
        for (int c = 0; c < 8; ++c) {
          uint8_t* dc = d + ((c ^ (r & 7)) * 16);
          if (n < N)
            std::memcpy(dc, src + static_cast<size_t>(n) * K + static_cast<size_t>(kb) * kKBlock +
                                c * 16,
                        16);
          else
            std::memset(dc, 0, 16);
        }
      }
}

}  // extern "C"
