// SPDX-License-Identifier: MIT
//
// weight_prepack.cuh -- the reference's `decode_gemm::prepack` interface
// (kernels/weight_prepack.cuh:45-120 of the reference) over the library's C
// ABI: raw [N, K] e4m3 weights -> the tile-contiguous layout
// [tile][k_block][OutputRowsPerCta rows][128 bytes], rows >= N zero.
// OutputTilesPerCta does not change the layout (as in the reference).

#pragma once

#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "decode_gemm_b200.h"

namespace decode_gemm {
namespace prepack {

// Layout constants of the reference's prepack namespace: one 128-byte K block
// per packed row, moved as 16-byte vectors.
inline constexpr uint32_t kKBlock = 128;
inline constexpr uint32_t kBytesPerUint4 = 16;
inline constexpr uint32_t kUint4PerKBlock = kKBlock / kBytesPerUint4;

inline int padded_n(int n, int output_rows_per_cta) {
  return ((n + output_rows_per_cta - 1) / output_rows_per_cta) * output_rows_per_cta;
}

inline size_t packed_weight_bytes(int n, int k, int output_rows_per_cta) {
  return static_cast<size_t>(padded_n(n, output_rows_per_cta)) * static_cast<size_t>(k);
}

// Returns cudaErrorInvalidValue when K is not a multiple of 128.
template <int OutputRowsPerCta, int OutputTilesPerCta = 1>
inline cudaError_t launch_prepack_weight(const __nv_fp8_e4m3* source, __nv_fp8_e4m3* destination, int n, int k,
                                         cudaStream_t stream = nullptr) {
  static_assert(OutputRowsPerCta > 0 && OutputRowsPerCta % 8 == 0,
                "OutputRowsPerCta must be a positive multiple of 8");
  static_assert(OutputTilesPerCta > 0, "OutputTilesPerCta must be positive");
  if (k % 128 != 0) return cudaErrorInvalidValue;
  return static_cast<cudaError_t>(
      dg_prepack_weight(source, destination, n, k, OutputRowsPerCta, DG_LAYOUT_PACKED, stream));
}

}  // namespace prepack
}  // namespace decode_gemm
