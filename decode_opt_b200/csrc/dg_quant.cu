// SPDX-License-Identifier: MIT
//
// dg_quant.cu -- the activation quantiser of the decode GEMM's input:
// bf16 rows [M, K] (row stride ldx, e.g. the previous layer's gathered
// output) -> e4m3 [M, K] plus fp32 block scales [M, K/128].
//
// It is the block quantisation the reference does on the host
// (bench/bench_decode.cu:459-467, inside make_activation): for every row and
// 128-column block, amax = max |v|, scale = max(amax, 1e-4) / 448,
// q = e4m3(clamp(v / scale, +-448)) rounded to nearest even.  One warp per
// (row, block): each lane loads 4 consecutive bf16 (8 bytes), the warp
// reduces the block's amax with shuffles, and each lane stores its 4 bytes;
// lane 0 stores the scale.  The comparisons follow the reference's
// std::max / std::min order and the division is the IEEE one, so the bytes
// and scales equal the oracle's for finite inputs.
//
// Under programmatic dependent launch the kernel releases its dependents at
// once (the next GEMM may prefetch its weights) and waits for the grid that
// produced its input before reading it.
//
// dg_copy_from_host is the same pattern for a request's input: a copy of
// pinned host memory (through its device address) into device memory done
// by GPU loads, so that it sits between two GEMMs as a kernel with
// programmatic dependent launch instead of a copy node (which a graph orders
// after the preceding GEMM's completion and before the next GEMM's launch).

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "decode_gemm_b200.h"
#include "sm100.cuh"

namespace {

constexpr int kQuantThreads = 256;
constexpr float kFp8Max = 448.0f;
constexpr float kQuantEps = 1.0e-4f;

__device__ __forceinline__ float max_ref(float a, float b) { return a < b ? b : a; }   // std::max
__device__ __forceinline__ float min_ref(float a, float b) { return b < a ? b : a; }   // std::min

__global__ void __launch_bounds__(kQuantThreads)
    quantize_act_kernel(const __nv_bfloat16* __restrict__ x, int ldx, int M, int K, uint8_t* __restrict__ q,
                        float* __restrict__ scales, int vec) {
  dg::sm100::griddep_launch_dependents();
  dg::sm100::griddep_wait();
  const int kb = K / 128;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (warp >= static_cast<long long>(M) * kb) return;
  const int m = static_cast<int>(warp / kb);
  const int b = static_cast<int>(warp - static_cast<long long>(m) * kb);
  const __nv_bfloat16* src = x + static_cast<size_t>(m) * ldx + static_cast<size_t>(b) * 128 + lane * 4;
  float v[4];
  if (vec) {
    const uint2 raw = *reinterpret_cast<const uint2*>(src);
    const __nv_bfloat162 lo = *reinterpret_cast<const __nv_bfloat162*>(&raw.x);
    const __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&raw.y);
    v[0] = __low2float(lo);
    v[1] = __high2float(lo);
    v[2] = __low2float(hi);
    v[3] = __high2float(hi);
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __bfloat162float(src[j]);
  }
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) amax = max_ref(amax, fabsf(v[j]));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = max_ref(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float scale = max_ref(amax, kQuantEps) / kFp8Max;
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float c = min_ref(max_ref(v[j] / scale, -kFp8Max), kFp8Max);
    packed |= static_cast<uint32_t>(__nv_fp8_e4m3(c).__x) << (8 * j);
  }
  uint8_t* dst = q + static_cast<size_t>(m) * K + static_cast<size_t>(b) * 128 + lane * 4;
  *reinterpret_cast<uint32_t*>(dst) = packed;
  if (lane == 0) scales[static_cast<size_t>(m) * kb + b] = scale;
}

constexpr int kCopyThreads = 256;
constexpr unsigned kCopyMaxBlocks = 592;   // 4 per SM on a 148-SM part

// dst[0, bytes) = src[0, bytes), src in mapped pinned host memory.  Loads are
// volatile (ld.global.cv): every launch reads the host's current bytes over
// PCIe, nothing cached from an earlier launch.  vec: both pointers 16-byte
// aligned (16-byte loads and stores, then the tail byte by byte).
__global__ void __launch_bounds__(kCopyThreads)
    copy_from_host_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, unsigned long long bytes,
                          int vec) {
  dg::sm100::griddep_launch_dependents();
  dg::sm100::griddep_wait();
  const unsigned long long tid = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const unsigned long long stride = static_cast<unsigned long long>(gridDim.x) * blockDim.x;
  unsigned long long done = 0;
  if (vec) {
    const unsigned long long n16 = bytes / 16;
    for (unsigned long long i = tid; i < n16; i += stride)
      reinterpret_cast<uint4*>(dst)[i] = __ldcv(reinterpret_cast<const uint4*>(src) + i);
    done = n16 * 16;
  }
  for (unsigned long long i = done + tid; i < bytes; i += stride) dst[i] = __ldcv(src + i);
}

}  // namespace

extern "C" {

int dg_copy_from_host(void* dst, const void* src, unsigned long long bytes, void* stream, int pdl_attr) {
  if (dst == nullptr || src == nullptr || bytes == 0) return cudaErrorInvalidValue;
  const int vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15u) == 0 ? 1 : 0;
  const unsigned long long units = vec ? (bytes + 15) / 16 : bytes;
  unsigned long long blocks = (units + kCopyThreads - 1) / kCopyThreads;
  if (blocks > kCopyMaxBlocks) blocks = kCopyMaxBlocks;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1]{};
  cfg.gridDim = dim3(static_cast<unsigned>(blocks), 1, 1);
  cfg.blockDim = dim3(kCopyThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (pdl_attr) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, copy_from_host_kernel, static_cast<uint8_t*>(dst),
                            static_cast<const uint8_t*>(src), bytes, vec);
}

int dg_quantize_act(const void* x, int ldx, int M, int K, void* q, float* scales, void* stream, int pdl_attr) {
  if (x == nullptr || q == nullptr || scales == nullptr || M < 1 || K < 128 || K % 128 != 0 || ldx < K)
    return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(q) & 3u) != 0) return cudaErrorInvalidValue;
  const int vec = ((reinterpret_cast<uintptr_t>(x) & 7u) == 0 && (ldx & 3) == 0) ? 1 : 0;
  const long long warps = static_cast<long long>(M) * (K / 128);
  const unsigned blocks = static_cast<unsigned>((warps * 32 + kQuantThreads - 1) / kQuantThreads);
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1]{};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(kQuantThreads, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 0;
  if (pdl_attr) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, quantize_act_kernel, static_cast<const __nv_bfloat16*>(x), ldx, M, K,
                            static_cast<uint8_t*>(q), scales, vec);
}

}  // extern "C"
