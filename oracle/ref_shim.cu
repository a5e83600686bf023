// SPDX-License-Identifier: MIT
//
// oracle/ref_shim.cu -- TEST INFRASTRUCTURE ONLY.  Builds the reference
// repository's own host-side generator and scalar oracle
// (kernels/smoke_test.cu: init_fp8_lut :60-69, generate_weight :102-140,
// generate_activation :142-168, compute_reference :173-207) from the source
// file where it lies, into oracle/_ref/libref_oracle.so, so that the CPU
// restatement in oracle/oracle.cpp can be checked bit-for-bit against the
// reference itself.  Nothing here is copied: the reference file is #included
// by path at build time (oracle/Makefile passes REF_SMOKE) and its GPU parts
// are never executed.
//
// generate_weight ends by uploading to the device (cudaMalloc/cudaMemcpy).
// This container and the CPU tests have no GPU, so those two calls are routed
// to host malloc/memcpy for the included file only.  The reference's SM90
// kernels are compiled (PTX only, never launched); the three CUDA-driver
// symbols its tensor-map helpers reference are stubbed so the library loads
// without libcuda.

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <cstring>

static cudaError_t ref_host_malloc(void** p, size_t n) {
  *p = std::malloc(n == 0 ? 1 : n);
  return *p ? cudaSuccess : cudaErrorMemoryAllocation;
}
static cudaError_t ref_host_memcpy(void* d, const void* s, size_t n, cudaMemcpyKind) {
  std::memcpy(d, s, n);
  return cudaSuccess;
}

#define cudaMalloc(p, n) ref_host_malloc(reinterpret_cast<void**>(p), (n))
#define cudaMemcpy(d, s, n, k) ref_host_memcpy((d), (s), (n), (k))
#define main reference_smoke_main
#include REF_SMOKE
#undef main
#undef cudaMalloc
#undef cudaMemcpy

extern "C" {

CUresult cuTensorMapEncodeTiled(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                CUtensorMapL2promotion, CUtensorMapFloatOOBfill) {
  return CUDA_ERROR_NOT_SUPPORTED;
}
CUresult cuGetErrorName(CUresult, const char** s) {
  *s = "stub";
  return CUDA_SUCCESS;
}
CUresult cuGetErrorString(CUresult, const char** s) {
  *s = "stub";
  return CUDA_SUCCESS;
}

// Reference generate_weight; weight [N,K] bytes, scales [ceil(N/128), K/128].
void ref_gen_weight(int N, int K, uint64_t seed, uint8_t* weight, float* scales) {
  init_fp8_lut();
  ShapeData sd;
  sd.N = N;
  sd.K = K;
  sd.num_scale_rows = (N + 127) / 128;
  generate_weight(&sd, seed);
  std::memcpy(weight, sd.weight.data(), sd.weight.size());
  std::memcpy(scales, sd.w_scales.data(), sd.w_scales.size() * sizeof(float));
  std::free(sd.d_weight_raw);
  std::free(sd.d_w_scales);
}

// Reference generate_activation (seed already mixed by the caller).
void ref_gen_activation(int M, int K, uint64_t seed, uint8_t* act, float* scales) {
  init_fp8_lut();
  ShapeData sd;
  sd.K = K;
  MData md;
  md.M = M;
  generate_activation(&md, sd, seed);
  std::memcpy(act, md.act.data(), md.act.size());
  std::memcpy(scales, md.a_scales.data(), md.a_scales.size() * sizeof(float));
}

// Reference compute_reference on caller-provided inputs, rows [0, N).
void ref_compute_reference(int M, int N, int K, const uint8_t* act, const float* a_scales,
                           const uint8_t* weight, const float* w_scales, float* out) {
  init_fp8_lut();
  ShapeData sd;
  sd.N = N;
  sd.K = K;
  sd.num_scale_rows = (N + 127) / 128;
  sd.weight.assign(weight, weight + static_cast<size_t>(N) * K);
  sd.w_scales.assign(w_scales, w_scales + static_cast<size_t>(sd.num_scale_rows) * (K / 128));
  MData md;
  md.M = M;
  md.act.assign(act, act + static_cast<size_t>(M) * K);
  md.a_scales.assign(a_scales, a_scales + static_cast<size_t>(M) * (K / 128));
  compute_reference(md, sd);
  std::memcpy(out, md.reference.data(), md.reference.size() * sizeof(float));
}

}  // extern "C"
