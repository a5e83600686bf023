// SPDX-License-Identifier: MIT
//
// dg_probe.cu -- achievable-HBM-read probe for sm_100a (the B200 rebuild of
// the reference's tools/peak_bw_probe.cu:82-211): it measures the denominator
// of "% of achievable bandwidth" for the decode GEMM.
//
//   dg_probe_bulk_stream  every CTA streams a contiguous slice of a cold
//                         buffer through an smem ring with cp.async.bulk
//                         (op_bytes per copy, `stages` in flight), the same
//                         copy engine and mbarrier handshake as the GEMM's
//                         producer, with no math behind it;
//   dg_probe_naive_read   grid-stride 16-byte ld.global.nc loads with 4
//                         independent loads in flight per thread (the
//                         reference's naive_read_nc control);
//
// The L2 honesty check (reference tma_l2_selftest, :190-211) is
// dg_probe_bulk_stream run repeatedly over a buffer small enough to stay in
// L2: it must read far above HBM speed, which shows the cold-buffer numbers
// are not L2 hits.
//
//   dg_probe_mma          tcgen05.mma cost: one thread issues a run of
//                         kind::f8f6f4 MMAs of one shape (zeroed smem
//                         operands) round-robin over TMEM accumulators and
//                         reads clock64 around the issue loop and around the
//                         completion (tcgen05.commit -> mbarrier).  It is the
//                         measurement behind the GEMM's operand placement.
//
// Timing of the two HBM probes is the caller's (CUDA events around the
// launch).  Every wait is bounded; a timeout is reported through *status
// (0x91 producer, 0x92 consumer, 0x93 MMA completion).

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "decode_gemm_b200.h"
#include "sm100.cuh"

namespace {

using namespace dg::sm100;

constexpr int kProbeThreads = 64;   // warp 0 issues, warp 1 consumes
constexpr uint64_t kProbeTimeoutNs = 2000000000ull;

__global__ void __launch_bounds__(kProbeThreads, 1)
    bulk_stream_kernel(const uint8_t* __restrict__ src, unsigned long long bytes, uint32_t op_bytes,
                       int stages, int* status, unsigned long long* sink) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127u) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * op_bytes);
  uint64_t* empty = full + stages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + stages);
  const unsigned long long ops_total = bytes / op_bytes;
  const unsigned long long op_begin = ops_total * blockIdx.x / gridDim.x;
  const unsigned long long op_end = ops_total * (blockIdx.x + 1) / gridDim.x;
  const int n = static_cast<int>(op_end - op_begin);
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const uint64_t pol = policy_evict_first();
  int issued = 0;
  if (threadIdx.x == 0) {
    for (int i = 0; i < n; ++i) {
      const int s = i % stages;
      if (i >= stages && !mbar_wait_bounded(&empty[s], static_cast<uint32_t>(((i / stages) & 1) ^ 1), abort_flag,
                                            status, 0x91, kProbeTimeoutNs))
        break;
      mbar_arrive_expect_tx(&full[s], op_bytes);
      bulk_load(smem + static_cast<size_t>(s) * op_bytes, src + (op_begin + i) * op_bytes, op_bytes, &full[s], pol);
      issued = i + 1;
    }
  } else if (threadIdx.x == 32) {
    uint32_t acc = 0;
    for (int i = 0; i < n; ++i) {
      const int s = i % stages;
      if (!mbar_wait_bounded(&full[s], static_cast<uint32_t>((i / stages) & 1), abort_flag, status, 0x92,
                             kProbeTimeoutNs))
        break;
      acc ^= *reinterpret_cast<const volatile uint32_t*>(smem + static_cast<size_t>(s) * op_bytes);
      mbar_arrive(&empty[s]);
    }
    if (acc == 0x9e3779b9u) atomicAdd(sink, 1ull);   // keeps the consumer's reads live
  }
  __syncthreads();
  if (threadIdx.x == 0 && *abort_flag != 0) {
    const int lo = issued > stages ? issued - stages : 0;
    for (int i = lo; i < issued; ++i) {
      const int s = i % stages;
      const uint32_t parity = static_cast<uint32_t>((i / stages) & 1);
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&full[s], parity) && global_timer_ns() - t0 < kProbeTimeoutNs) {
      }
    }
  }
}

__global__ void naive_read_kernel(const uint4* __restrict__ src, size_t n16, unsigned long long* sink) {
  uint32_t acc = 0;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n16; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4* p = src + i + j * stride;
      asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                   : "=r"(v[j].x), "=r"(v[j].y), "=r"(v[j].z), "=r"(v[j].w)
                   : "l"(p));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) acc ^= v[j].x ^ v[j].y ^ v[j].z ^ v[j].w;
  }
  for (; i < n16; i += stride) {
    const uint4 v = src[i];
    acc ^= v.x ^ v.y ^ v.z ^ v.w;
  }
  if (acc == 0x9e3779b9u) atomicAdd(sink, 1ull);
}

constexpr int kMmaProbeThreads = 128;
constexpr uint32_t kMmaProbeSmem = 120u * 1024u;   // > half the SM: one CTA (and one TMEM owner) per SM

// Bounded wait on `bar` completing the phase of `parity`; false (status set)
// after kProbeTimeoutNs.
__device__ bool probe_wait(uint64_t* bar, uint32_t parity, int* status, int code) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kProbeTimeoutNs) {
      if (status != nullptr) atomicCAS(status, 0, code);
      return false;
    }
  }
  return true;
}

__global__ void __launch_bounds__(kMmaProbeThreads, 1)
    mma_cost_kernel(int mma_m, int mma_n, int iters, int accumulators, long long* out, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;                 // 128 rows x 128 B, SWIZZLE_128B K-major
  uint8_t* b_tile = smem + 16384;         // 256 rows x 128 B
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 16384 + 32768);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  for (int i = threadIdx.x; i < (16384 + 32768) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_shared();             // zero fill -> tensor-core operand reads
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  if (threadIdx.x < 32) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t idesc = make_idesc_e4m3_f32(static_cast<uint32_t>(mma_m), static_cast<uint32_t>(mma_n));
    const uint32_t a0 = smem_addr(a_tile);
    const uint32_t b0 = smem_addr(b_tile);
    for (int i = 0; i < 8; ++i) mma_f8f6f4(tmem_base, make_desc_k_sw128(a0), make_desc_k_sw128(b0), idesc, 0u);
    mma_commit(bar);
    long long issue = -1, done = -1;
    if (probe_wait(bar, 0u, status, 0x93)) {
      const long long t0 = clock64();
      for (int i = 0; i < iters; ++i) {
        const int r = i % accumulators;
        const uint32_t d = tmem_base + static_cast<uint32_t>(r * mma_n);
        const uint32_t k = 32u * static_cast<uint32_t>(i & 3);
        mma_f8f6f4(d, make_desc_k_sw128(a0 + k), make_desc_k_sw128(b0 + k), idesc, ((i / accumulators) & 3) != 0 ? 1u : 0u);
      }
      const long long t1 = clock64();
      mma_commit(bar);
      if (probe_wait(bar, 1u, status, 0x93)) {
        issue = t1 - t0;
        done = clock64() - t0;
      }
    }
    out[2 * blockIdx.x] = issue;
    out[2 * blockIdx.x + 1] = done;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tmem_base, 512);
}

int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 148;
  return sms;
}

}  // namespace

extern "C" {

// Streams `bytes` (a multiple of op_bytes; op_bytes a multiple of 16) of the
// device buffer once.  `sink` is one device uint64 (may be NULL-free scratch).
int dg_probe_bulk_stream(const void* buf, unsigned long long bytes, unsigned op_bytes, int ctas, int stages,
                         int* status, unsigned long long* sink, void* stream) {
  if (buf == nullptr || sink == nullptr || op_bytes < 16 || op_bytes % 16 != 0 || stages < 1 || ctas < 1 ||
      bytes < op_bytes || (reinterpret_cast<uintptr_t>(buf) & 15u) != 0)
    return cudaErrorInvalidValue;
  const size_t smem = 128 + static_cast<size_t>(stages) * op_bytes + 16 * static_cast<size_t>(stages) + 16;
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(bulk_stream_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  bulk_stream_kernel<<<ctas, kProbeThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(buf), bytes, op_bytes, stages, status, sink);
  return cudaGetLastError();
}

int dg_probe_naive_read(const void* buf, unsigned long long bytes, int blocks_per_sm, unsigned long long* sink,
                        void* stream) {
  if (buf == nullptr || sink == nullptr || bytes < 16 || blocks_per_sm < 1) return cudaErrorInvalidValue;
  naive_read_kernel<<<sm_count() * blocks_per_sm, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(buf), static_cast<size_t>(bytes / 16), sink);
  return cudaGetLastError();
}

int dg_num_sms(void) { return sm_count(); }

// out: 2 * ctas long longs (issue cycles, completion cycles per CTA; -1 after
// a timeout).
int dg_probe_mma(int mma_m, int mma_n, int iters, int accumulators, int ctas, long long* out, int* status,
                 void* stream) {
  const int n_step = mma_m == 64 ? 8 : 16;
  if (out == nullptr || !(mma_m == 64 || mma_m == 128) || mma_n < n_step || mma_n > 256 || mma_n % n_step != 0 ||
      accumulators < 1 || accumulators * mma_n > 512 || iters < 1 || ctas < 1 || ctas > sm_count())
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(mma_cost_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kMmaProbeSmem));
  if (e != cudaSuccess) return e;
  mma_cost_kernel<<<ctas, kMmaProbeThreads, kMmaProbeSmem, static_cast<cudaStream_t>(stream)>>>(
      mma_m, mma_n, iters, accumulators, out, status);
  return cudaGetLastError();
}

}  // extern "C"
