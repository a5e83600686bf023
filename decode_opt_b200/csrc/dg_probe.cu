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
//   dg_probe_mma          tcgen05.mma cost: 1-4 warps each issue a run of
//                         kind::f8f6f4 MMAs of one shape (zeroed smem
//                         operands) round-robin over their own TMEM
//                         accumulators, clock64 around the issue loops and
//                         until every MMA has completed (tcgen05.commit ->
//                         mbarrier): the per-instruction cost of one issuing
//                         thread against the tensor pipe's throughput.
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

// `issuers` warps (lane 0 of warps 0..issuers-1) issue MMAs concurrently, each
// round-robin over its own `accumulators` TMEM accumulators (every MMA of a
// run of four into one accumulator depends on the previous one; different
// accumulators are independent), with the smem descriptors computed before
// the timed loop.  Per CTA: out[2c] = cycles until the slowest issuer has
// issued, out[2c+1] = cycles until every issued MMA has completed (each
// issuer commits to its own mbarrier), both from one common clock64 start.
__global__ void __launch_bounds__(kMmaProbeThreads, 1)
    mma_cost_kernel(int mma_m, int mma_n, int iters, int accumulators, int issuers, long long* out,
                    int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023u) & ~uintptr_t(1023));
  uint8_t* a_tile = smem;                 // 128 rows x 128 B, SWIZZLE_128B K-major
  uint8_t* b_tile = smem + 16384;         // 256 rows x 128 B
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 16384 + 32768);   // [4]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 4);
  long long* t_issue = reinterpret_cast<long long*>(bar + 6);          // [4]
  __shared__ long long t_start;
  for (int i = threadIdx.x; i < (16384 + 32768) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  fence_proxy_async_shared();             // zero fill -> tensor-core operand reads
  if (threadIdx.x == 0) {
    for (int w = 0; w < 4; ++w) {
      mbar_init(&bar[w], 1);
      t_issue[w] = -1;
    }
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
  const int warp = threadIdx.x / 32;
  const bool issuer = (threadIdx.x & 31) == 0 && warp < issuers;
  const uint32_t idesc = make_idesc_e4m3_f32(static_cast<uint32_t>(mma_m), static_cast<uint32_t>(mma_n));
  const uint32_t a0 = smem_addr(a_tile);
  const uint32_t b0 = smem_addr(b_tile);
  uint64_t adesc[4], bdesc[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    adesc[k] = make_desc_k_sw128(a0 + 32u * k);
    bdesc[k] = make_desc_k_sw128(b0 + 32u * k);
  }
  const uint32_t d0 = tmem_base + static_cast<uint32_t>(warp * accumulators * mma_n);
  bool ok = true;
  if (issuer) {   // warm-up: the first MMAs of each issuer, completed before timing
    for (int i = 0; i < 8; ++i) mma_f8f6f4(d0, adesc[i & 3], bdesc[i & 3], idesc, 0u);
    mma_commit(&bar[warp]);
    ok = probe_wait(&bar[warp], 0u, status, 0x93);
  }
  __syncthreads();
  if (threadIdx.x == 0) t_start = clock64();
  __syncthreads();
  const int mine = iters / issuers;
  if (issuer && ok) {
    int r = 0, run = 0;
    for (int i = 0; i < mine; ++i) {
      mma_f8f6f4(d0 + static_cast<uint32_t>(r * mma_n), adesc[i & 3], bdesc[i & 3], idesc, run != 0 ? 1u : 0u);
      if (++r == accumulators) {
        r = 0;
        run = (run + 1) & 3;
      }
    }
    const long long t = clock64();
    mma_commit(&bar[warp]);
    t_issue[warp] = probe_wait(&bar[warp], 1u, status, 0x93) ? t : -1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long done = clock64() - t_start;
    long long issue = 0;
    for (int w = 0; w < issuers; ++w) {
      if (t_issue[w] < 0) issue = -1;
      if (issue >= 0 && t_issue[w] - t_start > issue) issue = t_issue[w] - t_start;
    }
    out[2 * blockIdx.x] = issue;
    out[2 * blockIdx.x + 1] = issue >= 0 ? done : -1;
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
int dg_probe_mma(int mma_m, int mma_n, int iters, int accumulators, int issuers, int ctas, long long* out,
                 int* status, void* stream) {
  const int n_step = mma_m == 64 ? 8 : 16;
  if (out == nullptr || !(mma_m == 64 || mma_m == 128) || mma_n < n_step || mma_n > 256 || mma_n % n_step != 0 ||
      issuers < 1 || issuers > 4 || accumulators < 1 || issuers * accumulators * mma_n > 512 ||
      iters < issuers || ctas < 1 || ctas > sm_count())
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(mma_cost_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(kMmaProbeSmem));
  if (e != cudaSuccess) return e;
  mma_cost_kernel<<<ctas, kMmaProbeThreads, kMmaProbeSmem, static_cast<cudaStream_t>(stream)>>>(
      mma_m, mma_n, iters, accumulators, issuers, out, status);
  return cudaGetLastError();
}

}  // extern "C"
