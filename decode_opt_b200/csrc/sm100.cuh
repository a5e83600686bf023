// SPDX-License-Identifier: MIT
//
// sm100.cuh -- the sm_100a primitive layer of the B200 decode GEMM.
//
// Replaces the reference's SM90 wrapper header (kernels/sm90_compat.cuh:23-132:
// wgmma fence/commit/wait, GMMA smem descriptors, ld/st.shared, 2-D TMA) with
// the Blackwell equivalents, written directly as inline PTX:
//
//   * mbarrier init / arrive / arrive.expect_tx / try_wait.parity, and a
//     BOUNDED wait that gives up after a %globaltimer deadline or when the CTA
//     has raised its abort flag (no wait in this kernel can hang a GPU);
//   * TMA tiled loads (3-D, 4-D) and the untiled bulk copy, both completing on
//     an mbarrier transaction count, with an L2 cache-policy hint;
//   * tcgen05: TMEM alloc / relinquish / dealloc, the kind::f8f6f4 MMA with A
//     and B from shared memory, tcgen05.commit -> mbarrier, tcgen05.ld
//     (32x32b shape), wait::ld and the thread-sync fences;
//   * the UMMA shared-memory descriptor (K-major, SWIZZLE_128B) and the
//     instruction descriptor for e4m3 x e4m3 -> f32;
//   * programmatic dependent launch (griddepcontrol.wait / launch_dependents).
//
// Every copy here lands in the issuing CTA's own shared memory only.

#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace dg {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

// Makes barrier initialisation visible to the async proxy (TMA, tcgen05).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0u;
}

// Bounded wait for the phase of `bar` with the given parity to complete.
// Returns false -- without waiting further -- once *abort is set, or after
// `timeout_ns` of %globaltimer time, in which case it raises *abort and
// records `code` in *status (first error wins).  Every wait in the decode
// kernel goes through here.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort, int* status, int code,
                                                  uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (*abort != 0) return false;
    if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - start > timeout_ns) {
      *abort = 1;
      if (status != nullptr) atomicCAS(status, 0, code);
      return false;
    }
  }
}

// ------------------------------------------------------------------- TMA ----
// Cache policy for single-use streams (weights): evict first, so that the
// re-read activations and scales stay resident in L2.
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_3d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int32_t c0, int32_t c1, int32_t c2,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(const CUtensorMap* map, uint64_t* bar, void* dst,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "l"(policy)
      : "memory");
}

// Untiled bulk copy global -> shared.  Both addresses 16-byte aligned, size a
// multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// ------------------------------------------------------------------- PDL ----
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// --------------------------------------------------------------- tcgen05 ----
// Executed by one full warp.  Writes the TMEM base address to *dst (smem).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, e4m3 x e4m3 -> f32, one elected thread.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 async op issued so far by this
// thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

// 32 lanes x 32 bits, 8 or 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor for a K-major operand in the canonical
// SWIZZLE_128B layout: rows of 128 bytes, 8-row (1024-byte) swizzle atoms,
// atoms 1024 bytes apart along M/N.
//   bits  0-13 start address >> 4      bits 16-29 leading byte offset >> 4 (1)
//   bits 32-45 stride byte offset >> 4 (1024 >> 4)
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 49-51 base offset (0: atoms are 1024-byte aligned)
//   bits 61-63 layout type (2 = SWIZZLE_128B)
// Advancing K by 32 fp8 elements inside the 128-byte row is done by adding 32
// bytes to the start address; the hardware applies the swizzle on the final
// address bits, exactly as TMA wrote them.
__device__ __forceinline__ uint64_t make_desc_k_sw128(uint32_t smem_byte_addr) {
  uint64_t desc = 0;
  desc |= static_cast<uint64_t>((smem_byte_addr & 0x3FFFFu) >> 4);
  desc |= static_cast<uint64_t>(1u) << 16;
  desc |= static_cast<uint64_t>(1024u >> 4) << 32;
  desc |= static_cast<uint64_t>(1u) << 46;
  desc |= static_cast<uint64_t>(2u) << 61;
  return desc;
}

// Instruction descriptor, kind::f8f6f4: D f32 (bits 4-5 = 1), A and B e4m3
// (bits 7-9 and 10-12 = 0), both K-major (bits 15, 16 = 0), N >> 3 at bits
// 17-22, M >> 4 at bits 24-28.
__host__ __device__ __forceinline__ constexpr uint32_t make_idesc_e4m3_f32(uint32_t mma_m,
                                                                         uint32_t mma_n) {
  return (1u << 4) | ((mma_n >> 3) << 17) | ((mma_m >> 4) << 24);
}

// ------------------------------------------------------- global atomics ----
// Ticket increment with acquire-release semantics at GPU scope: releases the
// CTA's earlier writes (made visible to this thread through a CTA barrier) and
// acquires every write released by earlier increments of the same ticket.
__device__ __forceinline__ int atomic_add_acq_rel_gpu(int* addr, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void store_relaxed_gpu(int* addr, int v) {
  asm volatile("st.relaxed.gpu.global.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

// Orders this thread's earlier generic-proxy view of global memory (e.g.
// data acquired from other CTAs) before its later bulk copies (async proxy).
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// System scope (peer GPUs over NVLink): fence, release store, acquire load.
__device__ __forceinline__ void fence_sc_sys() { asm volatile("fence.sc.sys;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void store_release_sys(int* addr, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int load_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void store_relaxed_sys(int* addr, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int load_relaxed_sys(const int* addr) {
  int v;
  asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

__device__ __forceinline__ int load_relaxed_gpu(const int* addr) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// 16-byte line of two 8-byte words, each an aligned 64-bit element and so
// single-copy atomic on its own (a vector access is a set of element
// accesses): a reader that sees a word's tag sees that word's payload.
// Volatile = relaxed at system scope, for peer memory.
__device__ __forceinline__ void st_volatile_line(void* addr, uint64_t w0, uint64_t w1) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(addr), "l"(w0), "l"(w1) : "memory");
}

__device__ __forceinline__ void ld_volatile_line(const void* addr, uint64_t& w0, uint64_t& w1) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(addr) : "memory");
}

__device__ __forceinline__ int load_acquire_gpu(const int* addr) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Compare-and-swap with acquire-release semantics at GPU scope; returns the
// value found.
__device__ __forceinline__ int atomic_cas_acq_rel_gpu(int* addr, int expected, int desired) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.cas.b32 %0, [%1], %2, %3;"
               : "=r"(old)
               : "l"(addr), "r"(expected), "r"(desired)
               : "memory");
  return old;
}

// ------------------------------------------------------------ named barrier --
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ------------------------------------------------------------- packed fp32 --
// (d0, d1) = fma(a, (b0, b1), (d0, d1)): one fma.rn.f32x2, each lane rounded
// exactly as a scalar fmaf.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a, float b0, float b1) {
  uint64_t acc = (static_cast<uint64_t>(__float_as_uint(d1)) << 32) | __float_as_uint(d0);
  asm("{\n\t.reg .b64 sa, sb;\n\tmov.b64 sa, {%1, %1};\n\tmov.b64 sb, {%2, %3};\n\t"
      "fma.rn.f32x2 %0, sa, sb, %0;\n\t}"
      : "+l"(acc)
      : "f"(a), "f"(b0), "f"(b1));
  d0 = __uint_as_float(static_cast<uint32_t>(acc));
  d1 = __uint_as_float(static_cast<uint32_t>(acc >> 32));
}

// ----------------------------------------------------- register reallocation --
// Warpgroup-wide change of the per-thread register allocation.
template <uint32_t kRegs>
__device__ __forceinline__ void regs_increase() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <uint32_t kRegs>
__device__ __forceinline__ void regs_decrease() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// ------------------------------------------------- thread-block clusters --
// Cluster-wide barrier: every thread of every CTA of the cluster arrives
// (release: its earlier shared-memory writes become visible to the cluster)
// and waits for all the others (acquire).  A hardware barrier: it completes
// once every non-exited thread of the cluster has arrived.
__device__ __forceinline__ void cluster_sync_acq_rel() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Dynamic shared memory this launch gave the CTA, in bytes.
__device__ __forceinline__ uint32_t dynamic_smem_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(r));
  return r;
}
// CTAs of this CTA's cluster along y (1 when launched without clusters).
__device__ __forceinline__ uint32_t cluster_dim_y() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctaid.y;" : "=r"(r));
  return r;
}
// The shared::cluster address of offset `saddr` (a shared::cta address of
// this CTA) in the shared memory of cluster CTA `rank`.
__device__ __forceinline__ uint32_t map_shared_rank(uint32_t saddr, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
  return d;
}
__device__ __forceinline__ float4 ld_shared_cluster_f4(uint32_t caddr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(caddr)
               : "memory");
  return v;
}

}  // namespace sm100
}  // namespace dg
