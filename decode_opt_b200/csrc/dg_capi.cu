// SPDX-License-Identifier: MIT
//
// dg_capi.cu -- libdecode_gemm_b200.so: the C ABI declared in
// include/decode_gemm_b200.h, over the sm_100a kernel (dg_kernel.cuh) and the
// host planner (dg_host.cuh).  Also holds the weight prepack kernel and the
// L2 flush helper.

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "decode_gemm_b200.h"
#include "dg_host.cuh"

// Scratch of dg_launch_static_scratch: the split-K tickets (first
// DG_STATIC_SEM_INTS ints) followed by the split-K workspace
// (DG_STATIC_WS_FLOATS floats).  One copy per device, shared by every call on
// that device; it is zero at module load and otherwise keeps the last call's
// contents.
static_assert((DG_STATIC_SEM_INTS * sizeof(int)) % 256 == 0, "workspace must stay 256-byte aligned");
static __device__ __align__(256) unsigned char
    g_static_scratch[DG_STATIC_SEM_INTS * sizeof(int) + DG_STATIC_WS_FLOATS * sizeof(float)];

namespace {

using dg::Config;
using dg::KernelFn;
using dg::Plan;

Config to_config(const dg_config* c) {
  Config out;
  out.m_tile = c->m_tile;
  out.block_n = c->block_n;
  out.subs = c->subs;
  out.stages = c->stages;
  out.layout = c->layout;
  out.pdl = c->pdl;
  out.split_k = c->split_k;
  out.grid_ctas = c->grid_ctas;
  out.epi_warps = c->epi_warps;
  out.flags = c->flags;
  out.timeout_ns = c->timeout_ns;
  out.pack_rows = c->pack_rows;
  return out;
}

int current_sm_count() {
  int dev = 0;
  int sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

// One kernel per batch class (MMA M, batch copies, epilogue warps per
// quarter); everything else is runtime.
struct KernelEntry {
  KernelFn fn;
  std::atomic<unsigned long long> smem_set;          // per device: dynamic smem limit raised
  cudaError_t pool_check;                            // register pool covers the setmaxnreg split
  std::atomic<unsigned long long> nonportable_set;   // per device: cluster sizes above 8 allowed
};

template <int MMA_M, int COPIES, int EPW>
KernelEntry* entry() {
  static KernelEntry e{dg::kernel_ptr<MMA_M, COPIES, EPW>(), {0},
                       dg::check_register_pool(reinterpret_cast<const void*>(dg::kernel_ptr<MMA_M, COPIES, EPW>()),
                                               COPIES, EPW),
                       {0}};
  return &e;
}

KernelEntry* select_kernel(int mma_m, int copies, int epw) {
  if (mma_m == 64 && copies == 4 && epw == 1) return entry<64, 4, 1>();
  if (mma_m == 64 && copies == 2 && epw == 2) return entry<64, 2, 2>();
  if (mma_m == 128 && copies == 2 && epw == 2) return entry<128, 2, 2>();
  if (mma_m == 128 && copies == 1 && epw == 2) return entry<128, 1, 2>();
  return nullptr;
}

// The swap-AB class (no register reallocation, so no pool check).
KernelEntry* swap_entry() {
  static KernelEntry e{dg::swap_kernel_ptr(), {0}, cudaSuccess, {0}};
  return &e;
}

KernelEntry* select_kernel(const Plan& plan) {
  return plan.swap ? swap_entry() : select_kernel(plan.mma_m, plan.copies, plan.epw);
}

// Cluster occupancy of the current device: occ[S] clusters of S CTAs at one
// CTA per SM (every batch-class kernel holds an SM alone: its registers
// exceed half the register file), from cudaOccupancyMaxActiveClusters, asked
// once per device; the measured B200 table when no device answers.
constexpr int kMaxOccDevices = 64;
std::mutex g_occ_mutex;
int g_occ[kMaxOccDevices][dg::kMaxClusterSplit + 1];
bool g_occ_ready[kMaxOccDevices] = {};

const int* device_cluster_occupancy() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxOccDevices) {
    cudaGetLastError();
    return dg::kB200ClusterOccupancy;
  }
  std::lock_guard<std::mutex> lock(g_occ_mutex);
  if (g_occ_ready[dev]) return g_occ[dev];
  KernelEntry* k = entry<64, 4, 1>();
  const void* fn = reinterpret_cast<const void*>(k->fn);
  bool ok = dg::ensure_smem(fn, &k->smem_set) == cudaSuccess &&
            dg::set_func_attribute_once(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1,
                                        &k->nonportable_set) == cudaSuccess;
  g_occ[dev][0] = 0;
  for (int S = 1; ok && S <= dg::kMaxClusterSplit; ++S) {
    cudaLaunchConfig_t lc{};
    cudaLaunchAttribute attr[1]{};
    lc.gridDim = dim3(1u, static_cast<unsigned>(S), 1u);
    lc.blockDim = dim3(static_cast<unsigned>(dg::block_threads(4, 1)), 1u, 1u);
    lc.dynamicSmemBytes = dg::kMaxDynamicSmem;
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(S);
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    int n = 0;
    ok = cudaOccupancyMaxActiveClusters(&n, fn, &lc) == cudaSuccess;
    g_occ[dev][S] = n;
  }
  if (!ok) {
    cudaGetLastError();
    return dg::kB200ClusterOccupancy;
  }
  g_occ_ready[dev] = true;
  return g_occ[dev];
}

// The plan every entry point launches: cluster split-K with split_k <= 1
// takes its split from the device's cluster occupancy.
Plan plan_for(const Config& c, int M, int N, int K) {
  const bool ask = c.grid_ctas == dg::kGridCluster && c.split_k <= 1;
  return dg::make_plan(c, M, N, K, current_sm_count(), ask ? device_cluster_occupancy() : dg::kB200ClusterOccupancy);
}

void fill_info(const Plan& plan, dg_plan_info* out) {
  std::memset(out, 0, sizeof(*out));
  if (plan.error != nullptr) {
    std::snprintf(out->error, sizeof(out->error), "%s", plan.error);
    return;
  }
  out->grid_x = plan.grid.x;
  out->grid_y = plan.grid.y;
  out->grid_z = plan.grid.z;
  out->block_x = plan.block.x;
  out->smem_bytes = plan.smem_bytes;
  out->num_output_tiles = plan.params.num_tiles;
  out->padded_n = plan.padded_n;
  out->stages = plan.params.stages;
  out->n_mma = plan.params.n_mma;
  out->a_rows = plan.params.a_rows;
  out->mma_m = plan.mma_m;
  out->epi_warps = plan.epi_warps;
  out->num_ctas = plan.params.num_ctas;
  out->max_slabs = plan.max_slabs;
  out->ws_floats = plan.ws_floats;
  out->sem_ints = plan.sem_ints;
  out->cluster = plan.cluster;
}

// Fills the output copies and the fused-gather fields of `p` from `g`
// (nullptr: one output, row stride N).
cudaError_t apply_gather(dg::KernelParams& p, const dg_gather* g) {
  p.outs[0] = p.output;
  if (g == nullptr) return cudaSuccess;
  if (g->world < 1 || g->world > DG_MAX_RANKS || g->rank < 0 || g->rank >= g->world || g->ldo < p.N)
    return cudaErrorInvalidValue;
  if (static_cast<long long>(g->rank + 1) * p.N > g->ldo) return cudaErrorInvalidValue;
  for (int r = 0; r < g->world; ++r)
    if (g->outputs[r] == nullptr || (g->world > 1 && g->flags[r] == nullptr)) return cudaErrorInvalidValue;
  if (g->world > 1 && g->sync == nullptr) return cudaErrorInvalidValue;
  p.ldo = g->ldo;
  p.world = g->world;
  p.rank = g->rank;
  p.n_outs = g->world;
  p.output = static_cast<__nv_bfloat16*>(g->outputs[g->rank]);
  p.outs[0] = p.output;
  for (int r = 0, k = 1; r < g->world; ++r) {
    p.peer_flags[r] = g->flags[r];
    if (r != g->rank) p.outs[k++] = static_cast<__nv_bfloat16*>(g->outputs[r]);
  }
  p.my_flags = g->flags[g->rank];
  p.sync_ctr = g->sync;
  return cudaSuccess;
}

// Fills the fused-gather-in-lines fields of `p` from `gl` (world 1: a plain
// launch into gl->output with row stride gl->ldo).
cudaError_t apply_gather_lines(dg::KernelParams& p, const dg_gather_lines* gl) {
  if (gl->world < 1 || gl->world > DG_MAX_RANKS || gl->rank < 0 || gl->rank >= gl->world || gl->output == nullptr ||
      gl->ldo < 0 || static_cast<long long>(gl->world) * p.N > gl->ldo || (gl->ldo & 3) != 0 || (p.N & 3) != 0 ||
      (reinterpret_cast<uintptr_t>(gl->output) & 7u) != 0)
    return cudaErrorInvalidValue;
  p.output = static_cast<__nv_bfloat16*>(gl->output) + static_cast<size_t>(gl->rank) * p.N;
  p.outs[0] = p.output;
  p.ldo = gl->ldo;
  if (gl->world == 1) return (gl->q_out != nullptr || gl->q_scales != nullptr) ? cudaErrorInvalidValue : cudaSuccess;
  if (gl->sync == nullptr || (p.flags & dg::kFlagCluster) == 0) return cudaErrorInvalidValue;
  for (int r = 0; r < gl->world; ++r)
    if (gl->lines[r] == nullptr || (reinterpret_cast<uintptr_t>(gl->lines[r]) & 15u) != 0)
      return cudaErrorInvalidValue;
  p.world = gl->world;
  p.rank = gl->rank;
  p.output = static_cast<__nv_bfloat16*>(gl->output);   // the unpack writes all columns
  p.outs[0] = p.output;
  p.n_outs = 1;
  for (int r = 0; r < gl->world; ++r) p.lines[r] = static_cast<uint4*>(gl->lines[r]);
  p.lines_per_row = gl->world * p.N / 4;
  p.sync_ctr = gl->sync;
  p.flags |= dg::kFlagGatherLines;
  if (gl->q_out != nullptr || gl->q_scales != nullptr) {
    if (gl->q_out == nullptr || gl->q_scales == nullptr || (static_cast<long long>(gl->world) * p.N) % 128 != 0 ||
        (reinterpret_cast<uintptr_t>(gl->q_out) & 3u) != 0 || (reinterpret_cast<uintptr_t>(gl->q_scales) & 3u) != 0)
      return cudaErrorInvalidValue;
    p.q_out = static_cast<uint8_t*>(gl->q_out);
    p.q_scales = gl->q_scales;
    p.flags |= dg::kFlagGatherLinesQuant;
  }
  return cudaSuccess;
}

int launch_impl(const dg_config* cfg, const dg_problem* prob, const CUtensorMap* w_map,
                const CUtensorMap* a_map, cudaStream_t stream, bool pdl_attr, const dg_gather* g = nullptr,
                void* q_out = nullptr, float* q_scales = nullptr, const dg_gather_lines* gl = nullptr) {
  if (cfg == nullptr || prob == nullptr) return cudaErrorInvalidValue;
  const Config c = to_config(cfg);
  Plan plan = plan_for(c, prob->M, prob->N, prob->K);
  if (plan.error != nullptr) return cudaErrorInvalidValue;
  dg::KernelParams& p = plan.params;
  p.output = static_cast<__nv_bfloat16*>(prob->output);
  if (g != nullptr) p.output = static_cast<__nv_bfloat16*>(g->outputs[g->rank >= 0 && g->rank < DG_MAX_RANKS ? g->rank : 0]);
  const cudaError_t g_err = apply_gather(p, g);
  if (g_err != cudaSuccess) return g_err;
  if (gl != nullptr) {
    if (g != nullptr || q_out != nullptr) return cudaErrorInvalidValue;
    const cudaError_t l_err = apply_gather_lines(p, gl);
    if (l_err != cudaSuccess) return l_err;
  }
  p.w_scales = prob->weight_scales;
  p.a_scales = prob->activation_scales;
  p.ws = prob->splitk_ws;
  p.sem = prob->splitk_sem;
  p.status = prob->status;
  p.weight = static_cast<const uint8_t*>(prob->weight);
  const cudaError_t buf_err = dg::check_buffers(plan, p);
  if (buf_err != cudaSuccess) return buf_err;
  if (q_out != nullptr || q_scales != nullptr) {
    // The fused quantiser owns whole 128-column blocks of one tile and stores
    // 8-byte bf16 and 4-byte e4m3 vectors.
    if (q_out == nullptr || q_scales == nullptr || g != nullptr || (p.flags & dg::kFlagCluster) == 0 ||
        p.N % 128 != 0 || p.block_n % 128 != 0 || p.ldo != p.N ||
        (reinterpret_cast<uintptr_t>(p.output) & 7u) != 0 || (reinterpret_cast<uintptr_t>(q_out) & 3u) != 0 ||
        (reinterpret_cast<uintptr_t>(q_scales) & 3u) != 0)
      return cudaErrorInvalidValue;
    p.q_out = static_cast<uint8_t*>(q_out);
    p.q_scales = q_scales;
    p.flags |= dg::kFlagQuantizeOut;
  }
  KernelEntry* k = select_kernel(plan);
  if (k == nullptr) return cudaErrorInvalidValue;
  if (k->pool_check != cudaSuccess) return k->pool_check;
  const cudaError_t attr_err = dg::ensure_smem(reinterpret_cast<const void*>(k->fn), &k->smem_set);
  if (attr_err != cudaSuccess) return attr_err;
  if (plan.cluster > 8) {
    const cudaError_t e = dg::set_func_attribute_once(reinterpret_cast<const void*>(k->fn),
                                                      cudaFuncAttributeNonPortableClusterSizeAllowed, 1,
                                                      &k->nonportable_set);
    if (e != cudaSuccess) return e;
  }
  return dg::launch_kernel(k->fn, plan, p, *w_map, *a_map, stream, pdl_attr);
}

// raw [n,k] -> [tile][kb][row][128] (optionally 128-byte swizzled), one
// 16-byte vector per thread, grid-stride; rows >= n are zero.
__global__ void prepack_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int n, int k,
                               int block_n, int num_tiles, int swizzle) {
  const uint32_t vec_per_row = static_cast<uint32_t>(k) / 16u;
  const uint32_t kb_count = static_cast<uint32_t>(k) / 128u;
  const size_t total = static_cast<size_t>(num_tiles) * block_n * vec_per_row;
  for (size_t v = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<size_t>(gridDim.x) * blockDim.x) {
    // v enumerates destination vectors: ((tile*KB + kb)*BM + r)*8 + c
    const uint32_t c = static_cast<uint32_t>(v & 7u);
    const size_t rest = v >> 3;
    const uint32_t r = static_cast<uint32_t>(rest % block_n);
    const size_t tk = rest / block_n;
    const uint32_t kb = static_cast<uint32_t>(tk % kb_count);
    const uint32_t tile = static_cast<uint32_t>(tk / kb_count);
    const uint32_t row = tile * block_n + r;
    const uint32_t src_c = swizzle ? (c ^ (r & 7u)) : c;   // dst chunk c holds src chunk c^(r%8)
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (row < static_cast<uint32_t>(n)) val = src[static_cast<size_t>(row) * vec_per_row + kb * 8u + src_c];
    dst[v] = val;
  }
}

// Device address of g_static_scratch on the current device, looked up once per
// device (cudaGetSymbolAddress, with that device current) and cached for the
// life of the process: the cache assumes the device's primary context (which
// holds the array) lives as long as the process, i.e. nobody calls
// cudaDeviceReset on that device and then this entry point again.
constexpr int kMaxScratchDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxScratchDevices] = {};

cudaError_t static_scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxScratchDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (err != cudaSuccess) return err;
    if (ptr == nullptr || (reinterpret_cast<uintptr_t>(ptr) & 255u) != 0) return cudaErrorInvalidDevicePointer;
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

// ------------------------------------------------------------------ IPC ---
// cuMemGetAddressRange through the runtime's driver entry point (no libcuda
// link): the base of the allocation that holds a pointer.
using AddressRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
AddressRangeFn address_range_fn() {
  static std::atomic<AddressRangeFn> cached{nullptr};
  AddressRangeFn fn = cached.load(std::memory_order_acquire);
  if (fn != nullptr) return fn;
  void* sym = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &sym, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || sym == nullptr)
    return nullptr;
  fn = reinterpret_cast<AddressRangeFn>(sym);
  cached.store(fn, std::memory_order_release);
  return fn;
}

// A peer allocation is opened once per process (a second cudaIpcOpenMemHandle
// of the same handle fails), shared by every pointer into it.
struct OpenedAllocation {
  cudaIpcMemHandle_t handle;
  char* base;
  size_t size;   // bytes of the mapping (cuMemGetAddressRange of base)
  int refs;
};
std::mutex g_ipc_mutex;
OpenedAllocation g_ipc_open[64];
int g_ipc_count = 0;

// dg_gather_wait: one thread waits (bounded) until every peer has published
// this rank's latest epoch, i.e. the last fused launch before it on the
// stream has all ranks' slices in this rank's buffer.
__global__ void gather_wait_kernel(int world, int rank, const int* my_flags, int* status,
                                   unsigned long long timeout_ns) {
  using namespace dg::sm100;
  if (threadIdx.x != 0) return;
  const int epoch = load_relaxed_gpu(my_flags + rank);
  const uint64_t start = global_timer_ns();
  for (int r = 0; r < world; ++r) {
    if (r == rank) continue;
    while (load_relaxed_sys(my_flags + r) - epoch < 0) {
      if (global_timer_ns() - start > timeout_ns) {
        if (status != nullptr) atomicCAS(status, 0, DG_ERR_GATHER_WAIT);
        return;
      }
    }
  }
  fence_acq_rel_sys();
}

__global__ void flush_kernel(uint4* buf, size_t n16) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    buf[i] = make_uint4(static_cast<uint32_t>(i), 1u, 2u, 3u);
}

}  // namespace

extern "C" {

int dg_abi_version(void) { return DG_ABI_VERSION; }

int dg_plan(const dg_config* cfg, int M, int N, int K, dg_plan_info* out) {
  if (cfg == nullptr || out == nullptr) return cudaErrorInvalidValue;
  const Plan plan = plan_for(to_config(cfg), M, N, K);
  fill_info(plan, out);
  return plan.error == nullptr ? 0 : static_cast<int>(cudaErrorInvalidValue);
}

int dg_max_active_clusters(const dg_config* cfg, int M, int N, int K, int* out) {
  if (cfg == nullptr || out == nullptr) return cudaErrorInvalidValue;
  *out = 0;
  const Plan plan = plan_for(to_config(cfg), M, N, K);
  if (plan.error != nullptr) return cudaErrorInvalidValue;
  KernelEntry* k = select_kernel(plan);
  if (k == nullptr) return cudaErrorInvalidValue;
  cudaError_t err = dg::ensure_smem(reinterpret_cast<const void*>(k->fn), &k->smem_set);
  if (err != cudaSuccess) return err;
  if (plan.cluster > 8) {
    err = dg::set_func_attribute_once(reinterpret_cast<const void*>(k->fn),
                                      cudaFuncAttributeNonPortableClusterSizeAllowed, 1, &k->nonportable_set);
    if (err != cudaSuccess) return err;
  }
  cudaLaunchConfig_t lc{};
  cudaLaunchAttribute attr[1]{};
  lc.gridDim = plan.grid;
  lc.blockDim = plan.block;
  lc.dynamicSmemBytes = plan.smem_bytes;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(plan.cluster);
  attr[0].val.clusterDim.z = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaOccupancyMaxActiveClusters(out, reinterpret_cast<const void*>(k->fn), &lc);
}

int dg_make_weight_map(const dg_config* cfg, const void* weight, int N, int K, void* map128) {
  if (cfg == nullptr || map128 == nullptr) return cudaErrorInvalidValue;
  const Config c = to_config(cfg);
  if (dg::check_config(c) != nullptr || N < 1 || K < 128 || K % 128 != 0) return cudaErrorInvalidValue;
  return dg::make_weight_map(static_cast<CUtensorMap*>(map128), c, weight, N, K);
}

int dg_make_activation_map(const dg_config* cfg, const void* activation, int M, int K, void* map128) {
  if (cfg == nullptr || map128 == nullptr) return cudaErrorInvalidValue;
  const Config c = to_config(cfg);
  if (dg::check_config(c) != nullptr || M < 1 || M > c.m_tile || K < 128 || K % 128 != 0)
    return cudaErrorInvalidValue;
  return dg::make_activation_map(static_cast<CUtensorMap*>(map128), c, activation, M, K);
}

int dg_launch_with_maps(const dg_config* cfg, const dg_problem* p, const void* weight_map128,
                        const void* activation_map128, void* stream, int pdl_attr) {
  if (weight_map128 == nullptr || activation_map128 == nullptr) return cudaErrorInvalidValue;
  return launch_impl(cfg, p, static_cast<const CUtensorMap*>(weight_map128),
                     static_cast<const CUtensorMap*>(activation_map128),
                     static_cast<cudaStream_t>(stream), pdl_attr != 0);
}

int dg_launch_quantized(const dg_config* cfg, const dg_problem* p, const void* weight_map128,
                        const void* activation_map128, void* q_out, float* q_scales, void* stream, int pdl_attr) {
  if (weight_map128 == nullptr || activation_map128 == nullptr || q_out == nullptr || q_scales == nullptr)
    return cudaErrorInvalidValue;
  return launch_impl(cfg, p, static_cast<const CUtensorMap*>(weight_map128),
                     static_cast<const CUtensorMap*>(activation_map128), static_cast<cudaStream_t>(stream),
                     pdl_attr != 0, nullptr, q_out, q_scales);
}

int dg_launch(const dg_config* cfg, const dg_problem* p, void* stream) {
  if (cfg == nullptr || p == nullptr) return cudaErrorInvalidValue;
  const Config c = to_config(cfg);
  if (dg::check_config(c) != nullptr || p->M < 1 || p->M > c.m_tile || p->N < 1 || p->K < 128 ||
      p->K % 128 != 0)
    return cudaErrorInvalidValue;
  CUtensorMap w{};
  CUtensorMap a{};
  cudaError_t err = dg::make_weight_map(&w, c, p->weight, p->N, p->K);
  if (err != cudaSuccess) return err;
  err = dg::make_activation_map(&a, c, p->activation, p->M, p->K);
  if (err != cudaSuccess) return err;
  return launch_impl(cfg, p, &w, &a, static_cast<cudaStream_t>(stream), c.pdl != 0);
}

int dg_launch_static_scratch(const dg_config* cfg, const dg_problem* p, void* stream, dg_plan_info* info) {
  if (info != nullptr) std::memset(info, 0, sizeof(*info));
  if (cfg == nullptr || p == nullptr) return cudaErrorInvalidValue;
  const Config c = to_config(cfg);
  const Plan plan = plan_for(c, p->M, p->N, p->K);
  if (plan.error != nullptr) {
    if (info != nullptr) fill_info(plan, info);
    return cudaErrorInvalidValue;
  }
  if (plan.ws_floats > DG_STATIC_WS_FLOATS || static_cast<unsigned>(plan.sem_ints) > DG_STATIC_SEM_INTS) {
    if (info != nullptr) {
      fill_info(plan, info);
      std::snprintf(info->error, sizeof(info->error), "static scratch too small: needs %llu ws floats (max %u), %d tickets (max %u)",
                    static_cast<unsigned long long>(plan.ws_floats), DG_STATIC_WS_FLOATS, plan.sem_ints,
                    DG_STATIC_SEM_INTS);
    }
    return cudaErrorInvalidValue;
  }
  void* scratch = nullptr;
  cudaError_t err = static_scratch_on_current_device(&scratch);
  if (err != cudaSuccess) return err;
  int* sem = static_cast<int*>(scratch);
  float* ws = reinterpret_cast<float*>(static_cast<unsigned char*>(scratch) + DG_STATIC_SEM_INTS * sizeof(int));
  // The tickets must start at zero; the workspace slabs are fully written
  // before they are read, so they need no clearing.
  if (plan.sem_ints > 0) {
    err = cudaMemsetAsync(sem, 0, static_cast<size_t>(plan.sem_ints) * sizeof(int), static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) return err;
  }
  dg_problem q = *p;
  q.splitk_ws = ws;
  q.splitk_sem = sem;
  if (info != nullptr) fill_info(plan, info);
  return dg_launch(cfg, &q, stream);
}

int dg_launch_gather(const dg_config* cfg, const dg_problem* p, const dg_gather* g, const void* weight_map128,
                     const void* activation_map128, void* stream, int pdl_attr) {
  if (g == nullptr || weight_map128 == nullptr || activation_map128 == nullptr) return cudaErrorInvalidValue;
  return launch_impl(cfg, p, static_cast<const CUtensorMap*>(weight_map128),
                     static_cast<const CUtensorMap*>(activation_map128), static_cast<cudaStream_t>(stream),
                     pdl_attr != 0, g);
}

int dg_launch_gather_lines(const dg_config* cfg, const dg_problem* p, const dg_gather_lines* g,
                           const void* weight_map128, const void* activation_map128, void* stream, int pdl_attr) {
  if (g == nullptr || weight_map128 == nullptr || activation_map128 == nullptr) return cudaErrorInvalidValue;
  return launch_impl(cfg, p, static_cast<const CUtensorMap*>(weight_map128),
                     static_cast<const CUtensorMap*>(activation_map128), static_cast<cudaStream_t>(stream),
                     pdl_attr != 0, nullptr, nullptr, nullptr, g);
}

int dg_gather_wait(const dg_gather* g, int* status, unsigned long long timeout_ns, void* stream) {
  if (g == nullptr || g->world < 1 || g->world > DG_MAX_RANKS || g->rank < 0 || g->rank >= g->world ||
      g->flags[g->rank] == nullptr)
    return cudaErrorInvalidValue;
  if (g->world == 1) return cudaSuccess;
  gather_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      g->world, g->rank, g->flags[g->rank], status, timeout_ns ? timeout_ns : dg::kDefaultTimeoutNs);
  return cudaGetLastError();
}

int dg_ipc_export(const void* ptr, void* handle64, unsigned long long* offset) {
  if (ptr == nullptr || handle64 == nullptr || offset == nullptr) return cudaErrorInvalidValue;
  AddressRangeFn range = address_range_fn();
  if (range == nullptr) return cudaErrorInsufficientDriver;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h{};
  const cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (err != cudaSuccess) return err;
  std::memcpy(handle64, &h, sizeof(h));
  *offset = static_cast<unsigned long long>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return cudaSuccess;
}

int dg_ipc_import(const void* handle64, unsigned long long offset, void** ptr) {
  if (handle64 == nullptr || ptr == nullptr) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h{};
  std::memcpy(&h, handle64, sizeof(h));
  std::lock_guard<std::mutex> lock(g_ipc_mutex);
  for (int i = 0; i < g_ipc_count; ++i) {
    if (std::memcmp(&g_ipc_open[i].handle, &h, sizeof(h)) == 0) {
      if (offset >= g_ipc_open[i].size) return cudaErrorInvalidValue;
      ++g_ipc_open[i].refs;
      *ptr = g_ipc_open[i].base + offset;
      return cudaSuccess;
    }
  }
  if (g_ipc_count == 64) return cudaErrorMemoryAllocation;
  AddressRangeFn range = address_range_fn();
  if (range == nullptr) return cudaErrorInsufficientDriver;
  void* base = nullptr;
  const cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (err != cudaSuccess) return err;
  CUdeviceptr rbase = 0;
  size_t size = 0;
  if (range(&rbase, &size, reinterpret_cast<CUdeviceptr>(base)) != CUDA_SUCCESS ||
      reinterpret_cast<char*>(rbase) != static_cast<char*>(base) || offset >= size) {
    cudaIpcCloseMemHandle(base);
    return cudaErrorInvalidValue;
  }
  g_ipc_open[g_ipc_count] = {h, static_cast<char*>(base), size, 1};
  ++g_ipc_count;
  *ptr = static_cast<char*>(base) + offset;
  return cudaSuccess;
}

int dg_ipc_release(void* ptr) {
  if (ptr == nullptr) return cudaErrorInvalidValue;
  std::lock_guard<std::mutex> lock(g_ipc_mutex);
  // The opened mapping that holds ptr; a pointer inside none of them (never
  // imported, or released already) is rejected and changes nothing.
  int best = -1;
  const char* q = static_cast<const char*>(ptr);
  for (int i = 0; i < g_ipc_count; ++i)
    if (g_ipc_open[i].base <= q && q < g_ipc_open[i].base + g_ipc_open[i].size) best = i;
  if (best < 0) return cudaErrorInvalidValue;
  if (--g_ipc_open[best].refs > 0) return cudaSuccess;
  const cudaError_t err = cudaIpcCloseMemHandle(g_ipc_open[best].base);
  g_ipc_open[best] = g_ipc_open[g_ipc_count - 1];
  --g_ipc_count;
  return err;
}

int dg_prepack_weight(const void* src, void* dst, int n, int k, int block_n, int layout, void* stream) {
  if (src == nullptr || dst == nullptr || n < 1 || k < 128 || k % 128 != 0 || block_n < 8 ||
      block_n > 256 || block_n % 8 != 0)
    return cudaErrorInvalidValue;
  if (layout != DG_LAYOUT_PACKED && layout != DG_LAYOUT_PACKED_SWIZZLED) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0 || (reinterpret_cast<uintptr_t>(dst) & 15u) != 0)
    return cudaErrorInvalidValue;
  const int tiles = (n + block_n - 1) / block_n;
  const size_t total = static_cast<size_t>(tiles) * block_n * (k / 16);
  const int threads = 256;
  int sms = current_sm_count();
  if (sms <= 0) sms = 148;
  const size_t want = (total + threads - 1) / threads;
  const unsigned blocks = static_cast<unsigned>(want < static_cast<size_t>(sms) * 16 ? want : static_cast<size_t>(sms) * 16);
  prepack_kernel<<<blocks, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint4*>(src), static_cast<uint4*>(dst), n, k, block_n, tiles,
      layout == DG_LAYOUT_PACKED_SWIZZLED ? 1 : 0);
  return cudaGetLastError();
}

int dg_padded_n(int n, int block_n) { return block_n > 0 ? dg::padded_n(n, block_n) : 0; }

unsigned long long dg_packed_weight_bytes(int n, int k, int block_n) {
  return block_n > 0 ? static_cast<unsigned long long>(dg::packed_weight_bytes(n, k, block_n)) : 0ull;
}

const char* dg_status_string(int code) {
  switch (code) {
    case DG_STATUS_OK: return "ok";
    case DG_ERR_PRODUCER_EMPTY_WAIT: return "producer: timed out waiting for a free smem stage";
    case DG_ERR_MMA_FULL_WAIT: return "mma: timed out waiting for a TMA stage";
    case DG_ERR_MMA_ACCUM_WAIT: return "mma: timed out waiting for a free TMEM accumulator";
    case DG_ERR_EPILOGUE_ACCUM_WAIT: return "epilogue: timed out waiting for a TMEM accumulator";
    case DG_ERR_DRAIN_TMA: return "teardown: TMA copies did not complete in time";
    case DG_ERR_DRAIN_MMA: return "teardown: MMAs did not complete in time";
    case DG_ERR_INJECTED_TIMEOUT: return "injected timeout (test hook)";
    case DG_ERR_BAD_LAUNCH_SHAPE: return "launch grid/block does not match the plan";
    case DG_ERR_REDUCE_WAIT: return "split reduction: a workspace bulk copy did not land in time";
    case DG_ERR_GATHER_WAIT: return "fused gather: a peer's output slices did not arrive in time";
    default: return "unknown status";
  }
}

int dg_host_device_pointer(void* host, void** device) {
  if (host == nullptr || device == nullptr) return cudaErrorInvalidValue;
  void* d = nullptr;
  const cudaError_t err = cudaHostGetDevicePointer(&d, host, 0);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();   // not a sticky error: clear it for the caller's next call
    return err;
  }
  *device = d;
  return cudaSuccess;
}

int dg_flush_l2(void* buf, unsigned long long bytes, void* stream) {
  if (buf == nullptr || bytes < 16) return cudaErrorInvalidValue;
  int sms = current_sm_count();
  if (sms <= 0) sms = 148;
  flush_kernel<<<static_cast<unsigned>(sms) * 4u, 512, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(buf), static_cast<size_t>(bytes / 16));
  return cudaGetLastError();
}

}  // extern "C"
