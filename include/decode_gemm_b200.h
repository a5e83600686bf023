/* SPDX-License-Identifier: MIT
 *
 * decode_gemm_b200.h -- C ABI of the B200 (sm_100a) FP8 decode GEMM library
 * (libdecode_gemm_b200.so, built from decode_opt_b200/csrc/dg_capi.cu).
 *
 *   out[M,N] bf16 = act[M,K] e4m3 . W[N,K]^T e4m3, with per-128-K block scales
 *   weight_scales[ceil(N/128), K/128] and activation_scales[M, K/128], fp32
 *   accumulation, M = 1..128 (decode).
 *
 * Plain C: pointers, ints and sizes only.  All tensor pointers are device
 * pointers owned by the caller; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  Functions return a cudaError_t value (0 = success,
 * 1 = cudaErrorInvalidValue for a rejected configuration or shape), matching
 * the reference's host API, which returns cudaError_t from launch() /
 * launch_with_maps() / launch_prepack_weight().
 *
 * Each entry point replaces the reference interface named beside it
 * (paths are inside the reference repository ziyuhuang123/decode_opt):
 *
 *   dg_plan                 decode_gemm::KernelConfig::validate +
 *                           make_launch_plan   kernels/decode_gemm.cuh:319-346, 1086-1096
 *   dg_make_weight_map      make_weight_tma     kernels/decode_gemm.cuh:413-447
 *   dg_make_activation_map  make_activation_tma kernels/decode_gemm.cuh:449-468
 *   dg_launch_with_maps     launch_with_maps    kernels/decode_gemm.cuh:1113-1147
 *                           (and the harness's direct cudaLaunchKernelEx of
 *                           fp8_decode_gemm<Cfg>, bench/variant_impl.cuh:136-165)
 *   dg_launch_quantized     (new) launch_with_maps fused with the next layer's
 *                           activation quantisation (bench/bench_decode.cu:459-467)
 *   dg_launch               launch              kernels/decode_gemm.cuh:1150-1159
 *   dg_launch_static_scratch (none: no counterpart in the reference) dg_launch
 *                           with library-owned static split-K scratch
 *   dg_prepack_weight       prepack::launch_prepack_weight kernels/weight_prepack.cuh:101-120
 *   dg_padded_n             prepack::padded_n   kernels/weight_prepack.cuh:45-47
 *   dg_packed_weight_bytes  prepack::packed_weight_bytes kernels/weight_prepack.cuh:50-52
 *   dg_status_string        (new) text of the kernel's device status codes
 *   dg_quantize_act         host block quantisation of bench/bench_decode.cu:459-467
 *                           (make_activation), as a GPU kernel
 *   dg_flush_l2             bench helper flush_l2_kernel bench/bench_decode.cu:473-476
 *   dg_probe_bulk_stream    tools/peak_bw_probe.cu tma_stream_probe :82-134 (and the
 *                           L2 self-test :190-211 when run on a small buffer)
 *   dg_probe_naive_read     tools/peak_bw_probe.cu naive_read_nc :138-170
 *   dg_launch_gather        (new: the reference is single-GPU) tensor-parallel launch
 *                           with the all-gather fused into the epilogue
 *   dg_launch_gather_lines  (new) the same with the gather in tagged lines (no flags)
 *   dg_gather_wait          (new) completion wait for the fused gather
 *   dg_ipc_export / dg_ipc_import / dg_ipc_release  (new) peer buffers for it
 *   dg_num_sms              (new) SM count of the current device
 *   dg_host_device_pointer  (new) device address of pinned host memory (zero-copy output)
 *   dg_copy_from_host       (new) a request's input copied from pinned host memory by a
 *                           kernel that can sit under programmatic dependent launch
 *   dg_probe_mma            (new) tcgen05.mma issue / completion cost per shape
 */
#ifndef DECODE_GEMM_B200_H_
#define DECODE_GEMM_B200_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DG_ABI_VERSION 9

/* Weight layouts. */
#define DG_LAYOUT_RAW 0             /* W[N,K], K contiguous (checkpoint layout) */
#define DG_LAYOUT_PACKED 1          /* [tile][k_block][BM rows][128 B], zero-padded rows
                                       (the reference's prepack layout) */
#define DG_LAYOUT_PACKED_SWIZZLED 2 /* same order, each 8-row group pre-swizzled for the
                                       tcgen05 SWIZZLE_128B operand layout (B200 native) */

/* dg_config.grid_ctas value of the cluster split-K schedule (new). */
#define DG_GRID_CLUSTER (-2)

/* Kernel flags (dg_config.flags). */
#define DG_FLAG_INJECT_TIMEOUT 2     /* tests: one wait of CTA 0 can never complete, so its
                                        bounded wait expires, CTA 0 aborts (the other CTAs
                                        finish) and the kernel reports status 0x51 */
#define DG_FLAG_INDEPENDENT_INPUTS 4 /* the activation and scales are not written by the
                                        preceding kernel on the stream (e.g. back-to-back
                                        GEMMs on one activation): with programmatic
                                        dependent launch they are read before
                                        griddepcontrol.wait; global writes still wait */
#define DG_FLAG_CLASS_FROM_M_TILE 32 /* the kernel instantiation follows cfg.m_tile
                                        instead of M (8/16, 32: MMA M 64 with 4, 2
                                        batch copies; 64, 128: MMA M 128 with 2, 1),
                                        as the
                                        C++ header's fp8_decode_gemm<Cfg> is compiled */
#define DG_FLAG_SWAP_AB 512          /* (new) swap-AB batch class for M <= 16: the weights
                                        on the MMA's M side (tcgen05.mma M = 128 weight
                                        rows x N = 16 batch rows, two MMAs from two
                                        issuing warps per tile), a quarter of the
                                        multiply-adds per weight byte of the default
                                        M <= 16 class; needs block_n in [136, 256] and
                                        grid_ctas DG_GRID_CLUSTER (or 0 with split_k 1:
                                        one CTA per tile)
                                        (dg_plan reports mma_m 128, n_mma 16) */

/* Device status codes written to dg_problem.status (first error wins). */
#define DG_STATUS_OK 0
#define DG_ERR_PRODUCER_EMPTY_WAIT 0x11
#define DG_ERR_MMA_FULL_WAIT 0x21
#define DG_ERR_MMA_ACCUM_WAIT 0x22
#define DG_ERR_EPILOGUE_ACCUM_WAIT 0x31
#define DG_ERR_DRAIN_TMA 0x41
#define DG_ERR_DRAIN_MMA 0x42
#define DG_ERR_INJECTED_TIMEOUT 0x51
#define DG_ERR_BAD_LAUNCH_SHAPE 0x61
#define DG_ERR_REDUCE_WAIT 0x71
#define DG_ERR_GATHER_WAIT 0x81

/* Runtime configuration.  Zero-initialise, then set fields. */
typedef struct dg_config {
  int m_tile;    /* bound on M: 8, 16, 32, 64 or 128 (reference M_TILE); the batch is
                    the MMA's M side: 64 rows holding 4 copies of M <= 16, else 128
                    rows holding 4, 2 or 1 copies (M <= 32, 64, 128)                 */
  int block_n;   /* weight rows (output columns) per tile = the MMA's N side:
                    multiple of 8 in [8,256] (reference OUTPUT_ROWS_PER_CTA, <= 64
                    there; 256 = 8 KiB of weights per tcgen05.mma, the B200 default) */
  int subs;      /* 128-K blocks per pipeline stage: 1, 2, 4 (reference SUBS_PER_STAGE)*/
  int stages;    /* smem ring depth, 0 = as many as fit in 227 KiB                     */
  int layout;    /* DG_LAYOUT_*  (reference PREPACK: false = RAW, true = PACKED)       */
  int pdl;       /* 1: griddepcontrol.launch_dependents once the first weight copies
                    are issued, and dg_launch sets programmatic stream serialization
                    (reference PDL)                                                      */
  int split_k;   /* reference SPLITK_FACTOR S >= 1 (grid_ctas == 0), or the cluster
                    split (grid_ctas == DG_GRID_CLUSTER; 1 = as many as fit, <= 16)    */
  int grid_ctas; /* 0: grid = ceil(N/BM) x split_k (reference schedule);
                    >0: stream-K over this many CTAs; -1: stream-K, one CTA per SM;
                    DG_GRID_CLUSTER: cluster split-K (new): grid ceil(N/BM) x S,
                    the S CTAs of a tile form a thread-block cluster and reduce
                    through distributed shared memory -- no workspace          */
  int epi_warps; /* 0 (or the value block_n implies: 4 per 64 tile columns)            */
  int flags;     /* DG_FLAG_*: INDEPENDENT_INPUTS, SWAP_AB, CLASS_FROM_M_TILE; and
                    INJECT_TIMEOUT, a test hook                                         */
  unsigned long long timeout_ns; /* bounded-wait limit per wait; 0 = 2 s               */
  int pack_rows; /* DG_LAYOUT_PACKED only: rows per tile of the packed weights when one
                    tile of the kernel (block_n rows) spans several of them -- block_n a
                    multiple of pack_rows; 0 = block_n.  The reference's prepack layout
                    for OUTPUT_ROWS_PER_CTA = BM is read this way with block_n = T * BM
                    (its TILES_PER_CTA idea): one TMA box per 128-K block lands T
                    packed tiles as one MMA operand                                      */
} dg_config;

/* One GEMM (reference decode_gemm::Problem, kernels/decode_gemm.cuh:352-363). */
typedef struct dg_problem {
  int M, N, K;
  const void* activation;          /* [M,K] e4m3, K contiguous, 16-byte aligned     */
  const void* weight;              /* layout-dependent, 16-byte aligned              */
  const float* weight_scales;      /* [ceil(N/128), K/128]                           */
  const float* activation_scales;  /* [M, K/128]                                     */
  void* output;                    /* [M,N] bf16, N contiguous                       */
  float* splitk_ws;                /* >= plan.ws_floats floats when plan.max_slabs>1 */
  int* splitk_sem;                 /* >= plan.sem_ints ints, zeroed once; the kernel
                                      re-zeroes each ticket it uses                  */
  int* status;                     /* device int, 0 before the launch; may be NULL   */
} dg_problem;

/* Launch plan (reference decode_gemm::LaunchPlan, kernels/decode_gemm.cuh:373-380). */
typedef struct dg_plan_info {
  unsigned grid_x, grid_y, grid_z;
  unsigned block_x;
  unsigned smem_bytes;
  int num_output_tiles;
  int padded_n;
  int stages;
  int n_mma;                       /* MMA N = block_n rounded up to 16              */
  int a_rows;                      /* activation rows per TMA box = M rounded up to 8 */
  int mma_m;                       /* MMA M: 64 (M <= 16) or 128                    */
  int epi_warps;
  int num_ctas;
  int max_slabs;                   /* workspace slabs a split tile needs (1 = none) */
  unsigned long long ws_floats;    /* required splitk_ws size in floats             */
  int sem_ints;                    /* required splitk_sem size in ints              */
  int cluster;                     /* CTAs per cluster along grid y (1 = none)      */
  char error[96];                  /* empty when usable                             */
} dg_plan_info;

int dg_abi_version(void);

/* Validates (cfg, M, N, K) and fills *out.  Returns 0, or 1 with out->error set. */
int dg_plan(const dg_config* cfg, int M, int N, int K, dg_plan_info* out);

/* (new) How many clusters of the plan's size (dg_plan_info.cluster) can be
   resident on the current device at once, one CTA per SM
   (cudaOccupancyMaxActiveClusters); grids of cluster split-K above that run
   in more than one wave.  Returns a cudaError_t value. */
int dg_max_active_clusters(const dg_config* cfg, int M, int N, int K, int* out);

/* Encodes the tensor maps the kernel reads (opaque 128-byte CUtensorMap
   blobs).  The weight map is all zero for DG_LAYOUT_PACKED_SWIZZLED. */
int dg_make_weight_map(const dg_config* cfg, const void* weight, int N, int K, void* map128);
int dg_make_activation_map(const dg_config* cfg, const void* activation, int M, int K, void* map128);

/* Launches with pre-built maps; pdl_attr selects programmatic stream
   serialization for this launch independently of cfg->pdl. */
int dg_launch_with_maps(const dg_config* cfg, const dg_problem* p, const void* weight_map128,
                        const void* activation_map128, void* stream, int pdl_attr);

/* (new) The GEMM and the next layer's activation quantisation in one kernel:
   besides the bf16 output it writes q_out [M,N] e4m3 and q_scales [M,N/128]
   fp32 -- the block quantisation of that bf16 output (bench/bench_decode.cu
   459-467 of the reference, which the reference's decode chain runs as a
   separate step, here dg_quantize_act), bit for bit the bytes and scales
   dg_quantize_act would write from it.  Cluster split-K schedule only
   (grid_ctas == DG_GRID_CLUSTER), N and block_n multiples of 128, output
   8-byte and q_out / q_scales 4-byte aligned; the quantised stores, like the
   output's, follow griddepcontrol.wait.  Otherwise as dg_launch_with_maps. */
int dg_launch_quantized(const dg_config* cfg, const dg_problem* p, const void* weight_map128,
                        const void* activation_map128, void* q_out, float* q_scales, void* stream, int pdl_attr);

/* Encodes both maps, then launches (attribute follows cfg->pdl). */
int dg_launch(const dg_config* cfg, const dg_problem* p, void* stream);

/* Tensor-parallel GEMM with the all-gather fused into the kernel.  Rank r of
   `world` computes its N-shard (p->N rows of W) and stores every output element
   into all ranks' gathered [M, ldo] bf16 buffers over NVLink (peer memory
   mapped into this process, e.g. with dg_ipc_import), at column offset
   r * p->N.  The grid publishes a per-launch epoch into every rank's flag
   array after its stores and completes only after every peer has published
   the same epoch here (bounded wait; status DG_ERR_GATHER_WAIT otherwise):
   when it has completed, this rank's gathered [M, N] of the launch is whole.
   After any error re-zero the flags and sync words on every rank.
   p->output is ignored (outputs[rank] is used).
   Consecutive launches must alternate between two sets of gathered buffers;
   every rank must make the same sequence of launches. */
#define DG_MAX_RANKS 8
typedef struct dg_gather {
  int world, rank;            /* tensor-parallel group, 1 <= world <= DG_MAX_RANKS */
  int ldo;                    /* row stride of the gathered buffers in elements (world * N) */
  void* outputs[DG_MAX_RANKS];/* rank q's gathered buffer + rank * N (this rank's columns)   */
  int* flags[DG_MAX_RANKS];   /* rank q's flag array: int[world], zeroed once                  */
  int* sync;                  /* this rank's int[2] (CTA done count, reserved), zeroed once   */
} dg_gather;

/* Replaces no reference interface (the reference is single-GPU): launch with
   pre-built maps and the fused gather. */
int dg_launch_gather(const dg_config* cfg, const dg_problem* p, const dg_gather* g, const void* weight_map128,
                     const void* activation_map128, void* stream, int pdl_attr);

/* (new) The fused gather without flags: every output element travels as half
   of an 8-byte word {2 bf16, 32-bit epoch} -- single-copy atomic, so a rank
   that sees the epoch has the data, with no system-scope fence and no flag
   round trip (the low-latency protocol of collective libraries).  Rank r
   stores its N columns as 16-byte lines into every rank's line buffer (world
   * N / 4 lines per row); each CTA then waits (bounded, DG_ERR_GATHER_WAIT)
   until its slice of this rank's buffer carries the launch's epoch and
   unpacks it into `output`.  When the grid has completed, this rank's
   gathered [M, ldo] output is whole.  Cluster split-K schedule only
   (grid_ctas == DG_GRID_CLUSTER, at least two CTAs per tile), N a multiple of
   4, output 8-byte and lines 16-byte aligned, ldo a multiple of 4.  The
   epoch lives in sync[1]: consecutive launches must alternate between two
   sets of line buffers, every rank must make the same sequence of launches,
   and after any error every rank re-zeroes its line buffers and sync words.
   p->output is ignored. */
typedef struct dg_gather_lines {
  int world, rank;            /* tensor-parallel group, 1 <= world <= DG_MAX_RANKS            */
  int ldo;                    /* row stride of `output` in elements (>= world * N)             */
  void* output;               /* this rank's gathered [M, ldo] bf16 buffer, column 0           */
  void* lines[DG_MAX_RANKS];  /* rank q's line buffer of this launch's set (as mapped here):
                                 M * world * N * 4 bytes, zeroed once                          */
  int* sync;                  /* this rank's int[2] (CTA done count, last epoch), zeroed once  */
  void* q_out;                /* optional (NULL: none): e4m3 [M, world * N] block quantisation
                                 of the gathered output, written by the unpack -- the bytes
                                 dg_quantize_act would make from it (world > 1, world * N a
                                 multiple of 128, 4-byte aligned)                              */
  float* q_scales;            /* with q_out: fp32 [M, world * N / 128]                          */
} dg_gather_lines;

int dg_launch_gather_lines(const dg_config* cfg, const dg_problem* p, const dg_gather_lines* g,
                           const void* weight_map128, const void* activation_map128, void* stream, int pdl_attr);

/* Waits on `stream` (one thread, bounded by timeout_ns, 0 = 2 s) until every
   peer has published this rank's latest epoch -- already true once the last
   fused launch has completed; an explicit check for callers that want one.
   status (device int, may be NULL) receives DG_ERR_GATHER_WAIT on a timeout. */
int dg_gather_wait(const dg_gather* g, int* status, unsigned long long timeout_ns, void* stream);

/* CUDA IPC for the fused gather's peer buffers (no reference counterpart).
   dg_ipc_export: 64-byte handle of the allocation holding `ptr` and ptr's
   offset in it.  dg_ipc_import: maps a peer's allocation (once per process,
   reference-counted) and returns the peer pointer; dg_ipc_release drops one
   reference (`ptr` as returned by dg_ipc_import; a pointer inside no imported
   mapping returns cudaErrorInvalidValue and changes nothing). */
int dg_ipc_export(const void* ptr, void* handle64, unsigned long long* offset);
int dg_ipc_import(const void* handle64, unsigned long long offset, void** ptr);
int dg_ipc_release(void* ptr);

/* Capacity of the library's static split-K scratch (dg_launch_static_scratch):
   4096 tickets (16 KiB) + 2 Mi workspace floats (8 MiB) per device. */
#define DG_STATIC_SEM_INTS 4096u
#define DG_STATIC_WS_FLOATS 2097152u

/* No counterpart in the reference (which always takes caller-allocated
   splitk_ws / splitk_sem).  dg_launch for callers that cannot allocate device
   memory: p->splitk_ws and p->splitk_sem are ignored and the split-K tickets
   and workspace come from a file-scope __device__ array inside the library, so
   the call allocates nothing (no cudaMalloc / cudaFree, no allocating library
   routine).  It clears the tickets it will use (cudaMemsetAsync on `stream`)
   and launches on `stream` as dg_launch does.
   - Limit: returns cudaErrorInvalidValue (1), with info->error saying so, when
     the plan needs more than DG_STATIC_WS_FLOATS workspace floats or more than
     DG_STATIC_SEM_INTS tickets (dg_plan reports both as ws_floats, sem_ints).
   - The first call on each device looks up the array's address
     (cudaGetSymbolAddress with that device current): make that first call
     before any stream capture on the device.  The address is kept for the
     life of the process, so the device's primary context must live as long:
     no cudaDeviceReset on that device before a later call.
   - The ticket clear is a memset node between the previous kernel on the
     stream and this launch, so under programmatic dependent launch this call
     does not overlap the kernel before it (dg_launch does).
   - Every call on a device shares the one array: calls that overlap on the GPU
     (other streams, other host threads) race.  Calls in order on one stream are
     safe.
   `info` may be NULL; when given it receives the plan (or the error). */
int dg_launch_static_scratch(const dg_config* cfg, const dg_problem* p, void* stream, dg_plan_info* info);

/* raw [n,k] -> layout (DG_LAYOUT_PACKED or DG_LAYOUT_PACKED_SWIZZLED); dst has
   dg_packed_weight_bytes(n, k, block_n) bytes.  k must be a multiple of 128. */
int dg_prepack_weight(const void* src, void* dst, int n, int k, int block_n, int layout, void* stream);
int dg_padded_n(int n, int block_n);
unsigned long long dg_packed_weight_bytes(int n, int k, int block_n);

const char* dg_status_string(int code);

/* Activation quantiser: bf16 x[M, K] (row stride ldx >= K, e.g. a gathered
   [M, N] GEMM output feeding the next layer) -> e4m3 q[M, K] and fp32
   scales[M, K/128], per row and 128-column block scale = max(amax, 1e-4)/448,
   q = e4m3_rn(clamp(x / scale, +-448)) -- the reference's host quantisation
   (bench/bench_decode.cu:459-467) on the GPU.  K % 128 == 0, q 4-byte
   aligned.  pdl_attr: launch with programmatic stream serialization (the
   kernel releases its dependents at once and waits for the producer of x). */
int dg_quantize_act(const void* x, int ldx, int M, int K, void* q, float* scales, void* stream, int pdl_attr);

/* Writes `bytes` of `buf` (device) to evict L2 between timed launches. */
int dg_flush_l2(void* buf, unsigned long long bytes, void* stream);

/* Achievable-HBM probes.  Each reads `bytes` of `buf` once; the caller times
   the launch.  sink: one device unsigned long long the kernels may touch.
   bulk_stream: `ctas` CTAs, each streaming a contiguous slice through an smem
   ring of `stages` x op_bytes with cp.async.bulk (op_bytes % 16 == 0).
   naive_read: ld.global.nc grid-stride reads, blocks_per_sm x SMs x 512 threads. */
int dg_probe_bulk_stream(const void* buf, unsigned long long bytes, unsigned op_bytes, int ctas,
                         int stages, int* status, unsigned long long* sink, void* stream);
int dg_probe_naive_read(const void* buf, unsigned long long bytes, int blocks_per_sm,
                        unsigned long long* sink, void* stream);
int dg_num_sms(void);

/* (new) Device address of pinned, mapped host memory (cudaHostAlloc /
   cudaMallocHost, or cudaHostRegister with the mapped flag).  Passed as
   dg_problem.output (or dg_gather_lines.output) it makes the kernel write
   the bf16 result straight into host memory over PCIe: no device buffer and
   no separate device-to-host copy; the data is in host memory once the
   launch has completed.  Returns a cudaError_t value (an error, and *device
   untouched, for memory that is not mapped pinned memory). */
int dg_host_device_pointer(void* host, void** device);

/* (new) dst[0, bytes) = src[0, bytes) on `stream`, done by a small kernel whose
   loads read `src`, mapped pinned host memory given by its device address
   (dg_host_device_pointer), over PCIe.  With pdl_attr the kernel is launched
   with programmatic stream serialization: it releases its dependents at once
   (the next GEMM may prefetch its weights before its griddepcontrol.wait)
   and waits for the preceding grid before it writes dst, so a chain of
   "copy request i's input, GEMM request i" keeps one request at a time while
   every GEMM's launch and weight prefetch overlap the previous one, where a
   copy node would order the next launch after the previous GEMM's end.
   Returns a cudaError_t value. */
int dg_copy_from_host(void* dst, const void* src, unsigned long long bytes, void* stream, int pdl_attr);

/* tcgen05.mma cost probe: in each of `ctas` CTAs (at most one per SM)
   `issuers` warps (1..4) issue iters / issuers kind::f8f6f4 MMAs each, of
   shape mma_m x mma_n x 32 (mma_m 64 or 128; mma_n a multiple of 8 (M 64) or
   16 (M 128), at most 256) from zeroed smem operands, every warp round-robin
   over its own `accumulators` TMEM accumulators (runs of four MMAs
   accumulate; issuers * accumulators * mma_n <= 512).  out[2c] = clock64
   cycles until the slowest warp has issued, out[2c+1] = cycles until all
   have completed; -1 and *status = 0x93 if a completion wait timed out. */
int dg_probe_mma(int mma_m, int mma_n, int iters, int accumulators, int issuers, int ctas, long long* out,
                 int* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DECODE_GEMM_B200_H_ */
