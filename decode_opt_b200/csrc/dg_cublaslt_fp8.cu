// SPDX-License-Identifier: MIT
//
// dg_cublaslt_fp8.cu -- the library baseline: cuBLASLt FP8 (e4m3 x e4m3 ->
// bf16, fp32 accumulate) on the decode GEMM out[M,N] = act[M,K] . W[N,K]^T
// with the reference's scale layout -- one fp32 scale per 128x128 weight
// block and per 1x128 activation block (CUBLASLT_MATMUL_MATRIX_SCALE_
// BLK128x128_32F on the weights, VEC128_32F on the activation) -- or one
// per-tensor scale each (SCALAR_32F).  The reference reports a cuBLASLt FP8
// baseline (results/baseline_cublaslt.csv) without the program that made it;
// this is that program for B200, linked to the CUDA toolkit's cuBLASLt.
//
//   dg_cublaslt_fp8 [--n N] [--k K] [--ms 1,8,64,128] [--iters I] [--mode block|tensor]
//
// Column-major view: D (N x M, ld N) = op(A) . B with A = W stored K x N
// (ld K, transposed: "TN", the layout FP8 requires), B = act stored K x M
// (ld K), so D is out[M][N] row-major.  Weights rotate over enough device
// copies (>= max(1 GiB, 4 x L2)) that every launch reads them cold; the
// timed loop is `iters` launches captured in one CUDA graph, CUDA events
// around its replay (best of 3).  Before timing, the output of every M is
// checked against a plain fp32 GPU reference of the same scaled product
// (rel_l2 <= 2e-3); the scale tensors' layout is the first of the candidate
// orders that passes.  One JSON line per M on stdout; a configuration
// cuBLASLt has no algorithm for is reported as unavailable, with the reason.

#include <cublasLt.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

namespace {

#define CUDA_OK(x)                                                                             \
  do {                                                                                         \
    cudaError_t e_ = (x);                                                                      \
    if (e_ != cudaSuccess) {                                                                   \
      std::fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
      std::exit(2);                                                                            \
    }                                                                                          \
  } while (0)

// Deterministic e4m3 bytes with finite magnitudes in [1/8, 4) and both signs.
__global__ void fill_e4m3(uint8_t* p, size_t n, uint32_t seed) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    uint32_t x = static_cast<uint32_t>(i) * 2654435761u ^ seed ^ static_cast<uint32_t>(i >> 32) * 40503u;
    x ^= x >> 15;
    x *= 2246822519u;
    x ^= x >> 13;
    const uint32_t e = 4u + (x >> 8) % 6u;   // exponent field 4..9
    p[i] = static_cast<uint8_t>(((x >> 4) & 0x80u) | (e << 3) | (x & 7u));
  }
}

__global__ void fill_scales(float* p, size_t n, uint32_t seed, float lo, float span) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    uint32_t x = static_cast<uint32_t>(i) * 2654435761u ^ seed;
    x ^= x >> 16;
    x *= 2246822519u;
    x ^= x >> 13;
    p[i] = lo + span * static_cast<float>(x & 0xffffu) / 65536.0f;
  }
}

// Plain fp32 reference: out[m][n] = sum_kb ws[n/128][kb] * as[m][kb] * sum_k a[m][k] w[n][k].
__global__ void reference_gemm(const uint8_t* act, const uint8_t* w, const float* a_s, const float* w_s,
                               float* out, int M, int N, int K) {
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = blockIdx.y;
  if (n >= N || m >= M) return;
  const int kb_n = K / 128;
  float acc = 0.0f;
  for (int kb = 0; kb < kb_n; ++kb) {
    float part = 0.0f;
    for (int k = kb * 128; k < kb * 128 + 128; ++k) {
      const float av =
          static_cast<float>(*reinterpret_cast<const __nv_fp8_e4m3*>(act + static_cast<size_t>(m) * K + k));
      const float wv = static_cast<float>(*reinterpret_cast<const __nv_fp8_e4m3*>(w + static_cast<size_t>(n) * K + k));
      part = fmaf(av, wv, part);
    }
    acc = fmaf(w_s[static_cast<size_t>(n / 128) * kb_n + kb] * a_s[static_cast<size_t>(m) * kb_n + kb], part, acc);
  }
  out[static_cast<size_t>(m) * N + n] = acc;
}

// A scale tensor [rows][cols] in a candidate layout: `transposed` stores
// [cols][rows].
__global__ void relayout(const float* src, float* dst, int rows, int cols, int transposed) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * cols) return;
  const int r = i / cols, c = i % cols;
  dst[transposed ? static_cast<size_t>(c) * rows + r : static_cast<size_t>(i)] = src[i];
}

struct Args {
  int n = 7168, k = 16384, iters = 200;
  std::vector<int> ms{1, 8, 64, 128};
  bool block = true;
};

Args parse(int argc, char** argv) {
  Args a;
  for (int i = 1; i < argc; ++i) {
    const std::string s = argv[i];
    auto next = [&]() -> std::string {
      if (i + 1 >= argc) {
        std::fprintf(stderr, "%s needs a value\n", s.c_str());
        std::exit(2);
      }
      return argv[++i];
    };
    if (s == "--n") {
      a.n = std::atoi(next().c_str());
    } else if (s == "--k") {
      a.k = std::atoi(next().c_str());
    } else if (s == "--iters") {
      a.iters = std::atoi(next().c_str());
    } else if (s == "--mode") {
      a.block = next() == "block";
    } else if (s == "--ms") {
      a.ms.clear();
      const std::string v = next();
      size_t p = 0;
      while (p < v.size()) {
        size_t q = v.find(',', p);
        if (q == std::string::npos) q = v.size();
        a.ms.push_back(std::atoi(v.substr(p, q - p).c_str()));
        p = q + 1;
      }
    } else {
      std::fprintf(stderr, "usage: dg_cublaslt_fp8 [--n N] [--k K] [--ms list] [--iters I] [--mode block|tensor]\n");
      std::exit(2);
    }
  }
  return a;
}

double rel_l2(const std::vector<float>& got, const std::vector<float>& want) {
  double d = 0.0, r = 0.0;
  for (size_t i = 0; i < got.size(); ++i) {
    const double e = static_cast<double>(got[i]) - want[i];
    d += e * e;
    r += static_cast<double>(want[i]) * want[i];
  }
  return std::sqrt(d / std::max(r, 1e-30));
}

}  // namespace

int main(int argc, char** argv) {
  const Args args = parse(argc, argv);
  const int N = args.n, K = args.k;
  if (N % 128 != 0 || K % 128 != 0 || N < 128 || args.ms.empty() || args.iters < 1) {
    std::fprintf(stderr, "N and K must be positive multiples of 128\n");
    return 2;
  }
  int dev = 0;
  CUDA_OK(cudaGetDevice(&dev));
  cudaDeviceProp prop{};
  CUDA_OK(cudaGetDeviceProperties(&prop, dev));
  const size_t w_bytes = static_cast<size_t>(N) * K;
  const size_t cold = std::max<size_t>(size_t(1) << 30, 4 * static_cast<size_t>(prop.l2CacheSize));
  const int sets = static_cast<int>(std::max<size_t>(5, (cold + w_bytes - 1) / w_bytes));
  const int kb = K / 128, nb = N / 128, m_max = *std::max_element(args.ms.begin(), args.ms.end());

  std::vector<uint8_t*> w(sets);
  for (int s = 0; s < sets; ++s) {
    CUDA_OK(cudaMalloc(&w[s], w_bytes));
    if (s == 0) fill_e4m3<<<1184, 256>>>(w[0], w_bytes, 0x1234567u);
    else CUDA_OK(cudaMemcpy(w[s], w[0], w_bytes, cudaMemcpyDeviceToDevice));
  }
  uint8_t* act = nullptr;
  float *w_s = nullptr, *a_s = nullptr, *w_s_l = nullptr, *a_s_l = nullptr, *ref = nullptr;
  __nv_bfloat16* out = nullptr;
  CUDA_OK(cudaMalloc(&act, static_cast<size_t>(m_max) * K));
  CUDA_OK(cudaMalloc(&w_s, sizeof(float) * nb * kb));
  CUDA_OK(cudaMalloc(&a_s, sizeof(float) * m_max * kb));
  CUDA_OK(cudaMalloc(&w_s_l, sizeof(float) * nb * kb));
  CUDA_OK(cudaMalloc(&a_s_l, sizeof(float) * m_max * kb));
  CUDA_OK(cudaMalloc(&ref, sizeof(float) * m_max * N));
  CUDA_OK(cudaMalloc(&out, sizeof(__nv_bfloat16) * m_max * N));
  fill_e4m3<<<256, 256>>>(act, static_cast<size_t>(m_max) * K, 0x89abcdu);
  const float one_64 = 1.0f / 64;
  if (args.block) {
    fill_scales<<<64, 256>>>(w_s, static_cast<size_t>(nb) * kb, 11u, 0.5f / 64, 1.0f / 64);
    fill_scales<<<64, 256>>>(a_s, static_cast<size_t>(m_max) * kb, 12u, 0.5f / 64, 1.0f / 64);
  } else {   // per-tensor: the reference product with every block scale equal
    fill_scales<<<64, 256>>>(w_s, static_cast<size_t>(nb) * kb, 0u, one_64, 0.0f);
    fill_scales<<<64, 256>>>(a_s, static_cast<size_t>(m_max) * kb, 0u, one_64, 0.0f);
  }
  float *w_scalar = nullptr, *a_scalar = nullptr;
  CUDA_OK(cudaMalloc(&w_scalar, sizeof(float)));
  CUDA_OK(cudaMalloc(&a_scalar, sizeof(float)));
  CUDA_OK(cudaMemcpy(w_scalar, &one_64, sizeof(float), cudaMemcpyHostToDevice));
  CUDA_OK(cudaMemcpy(a_scalar, &one_64, sizeof(float), cudaMemcpyHostToDevice));
  CUDA_OK(cudaDeviceSynchronize());

  cublasLtHandle_t lt;
  if (cublasLtCreate(&lt) != CUBLAS_STATUS_SUCCESS) return 2;
  const size_t ws_bytes = 64u << 20;
  void* workspace = nullptr;
  CUDA_OK(cudaMalloc(&workspace, ws_bytes));
  cudaStream_t stream;
  CUDA_OK(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  int major = 0, minor = 0, patch = 0;
  cublasLtGetProperty(MAJOR_VERSION, &major);
  cublasLtGetProperty(MINOR_VERSION, &minor);
  cublasLtGetProperty(PATCH_LEVEL, &patch);
  const std::string version = std::to_string(major) + "." + std::to_string(minor) + "." + std::to_string(patch);

  for (int M : args.ms) {
    const double alg_bytes = static_cast<double>(N) * K + static_cast<double>(M) * K + 2.0 * M * N;
    std::string line = "{\"M\": " + std::to_string(M) + ", \"N\": " + std::to_string(N) + ", \"K\": " +
                       std::to_string(K) + ", \"mode\": \"" + (args.block ? "block 128x128 / 1x128" : "per-tensor") +
                       "\", \"cublaslt\": \"" + version + "\"";
    reference_gemm<<<dim3((N + 127) / 128, M), 128>>>(act, w[0], a_s, w_s, ref, M, N, K);
    CUDA_OK(cudaDeviceSynchronize());
    std::vector<float> want(static_cast<size_t>(M) * N);
    CUDA_OK(cudaMemcpy(want.data(), ref, want.size() * sizeof(float), cudaMemcpyDeviceToHost));

    bool done = false;
    std::string why = "no candidate layout";
    // Candidate scale layouts (weights, activation): [rows][K/128] or [K/128][rows].
    for (int cand = 0; cand < (args.block ? 4 : 1) && !done; ++cand) {
      const int wt = cand & 1, at = (cand >> 1) & 1;
      if (args.block) {
        relayout<<<(nb * kb + 255) / 256, 256>>>(w_s, w_s_l, nb, kb, wt);
        relayout<<<(M * kb + 255) / 256, 256>>>(a_s, a_s_l, M, kb, at);
        CUDA_OK(cudaDeviceSynchronize());
      }
      cublasLtMatmulDesc_t desc;
      cublasLtMatmulDescCreate(&desc, CUBLAS_COMPUTE_32F, CUDA_R_32F);
      const cublasOperation_t opT = CUBLAS_OP_T, opN = CUBLAS_OP_N;
      cublasLtMatmulDescSetAttribute(desc, CUBLASLT_MATMUL_DESC_TRANSA, &opT, sizeof(opT));
      cublasLtMatmulDescSetAttribute(desc, CUBLASLT_MATMUL_DESC_TRANSB, &opN, sizeof(opN));
      const void* sa = args.block ? static_cast<const void*>(w_s_l) : static_cast<const void*>(w_scalar);
      const void* sb = args.block ? static_cast<const void*>(a_s_l) : static_cast<const void*>(a_scalar);
      cublasLtMatmulDescSetAttribute(desc, CUBLASLT_MATMUL_DESC_A_SCALE_POINTER, &sa, sizeof(sa));
      cublasLtMatmulDescSetAttribute(desc, CUBLASLT_MATMUL_DESC_B_SCALE_POINTER, &sb, sizeof(sb));
      if (args.block) {
        const int32_t ma = CUBLASLT_MATMUL_MATRIX_SCALE_BLK128x128_32F, mb = CUBLASLT_MATMUL_MATRIX_SCALE_VEC128_32F;
        cublasLtMatmulDescSetAttribute(desc, CUBLASLT_MATMUL_DESC_A_SCALE_MODE, &ma, sizeof(ma));
        cublasLtMatmulDescSetAttribute(desc, CUBLASLT_MATMUL_DESC_B_SCALE_MODE, &mb, sizeof(mb));
      }
      cublasLtMatrixLayout_t la, lb, lc;
      cublasLtMatrixLayoutCreate(&la, CUDA_R_8F_E4M3, K, N, K);
      cublasLtMatrixLayoutCreate(&lb, CUDA_R_8F_E4M3, K, M, K);
      cublasLtMatrixLayoutCreate(&lc, CUDA_R_16BF, N, M, N);
      cublasLtMatmulPreference_t pref;
      cublasLtMatmulPreferenceCreate(&pref);
      cublasLtMatmulPreferenceSetAttribute(pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws_bytes,
                                           sizeof(ws_bytes));
      cublasLtMatmulHeuristicResult_t heur[8];
      int found = 0;
      const cublasStatus_t hs = cublasLtMatmulAlgoGetHeuristic(lt, desc, la, lb, lc, lc, pref, 8, heur, &found);
      const float alpha = 1.0f, beta = 0.0f;
      if (hs != CUBLAS_STATUS_SUCCESS || found == 0) {
        why = "cublasLtMatmulAlgoGetHeuristic found no algorithm (cublasStatus " +
              std::to_string(static_cast<int>(hs)) + ")";
      } else {
        auto run = [&](int set) {
          return cublasLtMatmul(lt, desc, &alpha, w[set], la, act, lb, &beta, out, lc, out, lc, &heur[0].algo,
                                workspace, ws_bytes, stream);
        };
        const cublasStatus_t st = run(0);
        CUDA_OK(cudaStreamSynchronize(stream));
        if (st != CUBLAS_STATUS_SUCCESS) {
          why = "cublasLtMatmul failed (cublasStatus " + std::to_string(static_cast<int>(st)) + ")";
        } else {
          std::vector<__nv_bfloat16> got_b(static_cast<size_t>(M) * N);
          CUDA_OK(cudaMemcpy(got_b.data(), out, got_b.size() * sizeof(__nv_bfloat16), cudaMemcpyDeviceToHost));
          std::vector<float> got(got_b.size());
          for (size_t i = 0; i < got.size(); ++i) got[i] = __bfloat162float(got_b[i]);
          const double rl2 = rel_l2(got, want);
          if (!(rl2 <= 2e-3)) {
            why = "output does not match the reference (rel_l2 " + std::to_string(rl2) + ")";
          } else {
            for (int i = 0; i < 3; ++i) run(i % sets);
            CUDA_OK(cudaStreamSynchronize(stream));
            cudaGraph_t graph;
            cudaGraphExec_t exec;
            CUDA_OK(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
            for (int i = 0; i < args.iters; ++i) run(i % sets);
            CUDA_OK(cudaStreamEndCapture(stream, &graph));
            CUDA_OK(cudaGraphInstantiate(&exec, graph, 0));
            CUDA_OK(cudaGraphLaunch(exec, stream));   // warm
            CUDA_OK(cudaStreamSynchronize(stream));
            cudaEvent_t e0, e1;
            CUDA_OK(cudaEventCreate(&e0));
            CUDA_OK(cudaEventCreate(&e1));
            float best = 1e30f;
            for (int r = 0; r < 3; ++r) {
              CUDA_OK(cudaEventRecord(e0, stream));
              CUDA_OK(cudaGraphLaunch(exec, stream));
              CUDA_OK(cudaEventRecord(e1, stream));
              CUDA_OK(cudaEventSynchronize(e1));
              float ms = 0.0f;
              CUDA_OK(cudaEventElapsedTime(&ms, e0, e1));
              best = std::min(best, ms);
            }
            const double us = best * 1e3 / args.iters;
            char buf[512];
            std::snprintf(buf, sizeof(buf),
                          ", \"us_per_gemm\": %.4f, \"GBps\": %.1f, \"rel_l2\": %.3e, \"weight_sets\": %d, "
                          "\"iters\": %d, \"algo_workspace\": %zu, \"scale_layout\": \"weights %s, activation %s\"",
                          us, alg_bytes / us / 1e3, rl2, sets, args.iters, heur[0].workspaceSize,
                          args.block ? (wt ? "[K/128][N/128]" : "[N/128][K/128]") : "scalar",
                          args.block ? (at ? "[K/128][M]" : "[M][K/128]") : "scalar");
            line += buf;
            cudaEventDestroy(e0);
            cudaEventDestroy(e1);
            cudaGraphExecDestroy(exec);
            cudaGraphDestroy(graph);
            done = true;
          }
        }
      }
      cublasLtMatmulPreferenceDestroy(pref);
      cublasLtMatrixLayoutDestroy(la);
      cublasLtMatrixLayoutDestroy(lb);
      cublasLtMatrixLayoutDestroy(lc);
      cublasLtMatmulDescDestroy(desc);
    }
    if (!done) line += ", \"unavailable\": \"" + why + "\"";
    line += "}";
    std::printf("%s\n", line.c_str());
    std::fflush(stdout);
  }
  return 0;
}
