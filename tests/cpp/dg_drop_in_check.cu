// SPDX-License-Identifier: MIT
//
// dg_drop_in_check.cu -- exercises the C++ interface (include/decode_gemm.cuh,
// include/weight_prepack.cuh) the way the reference's smoke test and bench
// use theirs: for every KernelConfig below that accepts the case's M it runs
//   1. decode_gemm::launch<Cfg>(problem, stream)
//   2. decode_gemm::launch_with_maps<Cfg>(problem, w_map, a_map, stream)
//   3. cudaLaunchKernelEx(decode_gemm::fp8_decode_gemm<Cfg>, ...) with the
//      grid / block / shared memory of make_launch_plan<Cfg>, after
//      ensure_smem_attribute<Cfg> -- the bench's direct launch
// and writes launch 1's bf16 output to <dir>/out_<name>.bin, with one JSON
// line per configuration on stdout (return codes, whether the three outputs
// are bit-identical).  The case comes from <dir>: meta.txt ("M N K"),
// w.bin (N x K e4m3), ws.bin (ceil(N/128) x K/128 fp32), a.bin (M x K),
// as.bin (M x K/128 fp32); tests/test_drop_in_gpu.py writes them from the
// oracle and checks the outputs against it.

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "decode_gemm.cuh"
#include "weight_prepack.cuh"

namespace {

using namespace decode_gemm;

// M_TILE 8: the reference's S0 canonical configuration (raw weights, no PDL).
using CfgS0 = KernelConfig<8, 64, 4, 112, 2, 1, 1, false, false, false, false>;
// M_TILE 8: BM 56, packed weights, PDL, 2-way split-K.
using CfgS5 = KernelConfig<8, 56, 2, 80, 3, 1, 2, true, true, false, true>;
// M_TILE 32: packed, PDL, SPLITK_FACTOR 4.
using CfgM32 = KernelConfig<32, 64, 2, 168, 2, 2, 2, true, true, false, false, 32, false, false, false, 4>;
// M_TILE 64: 256-row tiles (B200 width), packed.
using CfgM64 = KernelConfig<64, 256, 1, 112, 2, 1, 2, true, false, false, false>;
// M_TILE 128: 128-row tiles, raw, EPI_OVERLAP trigger without the PDL attribute.
using CfgM128 = KernelConfig<128, 128, 1, 232, 2, 1, 1, false, false, true, false>;

#define CHECK(x)                                                                             \
  do {                                                                                       \
    const cudaError_t e_ = (x);                                                              \
    if (e_ != cudaSuccess) {                                                                 \
      std::fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
      std::exit(2);                                                                          \
    }                                                                                        \
  } while (0)

std::vector<char> read_file(const std::string& path) {
  std::vector<char> out;
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) {
    std::fprintf(stderr, "cannot open %s\n", path.c_str());
    std::exit(2);
  }
  std::fseek(f, 0, SEEK_END);
  const long n = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  out.resize(static_cast<size_t>(n));
  if (n > 0 && std::fread(out.data(), 1, out.size(), f) != out.size()) std::exit(2);
  std::fclose(f);
  return out;
}

template <typename T>
T* to_device(const std::vector<char>& host) {
  void* d = nullptr;
  CHECK(cudaMalloc(&d, host.size() ? host.size() : 16));
  CHECK(cudaMemcpy(d, host.data(), host.size(), cudaMemcpyHostToDevice));
  return static_cast<T*>(d);
}

struct Case {
  int M = 0, N = 0, K = 0;
  __nv_fp8_e4m3* w = nullptr;
  float* ws = nullptr;
  __nv_fp8_e4m3* a = nullptr;
  float* as = nullptr;
};

template <typename Cfg>
void run(const char* name, const Case& c, const std::string& dir, cudaStream_t stream) {
  if (Cfg::validate(c.M, c.N, c.K) != nullptr) return;
  // Weights in the configuration's layout.
  __nv_fp8_e4m3* weight = c.w;
  __nv_fp8_e4m3* packed = nullptr;
  if (Cfg::kPrepack) {
    CHECK(cudaMalloc(&packed, prepack::packed_weight_bytes(c.N, c.K, Cfg::kOutputRows)));
    CHECK((prepack::launch_prepack_weight<Cfg::kOutputRows, Cfg::kOutputTilesPerCta>(c.w, packed, c.N, c.K,
                                                                                    stream)));
    weight = packed;
  }
  const size_t out_elems = static_cast<size_t>(c.M) * c.N;
  __nv_bfloat16* out[3] = {nullptr, nullptr, nullptr};
  for (auto& o : out) CHECK(cudaMalloc(&o, out_elems * sizeof(__nv_bfloat16)));
  float* ws = nullptr;
  int* sem = nullptr;
  if (Cfg::kSplitKCta) {
    CHECK(cudaMalloc(&ws, static_cast<size_t>(Cfg::kSplitKFactor) * out_elems * sizeof(float)));
    CHECK(cudaMalloc(&sem, Cfg::num_output_tiles(c.N) * sizeof(int)));
    CHECK(cudaMemset(sem, 0, Cfg::num_output_tiles(c.N) * sizeof(int)));
  }
  Problem p;
  p.M = c.M;
  p.N = c.N;
  p.K = c.K;
  p.activation = c.a;
  p.weight = weight;
  p.weight_scales = c.ws;
  p.activation_scales = c.as;
  p.splitk_ws = ws;
  p.splitk_sem = sem;

  int rc[3];
  p.output = out[0];
  rc[0] = launch<Cfg>(p, stream);

  p.output = out[1];
  const CUtensorMap w_map = make_weight_tma<Cfg>(p);
  const CUtensorMap a_map = make_activation_tma<Cfg>(p);
  rc[1] = launch_with_maps<Cfg>(p, w_map, a_map, stream);

  p.output = out[2];
  const LaunchPlan plan = make_launch_plan<Cfg>(p);
  rc[2] = plan.error != nullptr ? cudaErrorInvalidValue : ensure_smem_attribute<Cfg>(plan.smem_bytes);
  if (rc[2] == cudaSuccess) {
    GemmRuntime rt;
    rt.M = p.M;
    rt.N = p.N;
    rt.K = p.K;
    rt.splitk_ws = p.splitk_ws;
    rt.splitk_sem = p.splitk_sem;
    cudaLaunchConfig_t config{};
    cudaLaunchAttribute attributes[1]{};
    config.gridDim = plan.grid;
    config.blockDim = plan.block;
    config.dynamicSmemBytes = plan.smem_bytes;
    config.stream = stream;
    config.attrs = attributes;
    config.numAttrs = 0;
    if (Cfg::kPdl) {
      attributes[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      attributes[0].val.programmaticStreamSerializationAllowed = 1;
      config.numAttrs = 1;
    }
    rc[2] = cudaLaunchKernelEx(&config, fp8_decode_gemm<Cfg>, p.output, p.weight_scales, p.activation_scales,
                               w_map, a_map, rt);
  }
  CHECK(cudaStreamSynchronize(stream));
  CHECK(cudaGetLastError());

  std::vector<__nv_bfloat16> host[3];
  for (int i = 0; i < 3; ++i) {
    host[i].resize(out_elems);
    CHECK(cudaMemcpy(host[i].data(), out[i], out_elems * sizeof(__nv_bfloat16), cudaMemcpyDeviceToHost));
  }
  const bool eq12 = std::memcmp(host[0].data(), host[1].data(), out_elems * 2) == 0;
  const bool eq13 = std::memcmp(host[0].data(), host[2].data(), out_elems * 2) == 0;
  int sem_dirty = 0;
  if (sem != nullptr) {
    std::vector<int> s(Cfg::num_output_tiles(c.N));
    CHECK(cudaMemcpy(s.data(), sem, s.size() * sizeof(int), cudaMemcpyDeviceToHost));
    for (int v : s) sem_dirty |= (v != 0);
  }
  const std::string path = dir + "/out_" + name + ".bin";
  FILE* f = std::fopen(path.c_str(), "wb");
  if (f == nullptr || std::fwrite(host[0].data(), 2, out_elems, f) != out_elems) std::exit(2);
  std::fclose(f);
  std::printf("{\"cfg\": \"%s\", \"m_tile\": %u, \"rc\": [%d, %d, %d], \"grid\": [%u, %u], \"block\": %u, "
              "\"smem\": %u, \"launch_eq_with_maps\": %s, \"launch_eq_direct\": %s, \"sem_clean\": %s}\n",
              name, Cfg::kMTile, rc[0], rc[1], rc[2], plan.grid.x, plan.grid.y, plan.block.x, plan.smem_bytes,
              eq12 ? "true" : "false", eq13 ? "true" : "false", sem_dirty ? "false" : "true");
  for (auto& o : out) cudaFree(o);
  if (packed) cudaFree(packed);
  if (ws) cudaFree(ws);
  if (sem) cudaFree(sem);
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 2) {
    std::fprintf(stderr, "usage: %s <case-dir>\n", argv[0]);
    return 2;
  }
  const std::string dir = argv[1];
  Case c;
  {
    const std::vector<char> meta = read_file(dir + "/meta.txt");
    const std::string s(meta.begin(), meta.end());
    if (std::sscanf(s.c_str(), "%d %d %d", &c.M, &c.N, &c.K) != 3) return 2;
  }
  c.w = to_device<__nv_fp8_e4m3>(read_file(dir + "/w.bin"));
  c.ws = to_device<float>(read_file(dir + "/ws.bin"));
  c.a = to_device<__nv_fp8_e4m3>(read_file(dir + "/a.bin"));
  c.as = to_device<float>(read_file(dir + "/as.bin"));
  cudaStream_t stream;
  CHECK(cudaStreamCreate(&stream));
  run<CfgS0>("s0_mt8", c, dir, stream);
  run<CfgS5>("s5_mt8_bm56_sk2", c, dir, stream);
  run<CfgM32>("mt32_sk4", c, dir, stream);
  run<CfgM64>("mt64_bm256", c, dir, stream);
  run<CfgM128>("mt128_bm128_epi", c, dir, stream);
  CHECK(cudaStreamDestroy(stream));
  return 0;
}
