// dg_plan_smem_check.cu -- host-only check of the planner's shared-memory
// accounting (csrc/dg_host.cuh make_plan) against the kernel's carve-up
// (csrc/dg_kernel.cuh decode_gemm_body): 1 KiB alignment slack, the weight
// ring (w_region_bytes, tail pad included), the activation ring
// (a_region_bytes) and the barrier block of the class's accumulator buffers.
// For every plan that the planner accepts over batch classes (the default
// ones and swap-AB), M, tile widths, stage depths and layouts it requires
//   * smem_bytes == 1024 + w_region_bytes + a_region_bytes + barriers,
//   * smem_bytes <= 227 KiB,
//   * the last weight rows any MMA reads (n_mma rows of the ring's last
//     128-K block, 256 for the swap class's two 128-row halves) inside the
//     carve-up (inside the weight ring for the swap class).
// No kernel is referenced, so nothing runs on a GPU.
#include <cstdio>

#include "dg_host.cuh"

int main() {
  int bad = 0;
  int checked = 0;
  for (int swap = 0; swap < 2; ++swap)
    for (int M : {1, 5, 8, 16, 32, 64, 128})
      for (int bn = 8; bn <= 256; bn += 8)
        for (int subs : {1, 2, 4})
          for (int stages = 0; stages <= 6; ++stages)
            for (int layout = 0; layout < 3; ++layout) {
              dg::Config c;
              c.m_tile = M <= 8 ? 8 : (M <= 16 ? 16 : M);
              c.block_n = bn;
              c.subs = subs;
              c.stages = stages;
              c.layout = layout;
              c.grid_ctas = dg::kGridCluster;
              c.split_k = 2;
              c.flags = swap ? dg::kFlagSwapAB : 0;
              const dg::Plan p = dg::make_plan(c, M, 7168, 16384, 148);
              if (p.error != nullptr) continue;
              ++checked;
              const dg::KernelParams& q = p.params;
              const int bufs = swap ? dg::SwapTraits::kNumBufs : dg::kAccumBuffers;
              const unsigned want =
                  1024u + q.w_region_bytes + q.a_region_bytes + dg::SmemBarriers::bytes(q.stages, bufs);
              const unsigned rows_read = swap ? 2u * dg::SwapTraits::kMmaM : static_cast<unsigned>(q.n_mma);
              const unsigned last_end =
                  (static_cast<unsigned>((q.stages * q.subs - 1) * q.block_n) + rows_read) * 128u;
              const bool ok = q.smem_bytes == want && q.smem_bytes <= dg::kMaxDynamicSmem &&
                              last_end <= q.w_region_bytes + q.a_region_bytes &&
                              (!swap || last_end <= q.w_region_bytes);
              if (!ok && bad++ < 10)
                std::printf("mismatch: swap=%d M=%d block_n=%d subs=%d stages=%d layout=%d smem=%u want=%u\n", swap,
                            M, bn, subs, q.stages, layout, q.smem_bytes, want);
            }
  std::printf("%d plans checked, %d failure(s)\n", checked, bad);
  return bad == 0 && checked > 1000 ? 0 : 1;
}
