/* dg_c_caller.c -- a plain C99 caller of the C ABI (include/decode_gemm_b200.h),
 * compiled by tests/test_c_caller.py with gcc: version, layout geometry,
 * status strings, the C2 default plan (cluster split-K, 224-row tiles x 4
 * splits, no workspace) and the rejections -- none of which needs a GPU.
 * Prints one line per check; exits 0 only when every check passed. */
#include <stdio.h>
#include <string.h>

#include "decode_gemm_b200.h"

static int failures = 0;

static void check(int ok, const char* what) {
  printf("%s %s\n", ok ? "ok  " : "FAIL", what);
  if (!ok) ++failures;
}

int main(void) {
  dg_config cfg;
  dg_plan_info info;

  check(dg_abi_version() == DG_ABI_VERSION, "ABI version matches the header");
  check(dg_padded_n(7168, 56) == 7168 && dg_padded_n(100, 64) == 128, "dg_padded_n");
  check(dg_packed_weight_bytes(100, 256, 64) == 128ull * 256ull, "dg_packed_weight_bytes");
  check(dg_status_string(0) != NULL && dg_status_string(0)[0] != '\0', "status string of 0");

  memset(&cfg, 0, sizeof(cfg));
  cfg.m_tile = 8;
  cfg.block_n = 224;
  cfg.subs = 2;
  cfg.stages = 0;
  cfg.layout = DG_LAYOUT_PACKED_SWIZZLED;
  cfg.pdl = 1;
  cfg.split_k = 4;
  cfg.grid_ctas = DG_GRID_CLUSTER;
  check(dg_plan(&cfg, 1, 7168, 16384, &info) == 0 && info.error[0] == '\0', "C2 M=1 cluster plan");
  check(info.grid_x == 32 && info.grid_y == 4 && info.cluster == 4 && info.num_ctas == 128, "grid 32 x 4, cluster 4");
  check(info.mma_m == 64 && info.stages == 3 && info.smem_bytes <= 227u * 1024u, "MMA M 64, three stages, fits");
  check(info.ws_floats == 0 && info.sem_ints == 0, "no workspace");

  check(dg_plan(&cfg, 1, 7168, 16000, &info) != 0 && info.error[0] != '\0', "K not a multiple of 128 rejected");
  cfg.m_tile = 12;
  check(dg_plan(&cfg, 1, 7168, 16384, &info) != 0, "m_tile 12 rejected");
  check(dg_plan(NULL, 1, 7168, 16384, &info) != 0, "NULL config rejected");
  check(dg_launch(NULL, NULL, NULL) != 0, "NULL launch rejected before touching a GPU");

  printf("%d failure(s)\n", failures);
  return failures == 0 ? 0 : 1;
}
