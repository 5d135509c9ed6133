/* Calls the libb2x C ABI from plain C (no Python, no torch): library
 * version, argument validation and error messages, workspace queries and
 * default configuration.  Launches nothing, so it runs without a GPU.
 * Exit code 0 when every check holds; prints the failing check otherwise. */
#include <stdio.h>
#include <string.h>
#include "b2x.h"

static int failures = 0;
#define CHECK(cond)                                              \
  do {                                                           \
    if (!(cond)) {                                               \
      fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
      ++failures;                                                \
    }                                                            \
  } while (0)

int main(void) {
  CHECK(b2x_abi_version() == B2X_ABI_VERSION);

  b2x_gemm_args g;
  memset(&g, 0, sizeof(g));
  g.a = (const void*)0x10000;
  g.b = (const void*)0x20000;
  g.c = (void*)0x30000;
  g.M = 512;
  g.N = 512;
  g.K = 512;
  g.lda = 512;
  g.ldb_k = 1;
  g.ldb_n = 512;
  g.ldc = 512;
  g.a_type = B2X_E4M3;
  g.b_type = B2X_E4M3;
  g.c_type = B2X_BF16;
  g.scale_mode = B2X_SCALE_NONE;

  /* invalid requests come back as status codes with a message */
  b2x_gemm_args bad = g;
  bad.lda = 100;
  CHECK(b2x_fp8_gemm(&bad, NULL) == B2X_ERR_INVALID_ARG);
  CHECK(strlen(b2x_last_error()) > 0);
  bad = g;
  bad.c_type = B2X_E4M3;
  CHECK(b2x_fp8_gemm(&bad, NULL) == B2X_ERR_UNSUPPORTED);
  CHECK(b2x_fp8_gemm(NULL, NULL) == B2X_ERR_INVALID_ARG);

  /* workspace queries */
  CHECK(b2x_gemm_workspace_size(&g) == 0);
  bad = g;
  bad.config.split_k = 2;
  CHECK(b2x_gemm_workspace_size(&bad) >= (size_t)512 * 512 * 4);
  CHECK(b2x_fp8_gemm(&bad, NULL) == B2X_ERR_WORKSPACE);
  CHECK(b2x_grouped_gemm_workspace_size(4) > 0);
  CHECK(b2x_allreduce_signal_words(8192, 8192) == 64 + 64 * 32);

  /* the default configuration fills every field */
  b2x_gemm_config c;
  CHECK(b2x_gemm_default_config(&g, &c) == B2X_OK);
  CHECK(c.block_m == 128 && c.block_k == 128 && c.block_n > 0 && c.split_k >= 1 && c.group_size_m >= 1);

  /* casts, stochastic rounding, split-K reduce: argument checks */
  b2x_cast_args ca;
  memset(&ca, 0, sizeof(ca));
  ca.x = (const void*)0x10000;
  ca.x_type = B2X_F16;
  ca.rows = 4;
  ca.cols = 256;
  ca.ld_x = 256;
  ca.q = (void*)0x20000;
  ca.q_type = B2X_E4M3;
  ca.ld_q = 256;
  ca.mode = B2X_SCALE_NONE;
  CHECK(b2x_fp8_cast(&ca, NULL) == B2X_ERR_UNSUPPORTED);
  CHECK(b2x_stoch_round((const float*)0x10000, 4, 8, 8, (const uint32_t*)0x20000, 8, (void*)0x30000, B2X_F32, 8,
                        NULL) == B2X_ERR_UNSUPPORTED);
  CHECK(b2x_stoch_round((const float*)0x10000, 4, 8, 4, (const uint32_t*)0x20000, 8, (void*)0x30000, B2X_E4M3, 8,
                        NULL) == B2X_ERR_INVALID_ARG);
  CHECK(b2x_splitk_reduce(NULL, B2X_F32, (void*)0x1000, B2X_BF16, 4, 4, 4, 2, NULL) == B2X_ERR_INVALID_ARG);

  if (failures == 0) printf("abi_from_c: all checks passed\n");
  return failures == 0 ? 0 : 1;
}
