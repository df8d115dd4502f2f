/* A plain-C caller of libkda.so (no Python, no torch): the way a cgo / JNI /
 * N-API binding would use the C ABI.  It runs without a GPU: it checks the ABI
 * version and status strings, the workspace-size queries, and that invalid
 * arguments are rejected on the host with KDA_INVALID_ARG before any CUDA call.
 * Built and run by tests/test_abi.py; exit code 0 = every check passed. */
#include <stdio.h>
#include <string.h>

#include "kda.h"

static int failures = 0;
#define CHECK(cond)                                              \
  do {                                                           \
    if (!(cond)) {                                               \
      fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
      ++failures;                                                \
    }                                                            \
  } while (0)

int main(void) {
  CHECK(kda_abi_version() == KDA_ABI_VERSION);
  CHECK(strcmp(kda_status_string(KDA_OK), "KDA_OK") == 0);
  CHECK(strcmp(kda_status_string(KDA_INVALID_ARG), "KDA_INVALID_ARG") == 0);

  /* workspace queries: pure host arithmetic */
  CHECK(kda_rmsnorm_matmul_workspace_size(4096, 4096, 11008) >= (size_t)4096 * 4096 * 2);
  CHECK(kda_matmul_f32_workspace_size(64, 64, 64) == 4 * 8192);
  CHECK(kda_bmm_f32_workspace_size(0, 16, 16, 16) == 0);
  CHECK(kda_swiglu_backward_workspace_size(8, 8, 8) > 0);
  CHECK(kda_gqa_full_backward_workspace_size(1, 16, 2, 1, 128, 0.0f) > 0);
  CHECK(kda_ipc_handle_size() >= 64);

  /* invalid arguments: rejected before any launch, with a message */
  CHECK(kda_silu_f32(NULL, NULL, 16, NULL) == KDA_INVALID_ARG);
  CHECK(strlen(kda_last_error()) > 0);
  CHECK(kda_matmul_bf16(NULL, NULL, NULL, 16, 16, 16, NULL) == KDA_INVALID_ARG);
  CHECK(kda_matmul_f32(NULL, NULL, NULL, 0, 16, 16, NULL, 0, NULL) == KDA_INVALID_ARG);
  CHECK(kda_adamw_multi_f32(NULL, NULL, NULL, NULL, NULL, 1, 1e-3, 0.9, 0.999, 1e-8, 1e-2, 1, NULL) ==
        KDA_INVALID_ARG);
  CHECK(kda_zero1_adamw_f32(NULL, NULL, 9, 0, 0, 4, NULL, NULL, 1e-3, 0.9, 0.999, 1e-8, 1e-2, 1, NULL) ==
        KDA_INVALID_ARG);
  CHECK(kda_gqa_full_backward_bf16(NULL, NULL, NULL, NULL, NULL, NULL, NULL, 1, 16, 3, 2, 128, 0, 0.0f, NULL, 0,
                                   NULL) == KDA_INVALID_ARG);
  if (failures == 0) printf("abi host checks: OK\n");
  return failures == 0 ? 0 : 1;
}
