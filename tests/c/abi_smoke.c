/* A plain C host against the library: include/duplex_b200.h must compile as C99, and
 * libduplex_b200.so must link and answer without a GPU (version, error strings, and
 * argument rejection, which happens before any CUDA call).  Built and run by
 * tests/test_abi.py::test_plain_c_host_links_and_calls_the_library. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "duplex_b200.h"

static int failures = 0;

static void expect(int got, int want, const char* what) {
  if (got != want) {
    printf("FAIL %s: got %d, want %d\n", what, got, want);
    ++failures;
  }
}

int main(void) {
  void* p = (void*)(uintptr_t)(1u << 20); /* aligned, never dereferenced */
  size_t n = 0;
  expect(duplex_version() >= 100, 1, "duplex_version");
  expect(strlen(duplex_error_string(DUPLEX_ERR_ARG)) > 0, 1, "duplex_error_string");
  expect(duplex_tile_record_bytes(2048, 128, 1, &n), DUPLEX_OK, "duplex_tile_record_bytes");
  expect((int)n, 16384 + 16 * 32 + 16 * 8, "record bytes, K 2048, group 128, zero points");
  expect(duplex_moe_workspace_bytes(1, 128, 2048, 768, 8, &n), DUPLEX_OK,
         "duplex_moe_workspace_bytes");
  expect(duplex_moe_forward(p, DUPLEX_DTYPE_F16, 9, p, NULL, 128, 2048, 768, 8, 1, p, p,
                            DUPLEX_DTYPE_F16, 1, 128, NULL, p, NULL, NULL, p, n, NULL, 0.0f, 1,
                            NULL),
         DUPLEX_ERR_ARG, "duplex_moe_forward with 9 tokens");
  expect(duplex_moe_forward_noalloc(p, DUPLEX_DTYPE_F16, 8, p, NULL, 256, 4096, 4096, 8, 1, p,
                                    p, DUPLEX_DTYPE_F16, 1, 128, NULL, p, NULL, NULL, NULL, 0.0f,
                                    0, NULL),
         DUPLEX_ERR_SCRATCH_LIMIT, "duplex_moe_forward_noalloc beyond its scratch");
  expect(duplex_moe_stage_bytes(9, 128, 2048, 768, 8, 128, 1, &n), DUPLEX_ERR_ARG,
         "duplex_moe_stage_bytes with 9 tokens");
  expect(duplex_ep_wait(p, p, 0, 0, p, NULL), DUPLEX_ERR_ARG, "duplex_ep_wait with no ranks");
  if (failures == 0) printf("ok\n");
  return failures ? 1 : 0;
}
