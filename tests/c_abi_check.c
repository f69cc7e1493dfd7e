/* Plain C99 caller of include/vllm_exact_b200.h, compiled and run by tests/test_capi_host.py without a GPU: the
 * header must be valid C (the C ABI a cgo / JNI / ctypes / N-API binding would consume) and the library must link.
 * Only entry points that answer before touching a device are called. Prints "OK" and exits 0 on success. */
#include <stdio.h>
#include <string.h>

#include "vllm_exact_b200.h"

int main(void) {
  const char* v = ex_version();
  if (!v || !strstr(v, "sm_100a")) return 1;
  if (strcmp(ex_status_string(EX_OK), "ok") != 0) return 2;
  /* a negative row count is rejected before any launch */
  if (ex_digitize((const void*)16, EX_DTYPE_BF16, 64, -1, 64, 14, (void*)16, (void*)16, 64, (int32_t*)16,
                  (int32_t*)16, NULL) != EX_ERR_ARG)
    return 3;
  /* an empty batch is a no-op */
  if (ex_linear(NULL, NULL, 64, NULL, NULL, NULL, NULL, 64, NULL, NULL, 0, 8, 64, 14, 1, NULL, EX_DTYPE_BF16, 8,
                NULL, 0, 0, EX_ALGO_AUTO, NULL) != EX_OK)
    return 4;
  if (ex_paged_decode_workspace_bytes(2, 32, 128, 4096, 4096) == 0) return 5;
  printf("OK\n");
  return 0;
}
