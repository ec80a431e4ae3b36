/* A plain C99 consumer of include/b200tx.h: what a caller outside Python
 * (a C program, or another language's FFI generated from this header) sees.
 * It checks the ABI version and that argument errors come back as negative
 * status codes with a message, before any device work -- so it runs on a
 * machine without a GPU.  Built and run by tests/test_c_abi.py. */
#include <stdio.h>
#include <string.h>

#include "b200tx.h"

static int expect(int rc, int want, const char* fragment, const char* what) {
  const char* msg = b200tx_last_error();
  if (rc != want || strstr(msg, fragment) == NULL) {
    fprintf(stderr, "%s: rc=%d (want %d) message=\"%s\" (want \"%s\")\n", what, rc, want, msg,
            fragment);
    return 1;
  }
  return 0;
}

int main(void) {
  char buf[256];
  int failures = 0;
  printf("abi %d\n", b200tx_abi_version());
  failures += expect(b200tx_linear(NULL, NULL, NULL, NULL, B200TX_BF16, 128, 256, 64,
                                   B200TX_EPI_BIAS, NULL),
                     B200TX_ERR_INVALID_ARGUMENT, "null", "linear null pointers");
  failures += expect(b200tx_linear(buf, buf, NULL, buf, B200TX_BF16, 16, 20, 64, B200TX_EPI_BIAS,
                                   NULL),
                     B200TX_ERR_UNSUPPORTED, "multiples of 8", "linear N % 8");
  failures += expect(b200tx_attention(buf, buf, 1, 128, 1, 128, 0.125f, 1, NULL),
                     B200TX_ERR_UNSUPPORTED, "head_dim", "attention head_dim");
  failures += expect(b200tx_attention_ex(buf, buf, 1, 128, 1, 64, 0.125f, 1, 7, NULL),
                     B200TX_ERR_INVALID_ARGUMENT, "variant", "attention variant");
  failures += expect(b200tx_residual_layer_norm(buf, 5, NULL, B200TX_F32, NULL, buf, B200TX_BF16,
                                                (const float*)buf, (const float*)buf, 4, 8, 1e-5f,
                                                NULL),
                     B200TX_ERR_INVALID_ARGUMENT, "in_dtype", "layer norm dtype");
  if (failures == 0) printf("ok\n");
  return failures == 0 ? 0 : 1;
}
