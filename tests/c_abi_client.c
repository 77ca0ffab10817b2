/* A plain C99 client of libcudabridge.so, built and run by tests/test_abi.py: it shows
 * that include/cuda_bridge.h is valid C (no C++ needed by a caller such as a Rust or
 * cgo binding) and that the library links and answers host-only calls without a GPU. */
#include <stdio.h>
#include <string.h>

#include "cuda_bridge.h"

static int failures = 0;

static void expect(int cond, const char* what) {
  if (!cond) {
    fprintf(stderr, "FAILED: %s\n", what);
    ++failures;
  }
}

int main(void) {
  int32_t n = -1, info[8];
  cb_ctx* ctx = NULL;
  cb_model_config bad = {1536, 4096, 12, 12, 64, 512, 20, 8192}; /* hd != 128 */
  cb_model_config ok = {6656, 17920, 52, 52, 128, 2048, 60, 8192};

  printf("version %s\n", cb_version());
  expect(strstr(cb_version(), "sm_100a") != NULL, "version names sm_100a");
  expect(cb_device_count(&n) == CB_OK && n >= 0, "device count");
  printf("devices %d\n", n);

  expect(cb_create(&bad, 0, 1, &ctx) == CB_ERR_INVALID_ARG && ctx == NULL, "bad config rejected");
  expect(strlen(cb_create_error()) > 0, "create error describes the rejection");
  printf("create error: %s\n", cb_create_error());

  /* the tensor-parallel split of the ~32B shape over 8 ranks: rank 4 holds heads 28..33 */
  expect(cb_tp_partition(&ok, 8, 4, info) == CB_OK, "tp partition");
  expect(info[2] == 6 && info[5] == 28 && info[4] == 2240, "rank 4 share");
  expect(cb_tp_partition(&ok, 8, 8, info) == CB_ERR_INVALID_ARG, "rank out of range");

  expect(cb_last_error(NULL) != NULL, "null context message");
  expect(cb_forward_loss(NULL, NULL, NULL, 1, 0.0f, NULL, NULL) == CB_ERR_INVALID_ARG,
         "null context forward");
  if (n == 0) {
    expect(cb_create(&ok, 0, 1, &ctx) == CB_ERR_UNSUPPORTED && ctx == NULL,
           "no device: create fails loudly");
    printf("create without a GPU: %s\n", cb_create_error());
  }
  expect(cb_destroy(NULL) == CB_OK, "destroy(NULL)");
  printf(failures ? "c client: %d failure(s)\n" : "c client: ok\n", failures);
  return failures ? 1 : 0;
}
