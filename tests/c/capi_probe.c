/* Plain-C caller of the C ABI (include/flashact.h): creates a pi0.5 handle with the BASELINE
 * geometry and, without a GPU, expects a clean failure status and message (no crash, no
 * exception across the ABI). With a GPU it also loads nothing and destroys the handle.
 * Exit 0 on the expected behaviour. Built and run by tests/test_capi.py. */
#include <stdio.h>
#include <string.h>

#include "flashact.h"

int main(int argc, char** argv) {
  const int expect_gpu = argc > 1 && strcmp(argv[1], "gpu") == 0;
  fa_config cfg = {18, 1024, 8, 1, 256, 4096, 50, 32, 968, 1, 10, 0};
  fa_handle* h = NULL;
  fa_status st = fa_create(FA_MODEL_PI05, &cfg, 0, &h);
  if (!expect_gpu) {
    if (st == FA_OK || h != NULL) {
      fprintf(stderr, "fa_create succeeded without a GPU\n");
      return 1;
    }
    const char* msg = fa_last_error(NULL);
    printf("status %d: %s\n", (int)st, msg ? msg : "(null)");
    return (msg && msg[0]) ? 0 : 2;
  }
  if (st != FA_OK) {
    fprintf(stderr, "fa_create failed: %s\n", fa_last_error(NULL));
    return 3;
  }
  /* sampling before any weights must be refused with FA_ERR_STATE */
  float noise[50 * 32] = {0}, out[50 * 32];
  st = fa_sample_actions(h, 1, noise, out, NULL);
  printf("sample before load: status %d (%s)\n", (int)st, fa_last_error(h));
  fa_destroy(h);
  return st == FA_ERR_STATE ? 0 : 4;
}
