/*
 * A plain C99 caller of libpa_b200.so: it includes include/pa_b200.h, links against the
 * library and exercises the host side of the ABI (version, status strings, argument checks,
 * size queries). Nothing here launches GPU work, so it runs on a machine without a GPU.
 * Built and run by tests/test_capi.py; exits 0 when every check holds and prints the first
 * failing check otherwise.
 */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "pa_b200.h"

static int failures = 0;

#define CHECK(cond)                                                 \
  do {                                                              \
    if (!(cond)) {                                                  \
      fprintf(stderr, "check failed (line %d): %s\n", __LINE__, #cond); \
      ++failures;                                                   \
    }                                                               \
  } while (0)

/* A non-null, 256-byte-aligned address that is never dereferenced: every call below is
 * rejected by its host-side checks before any device work. */
static void* fake(void) { return (void*)(uintptr_t)0x100000; }

static int decode_f16(int B, int H, int KVH, int D, int NB, int bs) {
  return pa_decode_f16(fake(), fake(), fake(), fake(), (const int32_t*)fake(),
                       (const int32_t*)fake(), B, H, KVH, D, NB, bs, 2, 0.1f, fake(),
                       (size_t)1 << 30, NULL);
}

int main(void) {
  CHECK(pa_version() >= 100);
  CHECK(strcmp(pa_status_string(PA_OK), "ok") == 0);
  CHECK(strstr(pa_status_string(PA_ERR_TIMEOUT), "timed out") != NULL);
  CHECK(strstr(pa_status_string(PA_ERR_BLOCK_ID | PA_ERR_SLOT), "block_table") != NULL);

  /* Shape checks of the reference's launchers, plus this build's own limits. */
  CHECK(decode_f16(1, 8, 2, 64, 4, 16) == PA_ERR_UNSUPPORTED);
  CHECK(strstr(pa_last_error(), "head_dim") != NULL);
  CHECK(decode_f16(1, 7, 2, 128, 4, 16) == PA_ERR_INVALID_ARG);
  CHECK(decode_f16(1, 8, 2, 128, 4, 8) == PA_ERR_INVALID_ARG);
  CHECK(strstr(pa_last_error(), "block_size") != NULL);
  CHECK(decode_f16(1, 8, 0, 128, 4, 16) == PA_ERR_INVALID_ARG);
  CHECK(decode_f16(1, 8, 4, 128, 1 << 26, 16) == PA_ERR_UNSUPPORTED);
  CHECK(decode_f16(0, 8, 2, 128, 4, 16) == PA_OK); /* empty batch: nothing to launch */
  CHECK(pa_decode_i8(fake(), fake(), fake(), fake(), NULL, NULL, (const int32_t*)fake(),
                     (const int32_t*)fake(), 1, 8, 2, 128, 4, 16, 2, 0.1f, fake(),
                     (size_t)1 << 30, NULL) == PA_ERR_INVALID_ARG); /* scales required */

  /* Extensions. */
  CHECK(pa_decode_bf16q(fake(), fake(), fake(), fake(), NULL, NULL, (const int32_t*)fake(),
                        (const int32_t*)fake(), 1, 8, 2, 128, 4, 16, 2, PA_DTYPE_F32, 0, 0.1f,
                        fake(), (size_t)1 << 30, NULL) == PA_ERR_UNSUPPORTED);
  CHECK(pa_selftest_bounded_wait(NULL, NULL) == PA_ERR_INVALID_ARG);
  CHECK(pa_reset_workspace(NULL, 1024, NULL) == PA_ERR_INVALID_ARG);
  CHECK(pa_decode_f16_noalloc_read_status(NULL, NULL) == PA_ERR_INVALID_ARG);
  CHECK(pa_partial_floats(12, 2, 128) == 130 * 8);
  CHECK(pa_partial_floats(12, 5, 128) == 0);

  /* Cache writes: input dtype and null pointers. */
  CHECK(pa_quantize_into_cache(fake(), fake(), 9, 256, (const int32_t*)fake(), 4, 2, 128,
                               fake(), fake(), (float*)fake(), (float*)fake(), 4, 16, NULL,
                               NULL, NULL, NULL) == PA_ERR_UNSUPPORTED);
  CHECK(pa_quantize_into_cache_fp8(fake(), fake(), PA_DTYPE_F16, 256, (const int32_t*)fake(),
                                   4, 2, 128, fake(), fake(), NULL, (float*)fake(), 4, 16,
                                   NULL, NULL) == PA_ERR_INVALID_ARG);
  CHECK(pa_absmax_scale(fake(), 0, 10, (float*)fake(), 7, fake(), NULL) == PA_ERR_INVALID_ARG);

  if (failures) return 1;
  printf("c abi ok\n");
  return 0;
}
