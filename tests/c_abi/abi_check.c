/* A C99 host of the musc_b200 C ABI: compiled with gcc -std=c99 against
 * include/musc_b200.h and linked to the built library by tests/test_c_abi.py.
 * It makes host-only calls (no device work): the ABI version, the size
 * queries and contract violations that every entry point reports before any
 * CUDA call, with their status codes and messages. */
#include <stdio.h>
#include <string.h>

#include "musc_b200.h"

static int failures = 0;

static void expect(int cond, const char* what) {
  if (!cond) {
    fprintf(stderr, "FAIL: %s (last error: %s)\n", what, musc_b200_last_error());
    ++failures;
  }
}

int main(void) {
  expect(musc_b200_abi_version() == 3, "abi version");
  expect(musc_b200_lnamd_workspace_bytes(4) == 4 * 8 * 2 * sizeof(double), "lnamd workspace");
  expect(musc_b200_bank_bytes(1369, 1024) % 1024 == 0, "bank bytes aligned");
  expect(musc_b200_nearest_pool_bytes(16 * 1369, 1369, 16 * 1369) >= (size_t)16 * 16 * 1369 * 4,
         "nearest table bytes");
  expect(musc_b200_score_pool_bytes(16, 1370, 1024, 3) > musc_b200_bank_bytes(16 * 1369, 1024),
         "score pool workspace");
  expect(musc_b200_score_pool_bytes(0, 1370, 1024, 3) == 0, "score pool workspace, no images");

  size_t planes[5];
  expect(musc_b200_bank_layout(1369, 1024, planes) == MUSC_B200_OK, "bank layout");
  expect(planes[0] == 0 && planes[1] > planes[0] && planes[2] > planes[1] && planes[3] > planes[2] &&
             planes[4] > planes[3] && musc_b200_bank_bytes(1369, 1024) > planes[4],
         "bank planes ordered");
  expect(musc_b200_refine_bytes(16, 16 * 1369, 1024) > (size_t)16 * 16 * 1369 * 4, "refine workspace");
  expect(musc_b200_refine_bytes(0, 16 * 1369, 1024) == 0, "refine workspace, no images");

  /* screen and refinement contract violations */
  expect(musc_b200_screen_pool((const void*)(size_t)1024, 2738, 2738, 64, 1369, 0, 1, 2738, 0, NULL,
                               (void*)(size_t)1024, (void*)(size_t)1024, NULL) == MUSC_B200_ERR_INVALID,
         "screen null table");
  expect(musc_b200_screen_pool((const void*)(size_t)1024, 2738, 2738, 64, 1369, 2, 2, 2738, 0,
                               (void*)(size_t)1024, (void*)(size_t)1024, (void*)(size_t)1024, NULL) ==
             MUSC_B200_ERR_INVALID,
         "screen part out of range");
  expect(musc_b200_refine((const void*)(size_t)1024, 2738, 2738, 64, 1369, 0, 2738, 2,
                          (const void*)(size_t)1024, (const void*)(size_t)1024, 1, 0, 2738,
                          (float*)(size_t)1024, (void*)(size_t)1024, (size_t)1 << 40, NULL) == MUSC_B200_ERR_INVALID,
         "refine rank beyond N-1");

  /* contract violations: reported before any CUDA call */
  expect(musc_b200_trimmed_mean(NULL, 10, 5, 0, 1, NULL, NULL) == MUSC_B200_ERR_INVALID, "trimmed null");
  expect(strstr(musc_b200_last_error(), "null") != NULL, "trimmed null message");
  int radii[1] = {2};
  float* outs[1] = {(float*)(size_t)1024};
  expect(musc_b200_lnamd((const void*)(size_t)1024, MUSC_B200_F32, 2, 1370, 64, 1, radii, outs,
                         1369 * 64, 64, 1, (void*)(size_t)1024, 1024, NULL) == MUSC_B200_ERR_INVALID,
         "lnamd radius");
  int ks[9] = {1, 2, 3, 4, 5, 6, 7, 8, 9};
  expect(musc_b200_rscin((const float*)(size_t)1024, 10, 768, (const double*)(size_t)2048, 9, ks,
                         (double*)(size_t)4096, NULL) == MUSC_B200_ERR_INVALID,
         "rscin k list");
  expect(musc_b200_msm((const float*)(size_t)16, 1, 10, 8, 0, 1, (double*)(size_t)16,
                       (void*)(size_t)1024, (size_t)1 << 30, NULL) == MUSC_B200_ERR_INVALID,
         "msm N>=2");
  /* pool-image preprocessing: size queries and contract violations */
  expect(musc_b200_preprocess_workspace_bytes(900, 900, 518, 518, MUSC_B200_BICUBIC) >= (size_t)2 * 518 * 9 * 4,
         "preprocess workspace");
  expect(musc_b200_preprocess_workspace_bytes(900, 900, 36, 518, MUSC_B200_BICUBIC) == 0,
         "preprocess workspace, 25x reduction");
  expect(musc_b200_preprocess_workspace_bytes(900, 900, 518, 518, 7) == 0, "preprocess workspace, bad filter");
  const float mean[3] = {0.5f, 0.5f, 0.5f}, zero_std[3] = {1.0f, 0.0f, 1.0f}, std3[3] = {0.2f, 0.2f, 0.2f};
  expect(musc_b200_preprocess_images((const uint8_t*)(size_t)1024, 2, 900, 900, 900 * 900 * 3, 518, 518,
                                     MUSC_B200_BICUBIC, mean, zero_std, MUSC_B200_F32, (void*)(size_t)1024,
                                     (void*)(size_t)1024, 1 << 20, NULL) == MUSC_B200_ERR_INVALID,
         "preprocess zero std");
  expect(musc_b200_preprocess_images((const uint8_t*)(size_t)1024, 2, 900, 900, 100, 518, 518,
                                     MUSC_B200_BICUBIC, mean, std3, MUSC_B200_F32, (void*)(size_t)1024,
                                     (void*)(size_t)1024, 1 << 20, NULL) == MUSC_B200_ERR_INVALID,
         "preprocess image stride");
  expect(musc_b200_preprocess_images((const uint8_t*)(size_t)1024, 2, 900, 900, 900 * 900 * 3, 36, 518,
                                     MUSC_B200_BICUBIC, mean, std3, MUSC_B200_F32, (void*)(size_t)1024,
                                     (void*)(size_t)1024, 1 << 20, NULL) == MUSC_B200_ERR_INVALID,
         "preprocess 25x reduction");
  expect(strstr(musc_b200_last_error(), "15.75x") != NULL, "preprocess ratio message");

  int code = -1;
  expect(musc_b200_take_device_error(NULL) == MUSC_B200_ERR_INVALID, "device error null");
  (void)code;

  if (failures == 0) printf("c abi ok\n");
  return failures == 0 ? 0 : 1;
}
