/* A C caller of the C ABI (no Python): includes include/morph_b200.h, links
 * libmorph_b200.so and exercises the host-only entry points and the argument
 * checks of device entry points (which fail before touching a GPU). Exits 0 on
 * success; prints the failing check otherwise. */
#include <stdio.h>
#include <stddef.h>
#include <string.h>

#include "morph_b200.h"

#define CHECK(cond)                                           \
  do {                                                        \
    if (!(cond)) {                                            \
      fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
      return 1;                                               \
    }                                                         \
  } while (0)

int main(void) {
  CHECK(mb_version() >= 1);
  CHECK(strncmp(mb_status_string(MB_ERR_NONFINITE), "nonfinite gradient", 18) == 0);
  CHECK(sizeof(mb_segment) == 64 && sizeof(mb_group) == 32 && sizeof(mb_step_state) == 96);
  CHECK(sizeof(mb_muon_args) == 56 && offsetof(mb_muon_args, max_sms) == 48);

  mb_step_state st;
  CHECK(mb_step_state_init(&st, 65536.0, 2000) == MB_OK);
  CHECK(st.scale == 65536.0 && st.growth_interval == 2000 && st.clip_coef == 1.0f && st.skip == 0);
  CHECK(mb_step_state_init(&st, 0.0, 2000) == MB_ERR_ARG);

  mb_segment segs[3];
  memset(segs, 0, sizeof(segs));
  const int64_t sizes[3] = {1, 2048, 2049};
  for (int i = 0; i < 3; ++i) {
    segs[i].w = segs[i].m = segs[i].v = (float*)4096;
    segs[i].g = (const void*)4096;
    segs[i].numel = sizes[i];
  }
  int64_t tiles = 0;
  CHECK(mb_segments_plan(segs, 3, &tiles) == MB_OK);
  CHECK(segs[0].tile_begin == 0 && segs[1].tile_begin == 1 && segs[2].tile_begin == 2 && tiles == 4);
  CHECK(mb_workspace_bytes(10) % 256 == 0);

  /* argument checks fail before any device work */
  CHECK(mb_adamw_step(NULL, NULL, NULL) == MB_ERR_ARG);
  CHECK(mb_adamw_update(NULL, NULL, NULL, NULL, MB_F32, NULL, MB_NONE, 16, NULL, NULL) == MB_ERR_ARG);
  CHECK(mb_muon_batch_workspace_bytes(0, 64, 64) == 0);
  CHECK(mb_muon_batch_workspace_bytes(MB_MUON_MAX_BATCH + 1, 64, 64) == 0);
  CHECK(mb_muon_workspace_bytes(64, 64) > 0);
  CHECK(mb_grad_accumulate(NULL, NULL, MB_F32, 1, 1.0f, 0, NULL, NULL, NULL) == MB_ERR_ARG);
  CHECK(mb_export_f16(NULL, 1, NULL, NULL, NULL) == MB_ERR_ARG);
  CHECK(mb_ipc_open(NULL, NULL) == MB_ERR_ARG);
  printf("c abi ok\n");
  return 0;
}
