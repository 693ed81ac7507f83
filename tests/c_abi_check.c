/* A C host of librlenv.so: include/rlenv.h compiled as C99 and linked, the entry points called
 * on paths that need no GPU (version, messages, arguments rejected before any launch, empty
 * batches). Built and run by tests/test_abi.py. */
#include <stdio.h>
#include <string.h>

#include "rlenv.h"

static int fails = 0;

static void expect(int got, int want, const char* what) {
  if (got != want) {
    printf("%s: got %d, want %d\n", what, got, want);
    ++fails;
  }
}

int main(void) {
  void* fake = (void*)0x1000; /* never dereferenced: each call below is rejected first */
  expect(rlenv_abi_version(), 2, "abi version");
  expect(strcmp(rlenv_strerror(RLENV_OK), "ok"), 0, "strerror(ok)");
  expect(rlenv_cartpole_step(fake, fake, 7, 1, 4, 0, fake, fake, fake, NULL), RLENV_EINVAL, "unknown dtype");
  expect(rlenv_cartpole_step(NULL, NULL, RLENV_I32, 1, 0, 0, NULL, NULL, NULL, NULL), RLENV_OK, "empty batch");
  expect(rlenv_acrobot_step(NULL, NULL, RLENV_U2, 1, 0, 0, NULL, NULL, NULL, NULL), RLENV_OK, "packed, empty batch");
  expect(rlenv_pendulum_aba_step(8, fake, fake, RLENV_U2, 1, 4, 0, fake, fake, fake, NULL), RLENV_EINVAL,
         "packed actions outside the classic bodies");
  expect(rlenv_acrobot_step_many(fake, fake, RLENV_U8, 1, -1, 4, 0, fake, NULL, NULL, NULL, NULL, NULL),
         RLENV_EINVAL, "negative steps");
  expect(rlenv_pendulum_aba_step(193, fake, fake, RLENV_I32, 1, 4, 0, fake, fake, fake, NULL), RLENV_EUNSUPPORTED,
         "unbuilt K");
  expect(rlenv_legged_step_many(5, 8, fake, fake, RLENV_I32, 1, fake, 0.0f, NULL, 3, 4, 0, fake, NULL, NULL, NULL,
                                NULL),
         RLENV_EUNSUPPORTED, "unbuilt C");
  expect((int)rlenv_es_ranks_scratch_bytes(4097), 16 * 4097, "rank scratch bytes");
  expect(rlenv_es_centered_ranks_static(fake, 65537, fake, NULL), RLENV_EINVAL, "oversize population");
  printf(fails ? "FAIL\n" : "ok\n");
  return fails != 0;
}
