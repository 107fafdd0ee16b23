/* A plain-C host of the library (what a foreign-language binding sees): version, the
 * size queries, and argument errors that are reported before any device work, each with
 * its message. Needs no GPU. Prints one line per check; exits non-zero on a failure. */
#include <stdio.h>
#include <string.h>

#include "q3t.h"

static int failures = 0;

static void check(int ok, const char* what) {
  printf("%s %s\n", ok ? "ok  " : "FAIL", what);
  if (!ok) ++failures;
}

int main(void) {
  check(q3t_abi_version() == 1, "abi version 1");
  check(q3t_launch_count() == 0, "no launches in a fresh process");
  /* 128 x 64 bf16 tiles of 16 KB: 4096 x 2048 -> 32 x 32 tiles */
  check(q3t_weight_tiles_bytes(4096, 2048) == (size_t)32 * 32 * 16384, "weight tile bytes");
  check(q3t_weight_tiles_bytes(0, 2048) == 0, "weight tile bytes of an empty weight");
  check(q3t_decode_attention_workspace_bytes(32, 16, 128, 4096) > 0, "attention workspace size");
  check(q3t_decode_attention_workspace_bytes(0, 16, 128, 4096) == 0, "attention workspace of no rows");

  int64_t strides[3] = {1, 1, 1};
  int rc = q3t_kv_write(NULL, strides, NULL, strides, NULL, NULL, NULL, 1, 8, 128, 64, Q3T_BF16, NULL, NULL);
  check(rc == Q3T_EINVAL, "kv_write rejects null pointers");
  check(strstr(q3t_last_error(), "kv_write") != NULL, "kv_write error message");

  int64_t tshape[5] = {2, 4, 8, 16, 128}, sshape[5] = {2, 1, 8, 16, 128}, tstr[5] = {0}, sstr[5] = {0};
  char target[16], source[16];
  rc = q3t_copy_packed_prefix(target, tshape, tstr, source, sshape, sstr, 2, 4, 0, 1, NULL);
  check(rc == Q3T_EINVAL, "copy_packed_prefix rejects an out-of-range slot");
  rc = q3t_copy_packed_prefix(target, tshape, tstr, target, tshape, tstr, 2, 0, 0, 1, NULL);
  check(rc == Q3T_EINVAL, "copy_packed_prefix rejects an aliasing source");
  check(strstr(q3t_last_error(), "independent") != NULL, "copy_packed_prefix error message");

  check(q3t_launch_count() == 0, "rejected calls launch nothing");
  return failures ? 1 : 0;
}
