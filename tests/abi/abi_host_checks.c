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

/* Attention straight from the QKV rows over host memory: 32 slots, 16 query heads on 8 kv
 * heads, 64 positions. Every argument error is reported before the first device call, so the
 * host buffer is never touched. */
static int attention_qkv(void* buf, int64_t head_dim, size_t workspace_bytes, const void* p0, size_t p0_bytes,
                         const void* p1, size_t p1_bytes) {
  const int64_t* pos = (const int64_t*)buf;
  return q3t_decode_attention_qkv_ex(buf, (16 + 2 * 8) * head_dim, buf, buf, 1e-6f, buf, buf, 64, pos, buf, buf,
                                     pos, buf, 32, 16, 8, head_dim, 32, 64, 64, 0.088f,
                                     workspace_bytes ? buf : NULL, workspace_bytes, p0, p0_bytes, p1, p1_bytes,
                                     NULL, NULL);
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

  char raw[1024];
  char* a16 = raw + ((16 - ((uintptr_t)raw & 15)) & 15);
  rc = attention_qkv(a16, 128, 0, a16 + 4, 64, NULL, 0);
  check(rc == Q3T_EINVAL, "attention_qkv_ex rejects a misaligned prefetch range");
  check(strstr(q3t_last_error(), "prefetch") != NULL, "attention_qkv_ex prefetch error message");
  rc = attention_qkv(a16, 128, 0, NULL, 0, a16, 40);
  check(rc == Q3T_EINVAL, "attention_qkv_ex rejects a prefetch size that is not a multiple of 16");
  rc = attention_qkv(a16, 128, 0, NULL, 64, NULL, 0);
  check(rc == Q3T_EINVAL, "attention_qkv_ex rejects prefetch bytes without a pointer");
  rc = attention_qkv(a16, 96, 0, a16, 64, NULL, 0);
  check(rc == Q3T_EUNSUPPORTED, "attention_qkv_ex reports head_dim 96 as unsupported");
  rc = attention_qkv(a16, 128, 16, a16, 64, a16 + 16, 64);
  check(rc == Q3T_ESPACE, "attention_qkv_ex accepts two aligned prefetch ranges, then wants a workspace");
  check(strstr(q3t_last_error(), "workspace") != NULL, "attention_qkv_ex workspace error message");
  int64_t* pos = (int64_t*)a16;
  rc = q3t_decode_attention_qkv(a16, 32 * 128, a16, a16, 1e-6f, a16, a16, 64, pos, a16, a16, pos, a16, 32, 16, 8,
                                128, 32, 64, 128, 0.088f, NULL, 0, NULL, NULL);
  check(rc == Q3T_EINVAL, "attention_qkv rejects a context beyond the arena capacity");

  check(q3t_launch_count() == 0, "rejected calls launch nothing");
  return failures ? 1 : 0;
}
