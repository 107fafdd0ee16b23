// Launch description shared by the decode-attention kernels.
#pragma once

#include <stdint.h>

namespace q3t {

struct AttentionCall {
  const void* query;
  const void* keys;
  const void* values;
  const int64_t* positions;
  void* out;
  int64_t rows, rows_per_slot;
  const int64_t* slots;
  int64_t q_heads, kv_heads, head_dim;
  int64_t arena_slots, capacity, context, window;
  float scale;
  int chunk, max_chunks;
  float* partials;
  unsigned* counters;  // one chunk ticket per (row, kv head), zero between calls
  const unsigned* plan;  // keys per chunk planned for this batch (q3t_attention_plan), or null
  unsigned* status;
  void* stream;
  // L2 prefetch hint (fused kernel): up to two byte ranges (normally the weights of the
  // projections that follow this attention) pulled into L2 while the keys stream; each CTA
  // requests its share once. Null / 0 = none.
  const void* prefetch[2];
  uint64_t prefetch_bytes[2];
};

// Tensor-core (mma.sync) kernel for linear arenas: head_dim 64/128, 1 or 2 query heads per kv head.
bool attention_mma_supported(int64_t head_dim, int64_t group);
// Resident CTAs of the tensor-core kernel on this device (one wave), 0 when unknown.
int attention_wave_ctas(int64_t head_dim, int64_t group, bool fused);
int launch_attention_mma(const AttentionCall& call);
// Decode variant reading the raw QKV projection (per-head norm, RoPE and K/V write fused).
int launch_attention_fused(const AttentionCall& call, const void* qkv, int64_t qkv_stride, const void* q_norm,
                           const void* k_norm, float eps, const void* cos, const void* sin, int64_t table_len,
                           const int64_t* rot_pos);

}  // namespace q3t
