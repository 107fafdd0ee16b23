// QKV epilogue of packed attention: per-head q_norm / k_norm (RMSNorm over
// head_dim, HF rounding), text-only rotary with bf16 rounding after every
// product and sum, and the slot-table write of K and V at each row's cache
// position (packed_attention.py:42-74, rotary_triton_ascend.py:19-24,
// continuous.py:152-166).
//
// One CTA per row, one warp per head: lane l holds dims [l*D/32, (l+1)*D/32),
// so the rotate-half partner of a dim sits in lane l^16 (one shuffle).
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

template <int D>
__global__ void qk_norm_rope_kv_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t qkv_stride,
                                       const __nv_bfloat16* __restrict__ qw, const __nv_bfloat16* __restrict__ kw,
                                       float eps, const __nv_bfloat16* __restrict__ cos_t,
                                       const __nv_bfloat16* __restrict__ sin_t, int64_t table_len,
                                       const int64_t* __restrict__ rot_pos, const int64_t* __restrict__ cache_pos,
                                       __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ tk,
                                       __nv_bfloat16* __restrict__ tv, int length, const int64_t* __restrict__ slots,
                                       int q_heads, int kv_heads, int64_t capacity, unsigned* status) {
  constexpr int DL = D / 32;
  grid_dependency_wait();
  const int64_t r = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int head = warp;  // 0..q_heads-1: query heads, q_heads..q_heads+kv_heads-1: key heads
  int64_t rp = rot_pos[r];
  if (rp < 0 || rp >= table_len) {
    if (threadIdx.x == 0) raise_status(status, kStatusBadIndex);
    rp = rp < 0 ? 0 : table_len - 1;
  }
  const bool is_q = head < q_heads;
  const int kh = head - q_heads;
  const __nv_bfloat16* src = qkv + r * qkv_stride + int64_t(head) * D + lane * DL;
  float x[DL], w[DL], c[DL], s[DL];
#pragma unroll
  for (int d = 0; d < DL; ++d) {
    x[d] = __bfloat162float(src[d]);
    const __nv_bfloat16* nw = is_q ? qw : kw;
    w[d] = nw ? __bfloat162float(nw[lane * DL + d]) : 1.f;
    c[d] = __bfloat162float(cos_t[rp * D + lane * DL + d]);
    s[d] = __bfloat162float(sin_t[rp * D + lane * DL + d]);
  }
  float y[DL];
  if (qw != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) ss += x[d] * x[d];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(D) + eps);
#pragma unroll
    for (int d = 0; d < DL; ++d) y[d] = bf16r(w[d] * bf16r(x[d] * inv));
  } else {
#pragma unroll
    for (int d = 0; d < DL; ++d) y[d] = x[d];
  }
  // rotate half: first half of dims lives in lanes 0..15, second half in 16..31
  const bool first_half = lane < 16;
  float o[DL];
#pragma unroll
  for (int d = 0; d < DL; ++d) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[d], 16);
    const float rot = first_half ? -partner : partner;
    o[d] = bf16r(bf16r(y[d] * c[d]) + bf16r(rot * s[d]));
  }
  if (is_q) {
    __nv_bfloat16* dst = q_out + (r * q_heads + head) * D + lane * DL;
#pragma unroll
    for (int d = 0; d < DL; ++d) dst[d] = __float2bfloat16_rn(o[d]);
    return;
  }
  const int64_t pos = cache_pos[r];
  const int64_t slot = slots != nullptr ? slots[r / length] : r / length;
  if (pos < 0 || pos >= capacity) {
    if (lane == 0) raise_status(status, kStatusBadIndex);
    return;
  }
  const size_t dst = ((size_t(slot) * kv_heads + kh) * size_t(capacity) + size_t(pos)) * D + lane * DL;
  const __nv_bfloat16* vsrc = qkv + r * qkv_stride + int64_t(q_heads + kv_heads + kh) * D + lane * DL;
#pragma unroll
  for (int d = 0; d < DL; ++d) {
    tk[dst + d] = __float2bfloat16_rn(o[d]);
    tv[dst + d] = vsrc[d];
  }
}

}  // namespace

extern "C" int q3t_qk_norm_rope_kv(const void* qkv, int64_t qkv_stride, const void* q_norm_weight,
                                   const void* k_norm_weight, float eps, const void* cos_table, const void* sin_table,
                                   int64_t table_len, const int64_t* rotary_positions, const int64_t* cache_positions,
                                   void* query_out, void* target_keys, void* target_values, int64_t rows,
                                   int64_t length, const int64_t* slots, int64_t q_heads, int64_t kv_heads,
                                   int64_t head_dim, int64_t capacity, unsigned* status, void* stream) {
  if (!qkv || (q_norm_weight == nullptr) != (k_norm_weight == nullptr) || !cos_table || !sin_table || !rotary_positions || !cache_positions ||
      !query_out || !target_keys || !target_values)
    return fail(Q3T_EINVAL, "qk_norm_rope_kv: null pointer");
  if (rows < 1 || length < 1 || rows % length || q_heads < 1 || kv_heads < 1 || q_heads + kv_heads > 32 ||
      capacity < 1 || table_len < 1)
    return fail(Q3T_EINVAL, "qk_norm_rope_kv: invalid geometry");
  if (qkv_stride < (q_heads + 2 * kv_heads) * head_dim) return fail(Q3T_EINVAL, "qk_norm_rope_kv: qkv stride");
  const dim3 block(unsigned(32 * (q_heads + kv_heads)));
  if (head_dim == 128)
    return launch(qk_norm_rope_kv_kernel<128>, dim3(unsigned(rows)), block, 0, stream, true, "qk_norm_rope_kv",
                  static_cast<const __nv_bfloat16*>(qkv), qkv_stride, static_cast<const __nv_bfloat16*>(q_norm_weight),
                  static_cast<const __nv_bfloat16*>(k_norm_weight), eps,
                  static_cast<const __nv_bfloat16*>(cos_table), static_cast<const __nv_bfloat16*>(sin_table),
                  table_len, rotary_positions, cache_positions, static_cast<__nv_bfloat16*>(query_out),
                  static_cast<__nv_bfloat16*>(target_keys), static_cast<__nv_bfloat16*>(target_values), int(length),
                  slots, int(q_heads), int(kv_heads), capacity, status);
  if (head_dim == 64)
    return launch(qk_norm_rope_kv_kernel<64>, dim3(unsigned(rows)), block, 0, stream, true, "qk_norm_rope_kv",
                  static_cast<const __nv_bfloat16*>(qkv), qkv_stride, static_cast<const __nv_bfloat16*>(q_norm_weight),
                  static_cast<const __nv_bfloat16*>(k_norm_weight), eps,
                  static_cast<const __nv_bfloat16*>(cos_table), static_cast<const __nv_bfloat16*>(sin_table),
                  table_len, rotary_positions, cache_positions, static_cast<__nv_bfloat16*>(query_out),
                  static_cast<__nv_bfloat16*>(target_keys), static_cast<__nv_bfloat16*>(target_values), int(length),
                  slots, int(q_heads), int(kv_heads), capacity, status);
  return fail(Q3T_EUNSUPPORTED, "qk_norm_rope_kv: head_dim must be 64 or 128");
}
