// Causal prefill attention over packed prompts on tcgen05 tensor cores.
//
// A packed prefill holds several prompts end to end; row r of the packed rows is
// position positions[r] of some arena slot, and its K/V are already in the arena. The
// decode kernels would run every row as its own query and re-read the row's whole
// K/V prefix once per row (O(L^2) K/V traffic per prompt). Here one CTA owns a UNIT:
// up to 64 consecutive rows of one prompt for one KV head, i.e. a 128-row query tile
// (64 positions x the 2 query heads of the head group), and streams that prompt's keys
// 0..keys-1 once, in 64-key blocks:
//
//   S = Q K^T       tcgen05.mma M=128 N=64 K=128, fp32 accumulator in TMEM (64 columns)
//   P = softmax     one thread per query row (TMEM lane), causal mask key <= position,
//                   online max/sum in fp32, P rounded to bf16 into shared memory in the
//                   128-byte-swizzled K-major layout of a UMMA A operand
//   O += P V        tcgen05.mma M=128 N=128 K=64 into a second TMEM block; V is the
//                   MN-major B operand straight from its TMA tile (keys x dims rows),
//                   and each thread folds the block into its fp32 output row with the
//                   online-softmax rescale
//
// Q, K and V move by TMA (no multicast): Q as four {64 dims, 1 head, 64 rows} boxes of
// the [rows, q_heads, head_dim] query, K and V as two {64 dims, 64 keys} boxes each of
// the [slots * kv_heads * capacity, head_dim] arena layer. The next K block loads during
// the softmax, the next V block during the output update. Units come from the host in a
// table {first_row, rows, keys, slot}; rows == 0 marks an empty entry (the table of a
// captured graph has a fixed size). Every wait is bounded and reports through the
// status word.
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr int kQRows = 64;     // positions per unit
constexpr int kKeys = 64;      // keys per block
constexpr int kDim = 128;
constexpr int kQBytes = 2 * kQRows * kDim * 2;          // 128 query rows x 128 dims = 32 KB
constexpr int kKBytes = kKeys * kDim * 2;               // 16 KB
constexpr int kPBytes = 2 * kQRows * kKeys * 2;         // 128 rows x 64 keys = 16 KB
// shared memory: Q [0, 32K) | K [32K, 48K) | P [48K, 64K) | V [64K, 80K) | barriers
constexpr int kOffK = kQBytes, kOffP = kOffK + kKBytes, kOffV = kOffP + kPBytes, kOffBar = kOffV + kKBytes;
constexpr int kSmem = kOffBar + 128 + 1024;
constexpr int kTmemCols = 256;  // S: columns [0, 64), PV: [64, 192)

// K-major SW128 descriptor (rows of 128 B, 8-row groups 1024 B apart) is umma_desc_sw128.
// MN-major SW128 descriptor for the V operand: atoms of 64 dims x 8 keys (1024 B); the
// atom holding dims 64..127 sits `mn_stride` bytes on (leading byte offset), the next 8 keys
// 1024 B on (stride byte offset).
Q3T_DEV uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t mn_stride) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((mn_stride >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

Q3T_DEV void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
Q3T_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

struct PrefillArgs {
  const int4* units;        // {first_row, rows, keys, slot}
  const int64_t* positions; // [rows] position of each packed row
  __nv_bfloat16* out;       // [rows, q_heads, head_dim]
  int rows, q_heads, kv_heads, arena_slots;
  int64_t capacity;
  float scale_log2;         // softmax scale x log2(e)
  unsigned* status;
};

__global__ void __launch_bounds__(128, 2)
    prefill_attention_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                             const __grid_constant__ CUtensorMap tmv, PrefillArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_bar = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint64_t* k_bar = q_bar + 1;
  uint64_t* v_bar = q_bar + 2;
  uint64_t* s_bar = q_bar + 3;
  uint64_t* pv_bar = q_bar + 4;
  uint64_t* done_bar = q_bar + 5;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_bar + 6);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int head = blockIdx.y;  // KV head
  grid_dependency_wait();
  const int4 u = a.units[blockIdx.x];
  const int first = u.x, count = u.y, keys = u.z, slot = u.w;
  if (count <= 0) return;  // empty table entry (uniform over the CTA)
  if (count > kQRows || first < 0 || first + count > a.rows || keys < 1 || keys > a.capacity || slot < 0 ||
      slot >= a.arena_slots) {
    if (tid == 0) raise_status(a.status, kStatusBadIndex);
    return;
  }
  const int blocks = (keys + kKeys - 1) / kKeys;
  const int64_t key_row0 = (int64_t(slot) * a.kv_heads + head) * a.capacity;

  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(&q_bar[i], 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmq);
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint64_t pol = policy_evict_last();
  int k_loads = 0, v_loads = 0;  // thread 0: loads issued
  auto load_k = [&](int blk) {
    ++k_loads;
    mbar_expect_tx(k_bar, kKBytes);
    for (int h = 0; h < 2; ++h)
      tma_load_2d(smem + kOffK + h * (kKBytes / 2), &tmk, k_bar, h * 64, int(key_row0 + blk * kKeys), pol);
  };
  auto load_v = [&](int blk) {
    ++v_loads;
    mbar_expect_tx(v_bar, kKBytes);
    for (int h = 0; h < 2; ++h)
      tma_load_2d(smem + kOffV + h * (kKBytes / 2), &tmv, v_bar, h * 64, int(key_row0 + blk * kKeys), pol);
  };
  if (tid == 0) {
    // query tile row m = g * 64 + p: position first + p, query head 2 * head + g
    mbar_expect_tx(q_bar, kQBytes);
    for (int h = 0; h < 2; ++h)
      for (int g = 0; g < 2; ++g)
        tma_load_3d(smem + h * (kQBytes / 2) + g * (kQBytes / 4), &tmq, q_bar, h * 64, 2 * head + g, first,
                    policy_evict_first());
    load_k(0);
    load_v(0);
  }

  // this thread's query row
  const int m = warp * 32 + lane;  // TMEM lane
  const int p = m & (kQRows - 1);
  int64_t qpos = p < count ? a.positions[first + p] : a.positions[first + count - 1];
  if (qpos < 0 || qpos >= keys) {  // the unit's key count covers every row's position
    raise_status(a.status, kStatusBadIndex);
    qpos = qpos < 0 ? 0 : keys - 1;
  }
  float o[kDim];
#pragma unroll
  for (int i = 0; i < kDim; ++i) o[i] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const uint32_t lane_base = tmem + (uint32_t(warp * 32) << 16);
  constexpr uint32_t idesc_s = umma_idesc_bf16(128, kKeys);
  constexpr uint32_t idesc_pv = umma_idesc_bf16(128, kDim) | (1u << 16);  // B (V) MN-major
  bool ok = true;

  for (int blk = 0; blk < blocks; ++blk) {
    const uint32_t parity = uint32_t(blk & 1);
    // ---- S = Q K^T
    if (tid == 0) {
      bool landed = (blk > 0 || mbar_wait(q_bar, 0, a.status, kStatusTmaTimeout)) &&
                    mbar_wait(k_bar, parity, a.status, kStatusTmaTimeout);
      if (landed) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kDim / 16; ++k) {
          const int h = k >> 2, kk = k & 3;
          const uint64_t ad = umma_desc_sw128(smem_u32(smem + h * (kQBytes / 2))) + 2 * kk;
          const uint64_t bd = umma_desc_sw128(smem_u32(smem + kOffK + h * (kKBytes / 2))) + 2 * kk;
          umma_bf16(tmem, ad, bd, idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(s_bar);
      } else {
        *abort_flag = 1;
      }
    }
    __syncthreads();
    if (*abort_flag) {
      ok = false;
      break;
    }
    if (!__syncthreads_and(mbar_wait(s_bar, parity, a.status, kStatusMmaTimeout))) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0 && blk + 1 < blocks) load_k(blk + 1);  // the S MMAs have read the K tile
    // ---- softmax of this row over keys blk*64 .. +63
    uint32_t sr[4][16];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld16_nowait(lane_base + uint32_t(16 * c), sr[c]);
    tmem_ld_wait();
    const int k0 = blk * kKeys;
    float mx = m_run;
#pragma unroll
    for (int i = 0; i < kKeys; ++i)
      if (k0 + i <= qpos) mx = fmaxf(mx, __uint_as_float(sr[i >> 4][i & 15]));
    const float alpha = m_run == -INFINITY ? 0.f : exp2f((m_run - mx) * a.scale_log2);
    m_run = mx;
    float sum = 0.f;
    uint8_t* prow = smem + kOffP + m * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      float pv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int i = c * 8 + e;
        pv[e] = k0 + i <= qpos ? exp2f((__uint_as_float(sr[i >> 4][i & 15]) - mx) * a.scale_log2) : 0.f;
        sum += pv[e];
      }
      // 16-byte chunk c of row m at chunk position c ^ (m % 8) (128-byte swizzle)
      *reinterpret_cast<uint4*>(prow + ((c ^ (m & 7)) << 4)) = pack8(pv);
    }
    l_run = l_run * alpha + sum;
    fence_async_shared();  // P (generic proxy) before the MMA reads it
    tc_fence_before();
    __syncthreads();
    // ---- PV = P V
    if (tid == 0) {
      if (mbar_wait(v_bar, parity, a.status, kStatusTmaTimeout)) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k) {
          const uint64_t ad = umma_desc_sw128(smem_u32(smem + kOffP)) + 2 * k;
          const uint64_t bd = umma_desc_sw128_mn(smem_u32(smem + kOffV + k * 16 * 128), kKBytes / 2);
          umma_bf16(tmem + 64, ad, bd, idesc_pv, k > 0 ? 1u : 0u);
        }
        umma_commit(pv_bar);
      } else {
        *abort_flag = 1;
      }
    }
    __syncthreads();
    if (*abort_flag) {
      ok = false;
      break;
    }
    if (!__syncthreads_and(mbar_wait(pv_bar, parity, a.status, kStatusMmaTimeout))) {
      ok = false;
      break;
    }
    tc_fence_after();
    if (tid == 0 && blk + 1 < blocks) load_v(blk + 1);  // the PV MMAs have read the V tile
    // ---- o = o * alpha + PV
#pragma unroll
    for (int c0 = 0; c0 < kDim; c0 += 64) {
      uint32_t vr[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld16_nowait(lane_base + uint32_t(64 + c0 + 16 * c), vr[c]);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 64; ++i) o[c0 + i] = o[c0 + i] * alpha + __uint_as_float(vr[i >> 4][i & 15]);
    }
    tc_fence_before();
    __syncthreads();  // every TMEM read of this block is done before the next MMAs overwrite S / PV
  }

  if (ok && p < count) {
    const float inv = 1.0f / l_run;
    __nv_bfloat16* dst = a.out + (int64_t(first + p) * a.q_heads + 2 * head + (m >> 6)) * kDim;
#pragma unroll
    for (int c = 0; c < kDim / 8; ++c) {
      float v8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v8[e] = o[c * 8 + e] * inv;
      reinterpret_cast<uint4*>(dst)[c] = pack8(v8);
    }
  }
  if (tid == 0) {
    if (!ok) {  // loads still in flight land before the CTA exits (the last phase of each barrier)
      mbar_wait(q_bar, 0, a.status, kStatusTmaTimeout);
      if (k_loads > 0) mbar_wait(k_bar, uint32_t((k_loads - 1) & 1), a.status, kStatusTmaTimeout);
      if (v_loads > 0) mbar_wait(v_bar, uint32_t((v_loads - 1) & 1), a.status, kStatusTmaTimeout);
    }
    umma_commit(done_bar);  // every MMA of this CTA has completed before TMEM is released
    mbar_wait(done_bar, 0, a.status, kStatusMmaTimeout);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, kTmemCols);
}

int make_query_map(CUtensorMap* map, const void* query, int64_t rows, int64_t q_heads) {
  return make_map_bf16_3d(map, query, kDim, q_heads, rows, 64, 1, kQRows);
}

}  // namespace

extern "C" int q3t_prefill_attention(const void* query, const void* keys, const void* values,
                                     const int64_t* positions, const int32_t* units, int64_t unit_count, void* out,
                                     int64_t rows, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                                     int64_t arena_slots, int64_t capacity, float scale, unsigned* status,
                                     void* stream) {
  if (!query || !keys || !values || !positions || !units || !out) return fail(Q3T_EINVAL, "prefill_attention: null");
  if (head_dim != kDim || kv_heads < 1 || q_heads != 2 * kv_heads || kv_heads > 65535)
    return fail(Q3T_EUNSUPPORTED, "prefill_attention: needs head_dim 128 and 2 query heads per KV head");
  if (rows < 1 || rows > (int64_t(1) << 30) || unit_count < 1 || unit_count > 2147483647 || arena_slots < 1 ||
      capacity < 1 || arena_slots * kv_heads * capacity > (int64_t(1) << 31))
    return fail(Q3T_EINVAL, "prefill_attention: invalid geometry");
  if (!aligned16(query) || !aligned16(keys) || !aligned16(values) || !aligned16(out) || !aligned16(units))
    return fail(Q3T_EINVAL, "prefill_attention: 16-byte alignment");
  CUtensorMap tmq, tmk, tmv;
  int rc = make_query_map(&tmq, query, rows, q_heads);
  if (rc) return rc;
  const int64_t arena_rows = arena_slots * kv_heads * capacity;
  rc = make_map_bf16(&tmk, keys, arena_rows, kDim, kDim, 64, kKeys);
  if (rc) return rc;
  rc = make_map_bf16(&tmv, values, arena_rows, kDim, kDim, 64, kKeys);
  if (rc) return rc;
  static PerDevice smem_once;
  if (const int r = smem_limit(smem_once, prefill_attention_kernel, kSmem, "prefill_attention: set smem")) return r;
  PrefillArgs a;
  a.units = reinterpret_cast<const int4*>(units);
  a.positions = positions;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.rows = int(rows);
  a.q_heads = int(q_heads);
  a.kv_heads = int(kv_heads);
  a.arena_slots = int(arena_slots);
  a.capacity = capacity;
  a.scale_log2 = scale * kLog2e;
  a.status = status;
  return launch(prefill_attention_kernel, dim3(unsigned(unit_count), unsigned(kv_heads)), dim3(128), size_t(kSmem),
                stream, true, "prefill_attention", tmq, tmk, tmv, a);
}
