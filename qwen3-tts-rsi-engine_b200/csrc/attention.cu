// Ragged GQA decode attention over the slot-table KV arena.
//
// One query token per slot attends to keys 0..positions[b] of its own slot
// (continuous.py:188-198 mask `indices <= positions`). The KV of one
// (slot, kv_head) pair is contiguous ([slots, kv_heads, capacity, head_dim]),
// so each CTA streams a chunk of keys with untiled bulk copies
// (cp.async.bulk, mbarrier completion) into a two-slot shared-memory ring.
// Grid = (chunks, kv_heads, batch); all G = q_heads/kv_heads query heads of a
// kv head share every K/V tile. Inside a CTA each warp owns 32/G keys of a
// tile: lanes hold 4 (D=128) or 2 (D=64) dims, partial q.k products are
// combined with a 31-shuffle transpose reduction so lane l ends with the score
// of (key l/G, head l%G); softmax is online (base-2 exponent, q pre-scaled by
// scale*log2(e)). Chunks of a slot combine through fp32 partials and an
// atomic ticket: the last chunk CTA merges them in chunk order.
#include "attention.cuh"
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <int D, int G>
struct AttnCfg {
  static constexpr int kDL = D / 32;           // dims per lane
  static constexpr int kKW = 32 / G;           // keys per warp per tile
  static constexpr int kTK = 4 * kKW;          // keys per tile
  static constexpr int kTileBytes = kTK * D * 2;
  static constexpr int kSmem = 2 * 2 * kTileBytes + 1024;
  static constexpr int kPart = G * (D + 2);    // floats per chunk partial
};

// After the call lane l holds the warp-wide sum of v[l].
Q3T_DEV float transpose_reduce32(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool up = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = up ? v[i] : v[i + w];
      const float keep = up ? v[i + w] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  return v[0];
}

template <int D, int G>
__global__ void __launch_bounds__(128)
    decode_attention_kernel(const __nv_bfloat16* __restrict__ query, const __nv_bfloat16* __restrict__ keys,
                            const __nv_bfloat16* __restrict__ values, const int64_t* __restrict__ positions,
                            __nv_bfloat16* __restrict__ out, int kv_heads, int64_t capacity, int64_t context,
                            int window, int rows_per_slot, const int64_t* __restrict__ slots, int64_t ring,
                            int chunk, float qscale, float* __restrict__ partials,
                            unsigned* __restrict__ counters,
                            int max_chunks, unsigned* status) {
  using C = AttnCfg<D, G>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  __nv_bfloat16* kt[2] = {reinterpret_cast<__nv_bfloat16*>(smem),
                          reinterpret_cast<__nv_bfloat16*>(smem + C::kTileBytes)};
  __nv_bfloat16* vt[2] = {reinterpret_cast<__nv_bfloat16*>(smem + 2 * C::kTileBytes),
                          reinterpret_cast<__nv_bfloat16*>(smem + 3 * C::kTileBytes)};
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ float pbuf[4][32];
  __shared__ float wm[4][G], wl[4][G];
  __shared__ float wo[4][G][D];
  __shared__ int last_flag;
  __shared__ int tile_ok;

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  grid_dependency_wait();

  int64_t pos = positions[b];
  // linear arenas hold positions [0, context); ring arenas any position >= 0
  if (pos < 0 || (ring == 0 && pos >= context)) {
    if (c == 0 && h == 0 && threadIdx.x == 0) raise_status(status, kStatusBadIndex);
    pos = pos < 0 ? 0 : context - 1;
  }
  // visible keys: [k_lo, pos]; a sliding window keeps only the last `window`
  const int64_t k_lo = (window > 0 && pos + 1 > window) ? pos + 1 - window : 0;
  const int64_t nkeys = pos + 1;
  const int active = int((nkeys - k_lo + chunk - 1) / chunk);
  if (c >= active) return;
  const int64_t k_begin = k_lo + int64_t(c) * chunk;
  const int64_t k_end = (k_begin + chunk) < nkeys ? (k_begin + chunk) : nkeys;
  const int ntiles = int((k_end - k_begin + C::kTK - 1) / C::kTK);
  // query row b reads the keys of its slot (through the slot table when given)
  const int64_t slot = slots != nullptr ? slots[b / rows_per_slot] : int64_t(b / rows_per_slot);
  const size_t head_base = (size_t(slot) * kv_heads + h) * size_t(capacity) * D;

  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  auto issue = [&](int t) {
    const int64_t t0 = k_begin + int64_t(t) * C::kTK;
    const int64_t n = (k_end - t0) < C::kTK ? (k_end - t0) : C::kTK;
    const uint32_t bytes = uint32_t(n) * D * 2;
    uint64_t* bar = &bars[t & 1];
    mbar_expect_tx(bar, 2 * bytes);
    if (ring > 0) {
      // ring-buffered keys: position p lives in row p % ring; a tile wraps at most once
      const int64_t start = t0 % ring;
      const int64_t n1 = (ring - start) < n ? (ring - start) : n;
      bulk_load(kt[t & 1], keys + head_base + size_t(start) * D, uint32_t(n1) * D * 2, bar);
      bulk_load(vt[t & 1], values + head_base + size_t(start) * D, uint32_t(n1) * D * 2, bar);
      if (n > n1) {
        bulk_load(kt[t & 1] + n1 * D, keys + head_base, uint32_t(n - n1) * D * 2, bar);
        bulk_load(vt[t & 1] + n1 * D, values + head_base, uint32_t(n - n1) * D * 2, bar);
      }
    } else {
      bulk_load(kt[t & 1], keys + head_base + size_t(t0) * D, bytes, bar);
      bulk_load(vt[t & 1], values + head_base + size_t(t0) * D, bytes, bar);
    }
  };
  if (threadIdx.x == 0) {
    issue(0);
    if (ntiles > 1) issue(1);
  }

  // q for the G heads of this kv head, this lane's dims, pre-scaled.
  float q[G][C::kDL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const __nv_bfloat16* qp = query + (size_t(b) * kv_heads * G + size_t(h) * G + g) * D + lane * C::kDL;
#pragma unroll
    for (int d = 0; d < C::kDL; ++d) q[g][d] = __bfloat162float(qp[d]) * qscale;
  }
  float m_run[G], l_run[G], o[G][C::kDL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m_run[g] = -INFINITY;
    l_run[g] = 0.f;
#pragma unroll
    for (int d = 0; d < C::kDL; ++d) o[g][d] = 0.f;
  }

  int failed_tile = -1;
  for (int t = 0; t < ntiles; ++t) {
    // One thread waits with a time bound; the verdict is made uniform before
    // anyone proceeds, then every thread observes the completed phase.
    if (threadIdx.x == 0) tile_ok = mbar_wait(&bars[t & 1], (t >> 1) & 1, status, kStatusTmaTimeout) ? 1 : 0;
    __syncthreads();
    if (!tile_ok) {
      failed_tile = t;
      break;
    }
    mbar_wait(&bars[t & 1], (t >> 1) & 1, status, kStatusTmaTimeout);
    const int64_t t0 = k_begin + int64_t(t) * C::kTK;
    const __nv_bfloat16* ks = kt[t & 1] + warp * C::kKW * D + lane * C::kDL;
    const __nv_bfloat16* vs = vt[t & 1] + warp * C::kKW * D + lane * C::kDL;
    const int64_t wkey0 = t0 + warp * C::kKW;

    float part[32];
#pragma unroll
    for (int kl = 0; kl < C::kKW; ++kl) {
      float kf[C::kDL];
      if constexpr (C::kDL == 4) {
        const uint2 raw = *reinterpret_cast<const uint2*>(ks + kl * D);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 bb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
        kf[0] = a.x; kf[1] = a.y; kf[2] = bb.x; kf[3] = bb.y;
      } else {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(ks + kl * D));
        kf[0] = a.x; kf[1] = a.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float acc = 0.f;
#pragma unroll
        for (int d = 0; d < C::kDL; ++d) acc = fmaf(q[g][d], kf[d], acc);
        part[kl * G + g] = acc;
      }
    }
    float s = transpose_reduce32(part, lane);
    if (wkey0 + lane / G >= k_end) s = -INFINITY;
    // per-head tile max and running max
    float tmax = s;
#pragma unroll
    for (int off = 16; off >= G; off >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, off));
    float alpha[G], mnew[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float mt = __shfl_sync(0xffffffffu, tmax, g);
      mnew[g] = fmaxf(m_run[g], mt);
      alpha[g] = mnew[g] == -INFINITY ? 1.f : exp2f(m_run[g] - mnew[g]);
    }
    const float mine = (G == 1 || (lane & 1) == 0) ? mnew[0] : mnew[G - 1];
    const float p = (s == -INFINITY) ? 0.f : exp2f(s - mine);
    float psum = p;
#pragma unroll
    for (int off = 16; off >= G; off >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, off);
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float ls = __shfl_sync(0xffffffffu, psum, g);
      l_run[g] = l_run[g] * alpha[g] + ls;
      m_run[g] = mnew[g];
#pragma unroll
      for (int d = 0; d < C::kDL; ++d) o[g][d] *= alpha[g];
    }
    pbuf[warp][lane] = p;
    __syncwarp();
    // Keys past the chunk end hold stale shared memory: never touch them.
    const int nvalid = int((k_end - wkey0) < 0 ? 0 : ((k_end - wkey0) > C::kKW ? C::kKW : (k_end - wkey0)));
#pragma unroll 4
    for (int kl = 0; kl < nvalid; ++kl) {
      float vf[C::kDL];
      if constexpr (C::kDL == 4) {
        const uint2 raw = *reinterpret_cast<const uint2*>(vs + kl * D);
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.x));
        const float2 bb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.y));
        vf[0] = a.x; vf[1] = a.y; vf[2] = bb.x; vf[3] = bb.y;
      } else {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(vs + kl * D));
        vf[0] = a.x; vf[1] = a.y;
      }
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float pg = pbuf[warp][kl * G + g];
#pragma unroll
        for (int d = 0; d < C::kDL; ++d) o[g][d] = fmaf(pg, vf[d], o[g][d]);
      }
    }
    __syncwarp();
    __syncthreads();  // every warp is done with ring slot t&1
    if (threadIdx.x == 0 && t + 2 < ntiles) issue(t + 2);
  }
  if (failed_tile >= 0) {
    // Failure path: wait (bounded) for this CTA's copies still in flight
    // (the failed tile and the one prefetched behind it).
    if (threadIdx.x == 0)
      for (int t = failed_tile; t < ntiles && t < failed_tile + 2; ++t)
        mbar_wait(&bars[t & 1], (t >> 1) & 1, status, kStatusTmaTimeout);
    return;
  }

  // ---- merge the four warps
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      wm[warp][g] = m_run[g];
      wl[warp][g] = l_run[g];
    }
#pragma unroll
    for (int d = 0; d < C::kDL; ++d) wo[warp][g][lane * C::kDL + d] = o[g][d];
  }
  __syncthreads();
  float* part = partials + ((size_t(b) * kv_heads + h) * max_chunks + c) * C::kPart;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int g = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = wm[w][g] == -INFINITY ? 0.f : exp2f(wm[w][g] - M);
      L += wl[w][g] * f;
      O += wo[w][g][d] * f;
    }
    if (active == 1) {
      out[(size_t(b) * kv_heads * G + size_t(h) * G + g) * D + d] = __float2bfloat16_rn(O / L);
    } else {
      part[g * (D + 2) + 2 + d] = O;
      if (d == 0) {
        part[g * (D + 2)] = M;
        part[g * (D + 2) + 1] = L;
      }
    }
  }
  if (active == 1) return;

  // ---- chunk combine: last CTA of this (slot, kv head) merges in chunk order
  __threadfence();
  __syncthreads();
  unsigned* counter = counters + size_t(b) * kv_heads + h;
  if (threadIdx.x == 0) last_flag = (atomicAdd(counter, 1u) == unsigned(active - 1));
  __syncthreads();
  if (!last_flag) return;
  __threadfence();
  const float* base = partials + (size_t(b) * kv_heads + h) * max_chunks * C::kPart;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int g = e / D, d = e % D;
    float M = -INFINITY;
    for (int cc = 0; cc < active; ++cc) M = fmaxf(M, __ldcg(base + cc * C::kPart + g * (D + 2)));
    float L = 0.f, O = 0.f;
    for (int cc = 0; cc < active; ++cc) {
      const float* pc = base + cc * C::kPart + g * (D + 2);
      const float mc = __ldcg(pc);
      const float f = mc == -INFINITY ? 0.f : exp2f(mc - M);
      L += __ldcg(pc + 1) * f;
      O += __ldcg(pc + 2 + d) * f;
    }
    out[(size_t(b) * kv_heads * G + size_t(h) * G + g) * D + d] = __float2bfloat16_rn(O / L);
  }
  if (threadIdx.x == 0) *counter = 0u;
}

// Workspace layout: a fixed ticket region (one counter per (row, kv head),
// zero between calls; its last word holds the chunk plan of q3t_attention_plan)
// followed by the chunk partials; fixed so that calls of different shapes
// sharing a workspace never read partials as tickets.
constexpr size_t kMaxTickets = 65536;
constexpr size_t kTicketBytes = kMaxTickets * sizeof(unsigned);
constexpr size_t kPlanSlot = kMaxTickets - 1;

// Keys per chunk for one wave of `wave` resident CTAs over this batch's contexts: the keys of
// all (row, kv head) pairs per CTA, rounded up to chunk_min * 2^k (at most the context and
// kMaxPlannedChunk: inside a decode step the attention's last CTAs are not overlapped by the
// next kernel, so longer chunks lengthen the tail; measured on the talker step at 32 and 64 slots).
constexpr int64_t kMaxPlannedChunk = 1024;
__global__ void attention_plan_kernel(const int64_t* __restrict__ positions, int rows, int kv_heads, int64_t context,
                                      int chunk_min, int wave, unsigned* __restrict__ plan) {
  __shared__ unsigned long long total;
  grid_dependency_wait();
  if (threadIdx.x == 0) total = 0ull;
  __syncthreads();
  unsigned long long mine = 0ull;
  for (int i = threadIdx.x; i < rows; i += blockDim.x) {
    const int64_t p = positions[i];
    mine += uint64_t(p < 0 ? 0 : (p >= context ? context - 1 : p)) + 1ull;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xffffffffu, mine, o);
  if ((threadIdx.x & 31) == 0 && mine != 0ull) atomicAdd(&total, mine);
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long per_cta = (total * uint64_t(kv_heads) + uint64_t(wave) - 1) / uint64_t(wave);
    int64_t chunk = chunk_min;
    while (uint64_t(chunk) < per_cta && chunk < context && chunk < kMaxPlannedChunk) chunk <<= 1;
    *plan = unsigned(chunk);
  }
}

int pick_chunk(int64_t batch, int64_t kv_heads, int64_t context) {
  // Enough CTAs to cover every SM a few times at the bucket's full context.
  const int64_t target = 4LL * sm_count();
  int chunk = 512;
  while (chunk > 64 && batch * kv_heads * ((context + chunk - 1) / chunk) < target) chunk >>= 1;
  return chunk;
}

template <int D, int G>
int launch_attn(const void* q, const void* k, const void* v, const int64_t* pos, void* out, int64_t rows,
                int64_t rows_per_slot, const int64_t* slots, int64_t ring, int64_t kv_heads, int64_t capacity,
                int64_t context, int64_t window, float scale, void* ws, unsigned* status, void* stream) {
  using C = AttnCfg<D, G>;
  const int64_t span = window > 0 && window < context ? window : context;
  const int chunk = pick_chunk(rows, kv_heads, span);
  const int max_chunks = int((span + chunk - 1) / chunk);
  static PerDevice smem_once;
  if (const int rc = smem_limit(smem_once, decode_attention_kernel<D, G>, C::kSmem, "attention: set smem")) return rc;
  unsigned* counters = static_cast<unsigned*>(ws);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(ws) + kTicketBytes);
  return launch(decode_attention_kernel<D, G>, dim3(max_chunks, unsigned(kv_heads), unsigned(rows)), dim3(128),
                size_t(C::kSmem), stream, true, "decode_attention", static_cast<const __nv_bfloat16*>(q),
                static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), pos,
                static_cast<__nv_bfloat16*>(out), int(kv_heads), capacity, context, int(window), int(rows_per_slot),
                slots, ring, chunk, scale * kLog2e, partials, counters, max_chunks, status);
}

size_t attn_workspace(int64_t batch, int64_t q_heads, int64_t kv_heads_unused, int64_t head_dim, int64_t context) {
  (void)kv_heads_unused;
  // worst case over G: partial floats per (b, kv head, chunk) = G*(D+2); bound with q_heads*(D+2) per (b, chunk)
  const int chunk = 64;
  const int64_t max_chunks = (context + chunk - 1) / chunk;
  return kTicketBytes + size_t(batch) * max_chunks * q_heads * (head_dim + 2) * sizeof(float);
}

}  // namespace

extern "C" size_t q3t_decode_attention_workspace_bytes(int64_t batch, int64_t q_heads, int64_t head_dim,
                                                       int64_t context) {
  if (batch < 1 || q_heads < 1 || head_dim < 1 || context < 1) return 0;
  return attn_workspace(batch, q_heads, 0, head_dim, context);
}

extern "C" int q3t_decode_attention_qkv(const void* qkv, int64_t qkv_stride, const void* q_norm_weight,
                                        const void* k_norm_weight, float eps, const void* cos_table,
                                        const void* sin_table, int64_t table_len, const int64_t* rotary_positions,
                                        void* keys, void* values, const int64_t* positions, void* out, int64_t rows,
                                        int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t arena_slots,
                                        int64_t capacity, int64_t context, float scale, void* workspace,
                                        size_t workspace_bytes, unsigned* status, void* stream) {
  return q3t_decode_attention_qkv_ex(qkv, qkv_stride, q_norm_weight, k_norm_weight, eps, cos_table, sin_table,
                                     table_len, rotary_positions, keys, values, positions, out, rows, q_heads,
                                     kv_heads, head_dim, arena_slots, capacity, context, scale, workspace,
                                     workspace_bytes, nullptr, 0, nullptr, 0, status, stream);
}

extern "C" int q3t_decode_attention_qkv_ex(const void* qkv, int64_t qkv_stride, const void* q_norm_weight,
                                           const void* k_norm_weight, float eps, const void* cos_table,
                                           const void* sin_table, int64_t table_len,
                                           const int64_t* rotary_positions, void* keys, void* values,
                                           const int64_t* positions, void* out, int64_t rows, int64_t q_heads,
                                           int64_t kv_heads, int64_t head_dim, int64_t arena_slots,
                                           int64_t capacity, int64_t context, float scale, void* workspace,
                                           size_t workspace_bytes, const void* prefetch0, size_t prefetch0_bytes,
                                           const void* prefetch1, size_t prefetch1_bytes, unsigned* status,
                                           void* stream) {
  if ((prefetch0_bytes && (!prefetch0 || !aligned16(prefetch0) || prefetch0_bytes % 16)) ||
      (prefetch1_bytes && (!prefetch1 || !aligned16(prefetch1) || prefetch1_bytes % 16)))
    return fail(Q3T_EINVAL, "attention_qkv: prefetch ranges need 16-byte alignment and size");
  if (!qkv || !cos_table || !sin_table || !rotary_positions || !keys || !values || !positions || !out)
    return fail(Q3T_EINVAL, "attention_qkv: null pointer");
  if (rows < 1 || rows > 65535 || kv_heads < 1 || q_heads % kv_heads || arena_slots < rows || table_len < 1)
    return fail(Q3T_EINVAL, "attention_qkv: invalid row or head geometry");
  if (context < 1 || context > capacity) return fail(Q3T_EINVAL, "Attention context must fit the KV arena");
  if (size_t(rows) * size_t(kv_heads) > kPlanSlot) return fail(Q3T_EUNSUPPORTED, "attention: rows x kv_heads > 65535");
  const int64_t g = q_heads / kv_heads;
  if (!attention_mma_supported(head_dim, g))
    return fail(Q3T_EUNSUPPORTED, "attention_qkv: head_dim %lld with %lld query heads per kv head",
                (long long)head_dim, (long long)g);
  if (qkv_stride < (q_heads + 2 * kv_heads) * head_dim || qkv_stride % 8 || !aligned16(qkv) || !aligned16(keys) ||
      !aligned16(values))
    return fail(Q3T_EINVAL, "attention_qkv: 16-byte aligned rows required");
  const size_t need = attn_workspace(rows, q_heads, kv_heads, head_dim, context);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(Q3T_ESPACE, "attention: workspace needs %zu bytes", need);
  AttentionCall call = {};
  call.query = qkv;
  call.keys = keys;
  call.values = values;
  call.positions = positions;
  call.out = out;
  call.rows = rows;
  call.rows_per_slot = 1;
  call.slots = nullptr;
  call.q_heads = q_heads;
  call.kv_heads = kv_heads;
  call.head_dim = head_dim;
  call.arena_slots = arena_slots;
  call.capacity = capacity;
  call.context = context;
  call.window = 0;
  call.scale = scale;
  call.chunk = pick_chunk(rows, kv_heads, context);
  call.max_chunks = int((context + call.chunk - 1) / call.chunk);
  call.counters = static_cast<unsigned*>(workspace);
  call.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kTicketBytes);
  call.plan = call.counters + kPlanSlot;
  call.status = status;
  call.stream = stream;
  call.prefetch[0] = prefetch0;
  call.prefetch_bytes[0] = prefetch0_bytes;
  call.prefetch[1] = prefetch1;
  call.prefetch_bytes[1] = prefetch1_bytes;
  return launch_attention_fused(call, qkv, qkv_stride, q_norm_weight, k_norm_weight, eps, cos_table, sin_table,
                                table_len, rotary_positions);
}

extern "C" int q3t_decode_attention(const void* query, const void* keys, const void* values, const int64_t* positions,
                                    void* out, int64_t rows, int64_t rows_per_slot, const int64_t* slots, int64_t ring,
                                    int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t arena_slots,
                                    int64_t capacity, int64_t context, int64_t window, float scale, void* workspace,
                                    size_t workspace_bytes, unsigned* status, void* stream) {
  if (!query || !keys || !values || !positions || !out) return fail(Q3T_EINVAL, "attention: null pointer");
  if (rows < 1 || rows > 65535 || rows_per_slot < 1 || rows % rows_per_slot || kv_heads < 1 || kv_heads > 65535 ||
      q_heads % kv_heads || window < 0 || arena_slots < 1)
    return fail(Q3T_EINVAL, "attention: invalid row or head geometry");
  if (slots == nullptr && arena_slots * rows_per_slot < rows)
    return fail(Q3T_EINVAL, "attention: more query rows than arena slots");
  if (context < 1 || context > capacity) return fail(Q3T_EINVAL, "Attention context must fit the KV arena");
  if (size_t(rows) * size_t(kv_heads) > kPlanSlot) return fail(Q3T_EUNSUPPORTED, "attention: rows x kv_heads > 65535");
  if (ring < 0 || (ring > 0 && (ring != capacity || window < 1 || window > ring)))
    return fail(Q3T_EINVAL, "attention: a ring arena needs capacity == ring and 1 <= window <= ring");
  if (!aligned16(keys) || !aligned16(values) || !aligned16(query))
    return fail(Q3T_EINVAL, "attention: 16-byte alignment");
  const int64_t g = q_heads / kv_heads;
  const size_t need = attn_workspace(rows, q_heads, kv_heads, head_dim, context);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(Q3T_ESPACE, "attention: workspace needs %zu bytes", need);
  if (ring == 0 && attention_mma_supported(head_dim, g)) {
    // linear arenas: tensor-core kernel (TMA-swizzled K/V tiles, mma.sync fragments)
    const int64_t span = window > 0 && window < context ? window : context;
    AttentionCall call = {};
    call.query = query;
    call.keys = keys;
    call.values = values;
    call.positions = positions;
    call.out = out;
    call.rows = rows;
    call.rows_per_slot = rows_per_slot;
    call.slots = slots;
    call.q_heads = q_heads;
    call.kv_heads = kv_heads;
    call.head_dim = head_dim;
    call.arena_slots = arena_slots;
    call.capacity = capacity;
    call.context = context;
    call.window = window;
    call.scale = scale;
    call.chunk = pick_chunk(rows, kv_heads, span);
    call.max_chunks = int((span + call.chunk - 1) / call.chunk);
    call.counters = static_cast<unsigned*>(workspace);
    call.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kTicketBytes);
    call.plan = (window == 0 && rows_per_slot == 1) ? call.counters + kPlanSlot : nullptr;
    call.status = status;
    call.stream = stream;
    return launch_attention_mma(call);
  }
#define Q3T_ATTN(DD, GG)                                                                                       \
  if (head_dim == DD && g == GG)                                                                               \
    return launch_attn<DD, GG>(query, keys, values, positions, out, rows, rows_per_slot, slots, ring, kv_heads, \
                               capacity, context, window, scale, workspace, status, stream);
  Q3T_ATTN(128, 2)
  Q3T_ATTN(128, 1)
  Q3T_ATTN(64, 1)
  Q3T_ATTN(64, 2)
#undef Q3T_ATTN
  return fail(Q3T_EUNSUPPORTED, "attention: head_dim %lld with %lld query heads per kv head", (long long)head_dim,
              (long long)g);
}

// ======================================================================
// Allocation-free variant.
//
// Some callers cannot allocate device memory at all: a host runtime that
// owns a fixed, pre-reserved memory pool, a foreign-language embedding that
// links this library but has no CUDA allocator of its own, or code running
// while allocation is forbidden. For them the split-KV scratch (tickets and
// chunk partials) lives in one file-scope device array of fixed size instead
// of a caller workspace. Every GPU that loads this library holds the array
// (4 MiB) until the process exits.
//
// The array is shared by every call on a device and keeps the previous
// call's contents; each call clears the tickets it uses before its kernel
// runs. Calls whose kernels overlap on the GPU (different streams, no
// ordering between them) race on the array and must not be issued.
// ======================================================================
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB
constexpr size_t kStaticTickets = 16384;                  // first 64 KiB
constexpr size_t kStaticTicketBytes = kStaticTickets * sizeof(unsigned);

__device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

// The array's device address differs per CUDA context, so the resolved address is
// cached per device together with the unique id of the context it was resolved in
// (cuCtxGetId; ids are never reused within a process): a caller on a non-primary
// context, or one that reset the device since, gets the address re-resolved.
using CtxGetCurrent = CUresult (*)(CUcontext*);
using CtxGetId = CUresult (*)(CUcontext, unsigned long long*);

struct ScratchAddress {
  unsigned long long context_id = 0;
  void* address = nullptr;
};
std::mutex g_static_mutex;
ScratchAddress g_static_address[64];

int current_context_id(unsigned long long* id) {
  static CtxGetCurrent get_current = nullptr;
  static CtxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrent>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetId>(p);
  });
  if (get_current == nullptr || get_id == nullptr)
    return fail(Q3T_ECUDA, "attention (no-alloc): context queries unavailable");
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr || get_id(ctx, id) != CUDA_SUCCESS)
    return fail(Q3T_ECUDA, "attention (no-alloc): no current CUDA context");
  return Q3T_OK;
}

// Device address of g_attention_scratch in the current context. The first call in a
// context resolves it with cudaGetSymbolAddress (that device and context current).
int static_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(Q3T_ECUDA, "attention (no-alloc): no current CUDA device");
  unsigned long long id = 0;
  if (const int rc = current_context_id(&id)) return rc;
  std::lock_guard<std::mutex> lock(g_static_mutex);
  ScratchAddress& entry = g_static_address[dev];
  if (entry.address == nullptr || entry.context_id != id) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (err != cudaSuccess || p == nullptr)
      return fail(Q3T_ECUDA, "attention (no-alloc): cudaGetSymbolAddress failed: %s", cudaGetErrorString(err));
    entry.address = p;
    entry.context_id = id;
  }
  *out = entry.address;
  return Q3T_OK;
}

template <int D, int G>
int launch_attn_static(const void* q, const void* k, const void* v, const int64_t* pos, void* out, int64_t rows,
                       int64_t rows_per_slot, int64_t kv_heads, int64_t capacity, int64_t context, int64_t window,
                       float scale, unsigned* status, void* stream) {
  using C = AttnCfg<D, G>;
  const int64_t span = window > 0 && window < context ? window : context;
  const int chunk = pick_chunk(rows, kv_heads, span);
  const int max_chunks = int((span + chunk - 1) / chunk);
  const size_t tickets = size_t(rows) * size_t(kv_heads);
  const size_t partial_bytes = tickets * size_t(max_chunks) * C::kPart * sizeof(float);
  if (tickets > kStaticTickets || kStaticTicketBytes + partial_bytes > kStaticScratchBytes)
    return fail(Q3T_ESPACE,
                "attention (no-alloc): needs %zu tickets and %zu partial bytes; the static scratch holds %zu tickets "
                "and %zu bytes",
                tickets, partial_bytes, kStaticTickets, kStaticScratchBytes - kStaticTicketBytes);
  void* base = nullptr;
  int rc = static_scratch(&base);
  if (rc != Q3T_OK) return rc;
  static PerDevice smem_once;
  rc = smem_limit(smem_once, decode_attention_kernel<D, G>, C::kSmem, "attention (no-alloc): set smem");
  if (rc != Q3T_OK) return rc;
  if (cudaMemsetAsync(base, 0, tickets * sizeof(unsigned), as_stream(stream)) != cudaSuccess)
    return check_cuda("attention (no-alloc): clear tickets");
  unsigned* counters = static_cast<unsigned*>(base);
  float* partials = reinterpret_cast<float*>(static_cast<char*>(base) + kStaticTicketBytes);
  return launch(decode_attention_kernel<D, G>, dim3(max_chunks, unsigned(kv_heads), unsigned(rows)), dim3(128),
                size_t(C::kSmem), stream, false, "decode_attention_noalloc", static_cast<const __nv_bfloat16*>(q),
                static_cast<const __nv_bfloat16*>(k), static_cast<const __nv_bfloat16*>(v), pos,
                static_cast<__nv_bfloat16*>(out), int(kv_heads), capacity, context, int(window), int(rows_per_slot),
                static_cast<const int64_t*>(nullptr), int64_t(0), chunk, scale * kLog2e, partials, counters,
                max_chunks, status);
}

}  // namespace

extern "C" int q3t_decode_attention_noalloc(const void* query, const void* keys, const void* values,
                                            const int64_t* positions, void* out, int64_t rows, int64_t rows_per_slot,
                                            int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t arena_slots,
                                            int64_t capacity, int64_t context, int64_t window, float scale,
                                            unsigned* status, void* stream) {
  if (!query || !keys || !values || !positions || !out) return fail(Q3T_EINVAL, "attention (no-alloc): null pointer");
  if (rows < 1 || rows > 65535 || rows_per_slot < 1 || rows % rows_per_slot || kv_heads < 1 || kv_heads > 65535 ||
      q_heads % kv_heads || window < 0 || arena_slots < 1)
    return fail(Q3T_EINVAL, "attention (no-alloc): invalid row or head geometry");
  if (arena_slots * rows_per_slot < rows)
    return fail(Q3T_EINVAL, "attention (no-alloc): more query rows than arena slots");
  if (context < 1 || context > capacity) return fail(Q3T_EINVAL, "Attention context must fit the KV arena");
  if (!aligned16(keys) || !aligned16(values) || !aligned16(query))
    return fail(Q3T_EINVAL, "attention (no-alloc): 16-byte alignment");
  const int64_t g = q_heads / kv_heads;
#define Q3T_ATTN_STATIC(DD, GG)                                                                                \
  if (head_dim == DD && g == GG)                                                                               \
    return launch_attn_static<DD, GG>(query, keys, values, positions, out, rows, rows_per_slot, kv_heads,    \
                                      capacity, context, window, scale, status, stream);
  Q3T_ATTN_STATIC(128, 2)
  Q3T_ATTN_STATIC(128, 1)
  Q3T_ATTN_STATIC(64, 1)
  Q3T_ATTN_STATIC(64, 2)
#undef Q3T_ATTN_STATIC
  return fail(Q3T_EUNSUPPORTED, "attention (no-alloc): head_dim %lld with %lld query heads per kv head",
              (long long)head_dim, (long long)g);
}

extern "C" int q3t_attention_plan(const int64_t* positions, int64_t rows, int64_t q_heads, int64_t kv_heads,
                                  int64_t head_dim, int64_t context, void* workspace, size_t workspace_bytes,
                                  void* stream) {
  if (!positions || !workspace || rows < 1 || rows > 65535 || kv_heads < 1 || q_heads % kv_heads || context < 1)
    return fail(Q3T_EINVAL, "attention_plan: invalid arguments");
  if (workspace_bytes < kTicketBytes || !aligned16(workspace))
    return fail(Q3T_ESPACE, "attention_plan: workspace needs %zu bytes", kTicketBytes);
  const int wave = attention_wave_ctas(head_dim, q_heads / kv_heads, true);
  if (wave < 1) return fail(Q3T_EUNSUPPORTED, "attention_plan: unsupported head geometry");
  return launch(attention_plan_kernel, dim3(1), dim3(256), 0, stream, true, "attention_plan", positions, int(rows),
                int(kv_heads), context, pick_chunk(rows, kv_heads, context), wave,
                static_cast<unsigned*>(workspace) + kPlanSlot);
}
