// Ragged GQA decode attention on tensor-core fragments (mma.sync m16n8k16).
//
// Decode attention is HBM-bound, but computing q.k and p.V with fp32 CUDA-core
// FMAs costs ~40 warp instructions per key and made the previous kernel
// issue-bound. Here the G query heads of one kv head are the M rows of a
// 16-row fragment (rows >= G are zero), so per warp and 16 keys:
//   S = Q K^T : 2 n-tiles x (D/16) k-steps of m16n8k16, K from ldmatrix,
//   P = exp2(S - m) kept in registers as the A fragment of the next product,
//   O += P V  : (D/8) n-tiles x 1 k-step, V from ldmatrix.trans,
// i.e. ~100 instructions per 16 keys. K/V tiles (64 keys) arrive by 2-D TMA
// with 128-byte swizzle (conflict-free ldmatrix) into a 2-stage ring (three
// CTAs per SM keep six tiles in flight; contexts of one tile use a one-stage
// instance, four CTAs per SM), the query rows by one bulk copy on
// the first tile's barrier; each of
// the 4 warps owns 16 keys of a tile and keeps its own online softmax, and
// the warps, then the chunk CTAs of a slot (fp32 partials + ticket, chunk
// order), are merged at the end.
#include "attention.cuh"
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <int D, int G, int STAGES = 2>
struct MmaCfg {
  static constexpr int kTile = 64;                    // keys per tile, 16 per warp
  static constexpr int kBoxes = D / 64;               // 128-byte TMA boxes per key row
  static constexpr int kBoxBytes = kTile * 128;       // 8 KB
  static constexpr int kStageBytes = 2 * kBoxes * kBoxBytes;
  // 2 x 32 KB ring: three CTAs fit on an SM. One stage for contexts of one tile (the code
  // predictor's 17 positions): four CTAs per SM, so 512 (row, kv head) CTAs run as one wave.
  static constexpr int kStages = STAGES;
  static constexpr int kSmem = kStages * kStageBytes + 1024;
  static constexpr int kPart = G * (D + 2);
  static constexpr int kQBytes = G * D * 2;           // the G query rows of one (row, kv head)
};

Q3T_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
Q3T_DEV void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// D (16x8 fp32) += A (16x16 bf16, rows g/g+8) * B (16x8 bf16); a1 = a3 = 0 (rows 8..15 unused).
Q3T_DEV void mma_rows8(float (&c)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  const uint32_t zero = 0u;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(zero), "r"(a2), "r"(zero), "r"(b0), "r"(b1));
}
Q3T_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// Clear the bf16 halves of a B fragment register whose key index is invalid.
Q3T_DEV uint32_t keep_keys(uint32_t v, int key_lo, int valid) {
  if (key_lo >= valid) v &= 0xFFFF0000u;
  if (key_lo + 1 >= valid) v &= 0x0000FFFFu;
  return v;
}

// Decode step with the per-head q/k RMSNorm, RoPE and the K/V write fused in
// (FUSED = true): the kernel reads the raw QKV projection row instead of a
// finished query. Every chunk CTA of (row, kv head) normalises and rotates its
// G query heads in shared memory; the CTA of the last chunk (the one whose key
// range contains the row's position p) also builds the new key/value of p,
// stores them to the arena and patches them into its shared tile before using
// it, so no other CTA of the launch depends on that write.
struct FusedQKV {
  const __nv_bfloat16* qkv;     // [rows, (q_heads + 2 kv_heads) * D], row stride qkv_stride
  int64_t qkv_stride;
  const __nv_bfloat16* q_norm;  // [D] or null (no per-head norm)
  const __nv_bfloat16* k_norm;
  float eps;
  const __nv_bfloat16* cos;     // [table_len, D]
  const __nv_bfloat16* sin;
  int64_t table_len;
  const int64_t* rot_pos;       // [rows]
  __nv_bfloat16* keys;          // arena [slots, kv_heads, capacity, D] (row b = slot b)
  __nv_bfloat16* values;
  // L2 prefetch of up to two ranges (the next projections' weights): the key stream leaves
  // HBM bandwidth unused, and weights already in L2 shorten the latency-bound GEMMs that follow
  const uint8_t* pf[2];
  uint64_t pf_bytes[2];
};

// Per-head RMSNorm (optional weight) and rotate-half RoPE of D values, one warp,
// lane l holding dims [l*D/32, (l+1)*D/32); bf16 rounding after each op as the
// standalone q/k kernel does.
template <int D>
Q3T_DEV void norm_rope(float (&x)[D / 32], const __nv_bfloat16* w, float eps, const __nv_bfloat16* cs,
                       const __nv_bfloat16* sn, int lane) {
  constexpr int DL = D / 32;
  float y[DL];
  if (w != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int d = 0; d < DL; ++d) ss += x[d] * x[d];
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / float(D) + eps);
#pragma unroll
    for (int d = 0; d < DL; ++d) y[d] = bf16r(__bfloat162float(w[lane * DL + d]) * bf16r(x[d] * inv));
  } else {
#pragma unroll
    for (int d = 0; d < DL; ++d) y[d] = x[d];
  }
#pragma unroll
  for (int d = 0; d < DL; ++d) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[d], 16);
    const float rot = lane < 16 ? -partner : partner;
    x[d] = bf16r(bf16r(y[d] * __bfloat162float(cs[lane * DL + d])) + bf16r(rot * __bfloat162float(sn[lane * DL + d])));
  }
}

template <int D, int G, bool FUSED, int STAGES>
__global__ void __launch_bounds__(128, STAGES == 1 ? 4 : 3)
    decode_attention_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                                const __nv_bfloat16* __restrict__ query, const int64_t* __restrict__ positions,
                                __nv_bfloat16* __restrict__ out, int kv_heads, int64_t capacity, int64_t context,
                                int window, int rows_per_slot, const int64_t* __restrict__ slots, int chunk_min,
                                const unsigned* __restrict__ plan, float qscale, float* __restrict__ partials,
                                unsigned* __restrict__ counters,
                                int max_chunks, unsigned* status, const FusedQKV f) {
  using C = MmaCfg<D, G, STAGES>;
  constexpr int S = C::kStages;
  constexpr int KS = D / 16;  // k-steps of S = Q K^T
  constexpr int NT = D / 8;   // n-tiles of O = P V
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[S];
  __shared__ __align__(16) __nv_bfloat16 qs[G * D];
  __shared__ float wm[4][G], wl[4][G];
  __shared__ float wo[4][G][D];
  __shared__ int last_flag;

  const int c = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  grid_dependency_wait();
  if constexpr (FUSED) {
    if (threadIdx.x == 32) {  // this CTA's share of the prefetch ranges, requested once
      const uint64_t ctas = uint64_t(gridDim.x) * gridDim.y * gridDim.z;
      const uint64_t id = blockIdx.x + uint64_t(gridDim.x) * (blockIdx.y + uint64_t(gridDim.y) * blockIdx.z);
#pragma unroll
      for (int r = 0; r < 2; ++r)
        if (f.pf[r] != nullptr) prefetch_l2_share(f.pf[r], f.pf_bytes[r], id, ctas);
    }
  }

  int64_t pos = positions[b];
  // Keys per chunk: the step's plan (q3t_attention_plan: one wave of resident CTAs for this
  // batch's contexts) when present. Any multiple of 64 >= chunk_min is a valid split of the
  // grid's chunk range, so a stale plan costs speed only.
  int chunk = chunk_min;
  if (plan != nullptr) {
    const unsigned planned = *plan;
    if (planned >= unsigned(chunk_min) && planned % 64u == 0u && planned <= unsigned(1 << 30)) chunk = int(planned);
  }
  const bool pos_ok = pos >= 0 && pos < context;
  if (pos < 0 || pos >= context) {
    if (c == 0 && h == 0 && threadIdx.x == 0) raise_status(status, kStatusBadIndex);
    pos = pos < 0 ? 0 : context - 1;
  }
  const int64_t k_lo = (window > 0 && pos + 1 > window) ? pos + 1 - window : 0;
  const int64_t nkeys = pos + 1;
  const int active = int((nkeys - k_lo + chunk - 1) / chunk);
  if (c >= active) return;
  const int64_t k_begin = k_lo + int64_t(c) * chunk;
  const int64_t k_end = (k_begin + chunk) < nkeys ? (k_begin + chunk) : nkeys;
  const int ntiles = int((k_end - k_begin + C::kTile - 1) / C::kTile);
  const int64_t slot = slots != nullptr ? slots[b / rows_per_slot] : int64_t(b / rows_per_slot);
  const int64_t row0 = (slot * kv_heads + h) * capacity + k_begin;  // tensor-map row of the first key

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
  }
  __syncthreads();
  auto stage_k = [&](int s) { return smem + s * C::kStageBytes; };
  auto stage_v = [&](int s) { return smem + s * C::kStageBytes + C::kBoxes * C::kBoxBytes; };
  auto issue = [&](int t) {
    const int s = t % S;
    const uint64_t pol = policy_evict_first();
    mbar_expect_tx(&full[s], C::kStageBytes + (t == 0 ? C::kQBytes : 0));
    if (t == 0) {  // the query rows ride on the first tile's barrier
      const __nv_bfloat16* qsrc = FUSED ? f.qkv + int64_t(b) * f.qkv_stride + int64_t(h) * G * D
                                        : query + (int64_t(b) * kv_heads + h) * G * D;
      bulk_load(qs, qsrc, uint32_t(C::kQBytes), &full[0]);
    }
    const int y = int(row0 + int64_t(t) * C::kTile);
#pragma unroll
    for (int bx = 0; bx < C::kBoxes; ++bx) {
      tma_load_2d(stage_k(s) + bx * C::kBoxBytes, &tmk, &full[s], bx * 64, y, pol);
      tma_load_2d(stage_v(s) + bx * C::kBoxBytes, &tmv, &full[s], bx * 64, y, pol);
    }
  };
  if (threadIdx.x == 0)
    for (int t = 0; t < ntiles && t < S; ++t) issue(t);

  // ---- fused: rotary row, and (last chunk only) the new key/value of position p
  constexpr int DL = D / 32;
  const bool owns_p = FUSED && c == active - 1;
  const int t_p = int((pos - k_begin) / C::kTile);   // tile of this chunk holding p (last chunk)
  float knew[DL], vnew[DL];
  int64_t rp = 0;
  if constexpr (FUSED) {
    rp = f.rot_pos[b];
    if (rp < 0 || rp >= f.table_len) {
      if (c == 0 && h == 0 && threadIdx.x == 0) raise_status(status, kStatusBadIndex);
      rp = rp < 0 ? 0 : f.table_len - 1;
    }
    if (owns_p && warp == 3) {
      const int q_heads = kv_heads * G;
      const __nv_bfloat16* row = f.qkv + int64_t(b) * f.qkv_stride;
#pragma unroll
      for (int d = 0; d < DL; ++d) {
        knew[d] = __bfloat162float(row[int64_t(q_heads + h) * D + lane * DL + d]);
        vnew[d] = __bfloat162float(row[int64_t(q_heads + kv_heads + h) * D + lane * DL + d]);
      }
      norm_rope<D>(knew, f.k_norm, f.eps, f.cos + rp * D, f.sin + rp * D, lane);
      if (pos_ok) {
        const size_t dst = ((size_t(slot) * kv_heads + h) * size_t(capacity) + size_t(pos)) * D + lane * DL;
#pragma unroll
        for (int d = 0; d < DL; ++d) {
          f.keys[dst + d] = __float2bfloat16_rn(knew[d]);
          f.values[dst + d] = __float2bfloat16_rn(vnew[d]);
        }
      }
    }
  }

  uint32_t qa[KS][2];  // Q as the A fragment (rows g < G real, rows >= G and g+8 zero), filled at tile 0
  float o[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;

  const int mi = lane >> 3, ri = lane & 7;
  int failed = -1;
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % S;
    // Every thread waits for the stage itself (bounded); a timeout is made uniform by the
    // end-of-tile barrier below, which is the only CTA barrier per tile.
    const bool tile_ok = mbar_wait(&full[s], (t / S) & 1, status, kStatusTmaTimeout);
    if constexpr (FUSED) {
      if (t == 0 || (owns_p && t == t_p)) {  // CTA-uniform condition
        if (t == 0 && warp < G) {            // warp w finishes query head w in place
          float x[DL];
          __nv_bfloat16* qh = qs + warp * D + lane * DL;
#pragma unroll
          for (int d = 0; d < DL; ++d) x[d] = __bfloat162float(qh[d]);
          norm_rope<D>(x, f.q_norm, f.eps, f.cos + rp * D, f.sin + rp * D, lane);
#pragma unroll
          for (int d = 0; d < DL; ++d) qh[d] = __float2bfloat16_rn(x[d]);
        }
        if (owns_p && t == t_p && warp == 3) {  // the freshly built K/V of p replace the stale arena row
          const int rr = int(pos - k_begin) - t_p * C::kTile;
          const int col = (lane * DL) % 64, bx = (lane * DL) / 64;
          const int off = bx * C::kBoxBytes + rr * 128 + ((((col >> 3) ^ (rr & 7)) & 7) << 4) + (col & 7) * 2;
          __nv_bfloat16 kb[DL], vb[DL];
#pragma unroll
          for (int d = 0; d < DL; ++d) {
            kb[d] = __float2bfloat16_rn(knew[d]);
            vb[d] = __float2bfloat16_rn(vnew[d]);
          }
          memcpy(stage_k(s) + off, kb, sizeof(kb));
          memcpy(stage_v(s) + off, vb, sizeof(vb));
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // before TMA refills this stage
        }
        __syncthreads();
      }
    }
    if (t == 0) {
      const bool real = g < G;
      const __nv_bfloat16* qp = qs + (real ? g : 0) * D;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        qa[kk][0] = real ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * t4) : 0u;
        qa[kk][1] = real ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 8 + 2 * t4) : 0u;
      }
    }
    const uint32_t kbase = smem_u32(stage_k(s)), vbase = smem_u32(stage_v(s));
    const int64_t key0 = k_begin + int64_t(t) * C::kTile + 16 * warp;  // this warp's first key
    const int valid = int((k_end - key0) < 0 ? 0 : ((k_end - key0) > 16 ? 16 : (k_end - key0)));

    // ---- S = Q K^T (16 keys: n-tiles 0 and 1; even and odd k-steps accumulate
    // separately so four independent mma chains are in flight)
    float sacc[4][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
      const int key = 16 * warp + (mi >> 1) * 8 + ri;
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        const int ch = 2 * kk + (mi & 1);
        const uint32_t addr = kbase + (ch >> 3) * C::kBoxBytes + key * 128 + (((ch & 7) ^ (key & 7)) << 4);
        uint32_t b00, b01, b10, b11;
        ldsm_x4(addr, b00, b01, b10, b11);
        mma_rows8(sacc[(kk & 1) * 2 + 0], qa[kk][0], qa[kk][1], b00, b01);
        mma_rows8(sacc[(kk & 1) * 2 + 1], qa[kk][0], qa[kk][1], b10, b11);
      }
    }
    // ---- online softmax on row g (keys 2t4, 2t4+1 of each n-tile)
    float sv[4] = {(sacc[0][0] + sacc[2][0]) * qscale, (sacc[0][1] + sacc[2][1]) * qscale,
                   (sacc[1][0] + sacc[3][0]) * qscale, (sacc[1][1] + sacc[3][1]) * qscale};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int k = (e >> 1) * 8 + 2 * t4 + (e & 1);
      if (k >= valid) sv[e] = -INFINITY;
    }
    float mt = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
    mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
    // Lazy rescaling: the running reference max only moves when a score exceeds it by
    // more than 2^8 (p stays <= 256, exact in fp32 and bf16's range); the final O / L
    // and the chunk merge are invariant to the reference chosen. Most tiles then skip
    // the 2 x D/8 rescale multiplies (the skip is warp-uniform).
    const float m_new = (m_run == -INFINITY || mt > m_run + 8.f) ? fmaxf(m_run, mt) : m_run;
    const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_run - m_new);
    float p[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) p[e] = sv[e] == -INFINITY ? 0.f : exp2f(sv[e] - m_new);
    float ps = (p[0] + p[1]) + (p[2] + p[3]);
    ps += __shfl_xor_sync(0xffffffffu, ps, 1);
    ps += __shfl_xor_sync(0xffffffffu, ps, 2);
    l_run = l_run * alpha + ps;
    if (__any_sync(0xffffffffu, m_new != m_run)) {
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        o[n][0] *= alpha;
        o[n][1] *= alpha;
      }
    }
    m_run = m_new;
    const uint32_t pa0 = pack_bf16x2(p[0], p[1]), pa2 = pack_bf16x2(p[2], p[3]);

    // ---- O += P V (keys of this warp; stale rows past the chunk end are zeroed)
    {
      const int key = 16 * warp + (mi & 1) * 8 + ri;
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        const int ch = 2 * np + (mi >> 1);
        const uint32_t addr = vbase + (ch >> 3) * C::kBoxBytes + key * 128 + (((ch & 7) ^ (key & 7)) << 4);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_trans(addr, v0, v1, v2, v3);
        if (valid < 16) {
          v0 = keep_keys(v0, 2 * t4, valid);
          v1 = keep_keys(v1, 8 + 2 * t4, valid);
          v2 = keep_keys(v2, 2 * t4, valid);
          v3 = keep_keys(v3, 8 + 2 * t4, valid);
        }
        mma_rows8(o[2 * np], pa0, pa2, v0, v1);
        mma_rows8(o[2 * np + 1], pa0, pa2, v2, v3);
      }
    }
    // all warps are done with stage s (and agree whether it ever landed)
    if (__syncthreads_or(!tile_ok)) {
      failed = t;
      break;
    }
    if (threadIdx.x == 0 && t + S < ntiles) issue(t + S);
  }
  if (failed >= 0) {
    // Failure path: wait (bounded) for the copies this CTA still has in flight.
    if (threadIdx.x == 0)
      for (int t = failed; t < ntiles && t < failed + S; ++t) mbar_wait(&full[t % S], (t / S) & 1, status, kStatusTmaTimeout);
    return;
  }

  // ---- merge the four warps (rows g < G live in lanes 0 .. 4G-1)
  if (g < G) {
    if (t4 == 0) {
      wm[warp][g] = m_run;
      wl[warp][g] = l_run;
    }
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      wo[warp][g][8 * n + 2 * t4] = o[n][0];
      wo[warp][g][8 * n + 2 * t4 + 1] = o[n][1];
    }
  }
  __syncthreads();
  float* part = partials + ((size_t(b) * kv_heads + h) * max_chunks + c) * C::kPart;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int gg = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, wm[w][gg]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float f = wm[w][gg] == -INFINITY ? 0.f : exp2f(wm[w][gg] - M);
      L += wl[w][gg] * f;
      O += wo[w][gg][d] * f;
    }
    if (active == 1) {
      out[(size_t(b) * kv_heads * G + size_t(h) * G + gg) * D + d] = __float2bfloat16_rn(O / L);
    } else {
      part[gg * (D + 2) + 2 + d] = O;
      if (d == 0) {
        part[gg * (D + 2)] = M;
        part[gg * (D + 2) + 1] = L;
      }
    }
  }
  if (active == 1) return;

  // ---- chunk combine: the last CTA of this (row, kv head) merges in chunk order.
  // The barrier orders every thread's partial stores before thread 0's device-scope
  // fence and ticket (release); the last CTA fences again before reading (acquire).
  __syncthreads();
  unsigned* counter = counters + size_t(b) * kv_heads + h;
  if (threadIdx.x == 0) {
    __threadfence();
    last_flag = (atomicAdd(counter, 1u) == unsigned(active - 1));
    if (last_flag) __threadfence();
  }
  __syncthreads();
  if (!last_flag) return;
  const float* base = partials + (size_t(b) * kv_heads + h) * max_chunks * C::kPart;
  for (int e = threadIdx.x; e < G * D; e += blockDim.x) {
    const int gg = e / D, d = e % D;
    float M = -INFINITY;
    for (int cc = 0; cc < active; ++cc) M = fmaxf(M, __ldcg(base + cc * C::kPart + gg * (D + 2)));
    float L = 0.f, O = 0.f;
    for (int cc = 0; cc < active; ++cc) {
      const float* pc = base + cc * C::kPart + gg * (D + 2);
      const float mc = __ldcg(pc);
      const float f = mc == -INFINITY ? 0.f : exp2f(mc - M);
      L += __ldcg(pc + 1) * f;
      O += __ldcg(pc + 2 + d) * f;
    }
    out[(size_t(b) * kv_heads * G + size_t(h) * G + gg) * D + d] = __float2bfloat16_rn(O / L);
  }
  if (threadIdx.x == 0) *counter = 0u;
}

template <int D, int G, bool FUSED, int STAGES>
int launch_mma_stages(const AttentionCall& a, const FusedQKV& f) {
  using C = MmaCfg<D, G, STAGES>;
  static PerDevice smem_once;
  if (const int rc = smem_limit(smem_once, decode_attention_mma_kernel<D, G, FUSED, STAGES>, C::kSmem, "attention: set smem"))
    return rc;
  const int64_t arena_rows = a.arena_slots * a.kv_heads * a.capacity;
  CUtensorMap tmk, tmv;
  int rc = make_map_bf16(&tmk, a.keys, arena_rows, D, D, 64, C::kTile);
  if (rc) return rc;
  rc = make_map_bf16(&tmv, a.values, arena_rows, D, D, 64, C::kTile);
  if (rc) return rc;
  return launch(decode_attention_mma_kernel<D, G, FUSED, STAGES>, dim3(a.max_chunks, unsigned(a.kv_heads), unsigned(a.rows)),
                dim3(128), size_t(C::kSmem), a.stream, true, "decode_attention_mma", tmk, tmv,
                static_cast<const __nv_bfloat16*>(a.query), a.positions, static_cast<__nv_bfloat16*>(a.out),
                int(a.kv_heads), a.capacity, a.context, int(a.window), int(a.rows_per_slot), a.slots, a.chunk,
                a.plan, a.scale * kLog2e, a.partials, a.counters, a.max_chunks, a.status, f);
}

// Contexts of one key tile (every chunk is one tile) take the one-stage kernel.
template <int D, int G, bool FUSED>
int launch_mma(const AttentionCall& a, const FusedQKV& f) {
  if (a.context <= MmaCfg<D, G>::kTile) return launch_mma_stages<D, G, FUSED, 1>(a, f);
  return launch_mma_stages<D, G, FUSED, 2>(a, f);
}

}  // namespace

namespace q3t {

template <int D, int G, bool FUSED>
int wave_of() {
  static PerDevice once;
  static std::atomic<int> resident[64];
  const int rc = once.run(
      [&](int dev) {
        using C = MmaCfg<D, G>;
        if (cudaFuncSetAttribute(decode_attention_mma_kernel<D, G, FUSED, 2>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
          return check_cuda("attention: set smem");
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_attention_mma_kernel<D, G, FUSED, 2>, 128,
                                                          size_t(C::kSmem)) != cudaSuccess || per_sm < 1)
          per_sm = 1;
        resident[dev].store(per_sm * sm_count(), std::memory_order_relaxed);
        return int(Q3T_OK);
      },
      "attention: wave size");
  int dev = -1;
  if (rc != Q3T_OK || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  return resident[dev].load(std::memory_order_relaxed);
}

int attention_wave_ctas(int64_t head_dim, int64_t group, bool fused) {
  if (head_dim == 128 && group == 2) return fused ? wave_of<128, 2, true>() : wave_of<128, 2, false>();
  if (head_dim == 128 && group == 1) return fused ? wave_of<128, 1, true>() : wave_of<128, 1, false>();
  if (head_dim == 64 && group == 2) return fused ? wave_of<64, 2, true>() : wave_of<64, 2, false>();
  if (head_dim == 64 && group == 1) return fused ? wave_of<64, 1, true>() : wave_of<64, 1, false>();
  return 0;
}

bool attention_mma_supported(int64_t head_dim, int64_t group) {
  return (head_dim == 128 || head_dim == 64) && (group == 1 || group == 2);
}

int launch_attention_mma(const AttentionCall& a) {
  const int64_t g = a.q_heads / a.kv_heads;
  const FusedQKV none = {};
  if (a.head_dim == 128 && g == 2) return launch_mma<128, 2, false>(a, none);
  if (a.head_dim == 128 && g == 1) return launch_mma<128, 1, false>(a, none);
  if (a.head_dim == 64 && g == 2) return launch_mma<64, 2, false>(a, none);
  if (a.head_dim == 64 && g == 1) return launch_mma<64, 1, false>(a, none);
  return fail(Q3T_EUNSUPPORTED, "attention (mma): unsupported head geometry");
}

int launch_attention_fused(const AttentionCall& a, const void* qkv, int64_t qkv_stride, const void* q_norm,
                           const void* k_norm, float eps, const void* cos, const void* sin, int64_t table_len,
                           const int64_t* rot_pos) {
  FusedQKV f;
  f.qkv = static_cast<const __nv_bfloat16*>(qkv);
  f.qkv_stride = qkv_stride;
  f.q_norm = static_cast<const __nv_bfloat16*>(q_norm);
  f.k_norm = static_cast<const __nv_bfloat16*>(k_norm);
  f.eps = eps;
  f.cos = static_cast<const __nv_bfloat16*>(cos);
  f.sin = static_cast<const __nv_bfloat16*>(sin);
  f.table_len = table_len;
  f.rot_pos = rot_pos;
  f.keys = static_cast<__nv_bfloat16*>(const_cast<void*>(a.keys));
  f.values = static_cast<__nv_bfloat16*>(const_cast<void*>(a.values));
  for (int r = 0; r < 2; ++r) {
    f.pf[r] = a.prefetch_bytes[r] ? static_cast<const uint8_t*>(a.prefetch[r]) : nullptr;
    f.pf_bytes[r] = a.prefetch_bytes[r];
  }
  const int64_t g = a.q_heads / a.kv_heads;
  if (a.head_dim == 128 && g == 2) return launch_mma<128, 2, true>(a, f);
  if (a.head_dim == 128 && g == 1) return launch_mma<128, 1, true>(a, f);
  if (a.head_dim == 64 && g == 2) return launch_mma<64, 2, true>(a, f);
  if (a.head_dim == 64 && g == 1) return launch_mma<64, 1, true>(a, f);
  return fail(Q3T_EUNSUPPORTED, "attention (fused): unsupported head geometry");
}

}  // namespace q3t
