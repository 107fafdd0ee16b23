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
// with 128-byte swizzle (conflict-free ldmatrix) into a 3-stage ring; each of
// the 4 warps owns 16 keys of a tile and keeps its own online softmax, and
// the warps, then the chunks of a (row, kv head) (fp32 partials + ticket, chunk
// order), are merged at the end of each work item. The kernel is persistent
// and warp-specialised (two CTAs per SM; a producer warp pulls items from a
// counter and keeps the TMA ring full across items).
#include "attention.cuh"
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

constexpr float kLog2e = 1.4426950408889634f;

template <int D, int G>
struct MmaCfg {
  static constexpr int kTile = 64;                    // keys per tile, 16 per warp
  static constexpr int kBoxes = D / 64;               // 128-byte TMA boxes per key row
  static constexpr int kBoxBytes = kTile * 128;       // 8 KB
  static constexpr int kStageBytes = 2 * kBoxes * kBoxBytes;
  static constexpr int kStages = 3;
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

// One work item = (query row b, kv head h, chunk c of `chunk` keys). Items are
// numbered chunk-major (item = c * pairs + pair) so the chunks that exist for
// every row come first and the ragged tail of short rows comes last.
struct Item {
  int b, h, c, active, ntiles;
  int64_t k_begin, k_end, row0;
};

Q3T_DEV bool decode_item(int item, int pairs, int kv_heads, const int64_t* __restrict__ positions, int64_t context,
                         int window, int rows_per_slot, const int64_t* __restrict__ slots, int64_t capacity, int chunk,
                         int tile, Item& it) {
  it.c = item / pairs;
  const int pair = item - it.c * pairs;
  it.b = pair / kv_heads;
  it.h = pair - it.b * kv_heads;
  int64_t pos = positions[it.b];
  pos = pos < 0 ? 0 : (pos >= context ? context - 1 : pos);
  const int64_t k_lo = (window > 0 && pos + 1 > window) ? pos + 1 - window : 0;
  const int64_t nkeys = pos + 1;
  it.active = int((nkeys - k_lo + chunk - 1) / chunk);
  if (it.c >= it.active) return false;
  it.k_begin = k_lo + int64_t(it.c) * chunk;
  it.k_end = (it.k_begin + chunk) < nkeys ? (it.k_begin + chunk) : nkeys;
  it.ntiles = int((it.k_end - it.k_begin + tile - 1) / tile);
  const int64_t slot = slots != nullptr ? slots[it.b / rows_per_slot] : int64_t(it.b / rows_per_slot);
  it.row0 = (slot * kv_heads + it.h) * capacity + it.k_begin;
  return true;
}


// Persistent, warp-specialised: two CTAs per SM, each with four consumer warps
// (tensor-core math, 16 keys of every 64-key tile per warp) and one producer
// warp whose lane 0 claims work items from a global counter and streams their
// K/V tiles through a kStages-deep TMA ring, running ahead across item
// boundaries. The producer never waits for the consumers except for a free
// ring slot (empty barrier, one arrival per consumer warp), so item claims and
// tile decoding stay off the math path; each stage carries its (item, tile)
// tag, and an item id of -1 ends the stream.
template <int D, int G>
__global__ void __launch_bounds__(160, 2)
    decode_attention_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                                const __nv_bfloat16* __restrict__ query, const int64_t* __restrict__ positions,
                                __nv_bfloat16* __restrict__ out, int kv_heads, int64_t capacity, int64_t context,
                                int window, int rows_per_slot, const int64_t* __restrict__ slots, int chunk,
                                float qscale, float* __restrict__ partials, unsigned* __restrict__ counters,
                                int max_chunks, int total_items, unsigned* __restrict__ work, unsigned* status) {
  using C = MmaCfg<D, G>;
  constexpr int S = C::kStages;
  constexpr int KS = D / 16;  // k-steps of S = Q K^T
  constexpr int NT = D / 8;   // n-tiles of O = P V
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[S];
  __shared__ __align__(8) uint64_t empty[S];
  __shared__ int tile_item[S], tile_idx[S];
  __shared__ __align__(16) __nv_bfloat16 qbuf[S][G * D];  // query rows, loaded with an item's first tile
  __shared__ float wm[4][G], wl[4][G];
  __shared__ float wo[4][G][D];
  __shared__ __align__(8) uint64_t rv[4];  // consumer rendezvous: merged, fenced, ticket, released
  __shared__ int aborted, last_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pairs = total_items / max_chunks;
  grid_dependency_wait();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&rv[i], 4);
    fence_mbar_init();
    prefetch_tmap(&tmk);
    prefetch_tmap(&tmv);
    aborted = 0;
  }
  __syncthreads();
  auto stage_k = [&](int s) { return smem + s * C::kStageBytes; };
  auto stage_v = [&](int s) { return smem + s * C::kStageBytes + C::kBoxes * C::kBoxBytes; };

  if (warp == 4) {
    // ================= producer (one lane)
    if (lane == 0) {
      int64_t issued = 0;
      bool stop = false;
      const uint64_t pol = policy_evict_first();
      while (!stop) {
        Item it;
        int item = -1;
        for (;;) {
          const int claim = int(atomicAdd(work, 1u));
          if (claim >= total_items) break;
          if (claim < pairs) {  // chunk 0 of every (row, head): check the position once
            const int64_t p = positions[(claim % pairs) / kv_heads];
            if (p < 0 || p >= context) raise_status(status, kStatusBadIndex);
          }
          if (decode_item(claim, pairs, kv_heads, positions, context, window, rows_per_slot, slots, capacity, chunk,
                          C::kTile, it)) {
            item = claim;
            break;
          }
        }
        const int tiles = item >= 0 ? it.ntiles : 1;  // the end mark takes one stage
        for (int tile = 0; tile < tiles; ++tile) {
          const int s = int(issued % S);
          if (issued >= S && !mbar_wait(&empty[s], uint32_t(((issued / S) - 1) & 1), status, kStatusFlagTimeout)) {
            stop = true;
            break;
          }
          if (*static_cast<volatile int*>(&aborted)) {
            stop = true;
            break;
          }
          tile_item[s] = item;
          tile_idx[s] = tile;
          if (item >= 0) {
            mbar_expect_tx(&full[s], C::kStageBytes + (tile == 0 ? C::kQBytes : 0));
            if (tile == 0)
              bulk_load(qbuf[s], query + (int64_t(it.b) * kv_heads + it.h) * G * D, uint32_t(C::kQBytes), &full[s]);
            const int y = int(it.row0 + int64_t(tile) * C::kTile);
#pragma unroll
            for (int bx = 0; bx < C::kBoxes; ++bx) {
              tma_load_2d(stage_k(s) + bx * C::kBoxBytes, &tmk, &full[s], bx * 64, y, pol);
              tma_load_2d(stage_v(s) + bx * C::kBoxBytes, &tmv, &full[s], bx * 64, y, pol);
            }
          } else {
            mbar_arrive(&full[s]);
          }
          ++issued;
        }
        if (item < 0) stop = true;
      }
      // Copies still in flight must land before the CTA exits (bounded waits; on the
      // normal path every issued tile has been consumed and these return at once).
      for (int64_t j = issued > S ? issued - S : 0; j < issued; ++j)
        mbar_wait(&full[j % S], uint32_t((j / S) & 1), status, kStatusTmaTimeout);
    }
  } else {
    // ================= consumers (warps 0..3)
    const int g = lane >> 2, t4 = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    Item it{};
    int ends = 0, combines = 0;  // item ends and chunk merges this CTA has passed (rendezvous phases)
    // Bounded rendezvous of the four consumer warps (an mbarrier of count 4 per
    // point); a timeout marks the CTA aborted and returns false.
    auto rendezvous = [&](uint64_t* bar, int n) -> bool {
      __syncwarp();
      if (lane == 0) mbar_arrive(bar);
      if (mbar_wait(bar, uint32_t(n & 1), status, kStatusFlagTimeout)) return true;
      aborted = 1;
      return false;
    };
    uint32_t qa[KS][2];
    float o[NT][4];
    float m_run = -INFINITY, l_run = 0.f;
    for (int64_t t = 0;; ++t) {
      const int s = int(t % S);
      const uint32_t phase = uint32_t((t / S) & 1);
      // Each warp waits for the stage itself (bounded). A timeout marks the CTA
      // aborted and the warp leaves at once; the other consumer warps meet it only
      // at bounded rendezvous, so they leave too, and the producer stops issuing.
      if (!mbar_wait(&full[s], phase, status, kStatusTmaTimeout)) {
        aborted = 1;
        break;
      }
      const int item = tile_item[s], tile = tile_idx[s];
      if (item < 0) break;
      if (tile == 0) {
        decode_item(item, pairs, kv_heads, positions, context, window, rows_per_slot, slots, capacity, chunk,
                    C::kTile, it);
        const bool real = g < G;
        const __nv_bfloat16* qp = qbuf[s] + (real ? g : 0) * D;
#pragma unroll
        for (int kk = 0; kk < KS; ++kk) {
          qa[kk][0] = real ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * t4) : 0u;
          qa[kk][1] = real ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 8 + 2 * t4) : 0u;
        }
#pragma unroll
        for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        m_run = -INFINITY;
        l_run = 0.f;
      }
      const uint32_t kbase = smem_u32(stage_k(s)), vbase = smem_u32(stage_v(s));
      const int64_t key0 = it.k_begin + int64_t(tile) * C::kTile + 16 * warp;  // this warp's first key
      const int valid = int((it.k_end - key0) < 0 ? 0 : ((it.k_end - key0) > 16 ? 16 : (it.k_end - key0)));

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
      const float m_new = fmaxf(m_run, mt);
      const float alpha = m_new == -INFINITY ? 1.f : exp2f(m_run - m_new);
      float p[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) p[e] = sv[e] == -INFINITY ? 0.f : exp2f(sv[e] - m_new);
      float ps = (p[0] + p[1]) + (p[2] + p[3]);
      ps += __shfl_xor_sync(0xffffffffu, ps, 1);
      ps += __shfl_xor_sync(0xffffffffu, ps, 2);
      l_run = l_run * alpha + ps;
      m_run = m_new;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        o[n][0] *= alpha;
        o[n][1] *= alpha;
      }
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
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // this warp is done with stage s
      if (tile != it.ntiles - 1) continue;

      // ---- item end: merge the four warps (rows g < G live in lanes 0 .. 4G-1)
      const int b = it.b, h = it.h;
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
      if (!rendezvous(&rv[0], ends)) break;
      float* part = partials + ((size_t(b) * kv_heads + h) * max_chunks + it.c) * C::kPart;
      for (int e = threadIdx.x; e < G * D; e += 128) {
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
        if (it.active == 1) {
          out[(size_t(b) * kv_heads * G + size_t(h) * G + gg) * D + d] = __float2bfloat16_rn(O / L);
        } else {
          part[gg * (D + 2) + 2 + d] = O;
          if (d == 0) {
            part[gg * (D + 2)] = M;
            part[gg * (D + 2) + 1] = L;
          }
        }
      }
      if (it.active > 1) {
        // chunk combine: the last item of this (row, kv head) merges all chunks in chunk order
        __threadfence();
        if (!rendezvous(&rv[1], combines)) break;
        unsigned* counter = counters + size_t(b) * kv_heads + h;
        if (threadIdx.x == 0) last_flag = (atomicAdd(counter, 1u) == unsigned(it.active - 1));
        if (!rendezvous(&rv[2], combines)) break;
        ++combines;
        if (last_flag) {
          __threadfence();
          const float* base = partials + (size_t(b) * kv_heads + h) * max_chunks * C::kPart;
          for (int e = threadIdx.x; e < G * D; e += 128) {
            const int gg = e / D, d = e % D;
            float M = -INFINITY;
            for (int cc = 0; cc < it.active; ++cc) M = fmaxf(M, __ldcg(base + cc * C::kPart + gg * (D + 2)));
            float L = 0.f, O = 0.f;
            for (int cc = 0; cc < it.active; ++cc) {
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
      }
      if (!rendezvous(&rv[3], ends)) break;  // wm/wo/last_flag are free for the next item
      ++ends;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // The last CTA out resets the work and exit counters for the next call.
    __threadfence();
    if (atomicAdd(work + 1, 1u) == gridDim.x - 1) {
      work[0] = 0u;
      work[1] = 0u;
    }
  }
}

template <int D, int G>
int launch_mma(const AttentionCall& a) {
  using C = MmaCfg<D, G>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(decode_attention_mma_kernel<D, G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             C::kSmem) != cudaSuccess)
      return check_cuda("attention: set smem");
    configured[dev] = true;
  }
  const int64_t arena_rows = a.arena_slots * a.kv_heads * a.capacity;
  CUtensorMap tmk, tmv;
  int rc = make_map_bf16(&tmk, a.keys, arena_rows, D, D, 64, C::kTile);
  if (rc) return rc;
  rc = make_map_bf16(&tmv, a.values, arena_rows, D, D, 64, C::kTile);
  if (rc) return rc;
  const int64_t total = a.rows * a.kv_heads * a.max_chunks;
  if (total > (int64_t(1) << 30)) return fail(Q3T_EUNSUPPORTED, "attention: too many work items");
  const int64_t resident = 2LL * sm_count();
  const unsigned grid = unsigned(total < resident ? total : resident);
  return launch(decode_attention_mma_kernel<D, G>, dim3(grid), dim3(160), size_t(C::kSmem), a.stream, true,
                "decode_attention_mma", tmk, tmv, static_cast<const __nv_bfloat16*>(a.query), a.positions,
                static_cast<__nv_bfloat16*>(a.out), int(a.kv_heads), a.capacity, a.context, int(a.window),
                int(a.rows_per_slot), a.slots, a.chunk, a.scale * kLog2e, a.partials, a.counters, a.max_chunks,
                int(total), a.work, a.status);
}

}  // namespace

namespace q3t {

bool attention_mma_supported(int64_t head_dim, int64_t group) {
  return (head_dim == 128 || head_dim == 64) && (group == 1 || group == 2);
}

int launch_attention_mma(const AttentionCall& a) {
  const int64_t g = a.q_heads / a.kv_heads;
  if (a.head_dim == 128 && g == 2) return launch_mma<128, 2>(a);
  if (a.head_dim == 128 && g == 1) return launch_mma<128, 1>(a);
  if (a.head_dim == 64 && g == 2) return launch_mma<64, 2>(a);
  if (a.head_dim == 64 && g == 1) return launch_mma<64, 1>(a);
  return fail(Q3T_EUNSUPPORTED, "attention (mma): unsupported head geometry");
}

}  // namespace q3t
