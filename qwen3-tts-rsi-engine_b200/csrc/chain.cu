// Persistent chains of dependent projections (tcgen05 + TMEM), one launch per chain.
//
// A decode layer's projections after its attention - O (+ residual), gate/up (folded
// RMSNorm, SwiGLU), down (+ residual), then the next layer's QKV (folded RMSNorm) - are
// weight-streaming GEMMs with 16-64 activation rows. Launched one by one, each pays a
// fixed pipeline latency (prologue, activation load after the dependency wait, cluster
// reduction, grid drain) that at these sizes is as long as its weight stream. Here one
// persistent grid (one CTA per SM) runs the whole chain: the weights never depend on
// anything, so every CTA streams its share of ALL the chain's weight tiles through one
// shared-memory ring without a break, and only the activation tiles of a stage wait for
// the previous stage to be complete.
//
// Work split ("stream-K"): stage s has U = n_tiles x kblocks units (128 weight rows x 64
// inputs each, one 16 KB pre-swizzled tile); CTA c takes units [c U / G, (c+1) U / G),
// so every CTA streams the same number of weight bytes per stage. A CTA's range cuts
// across tiles: each (CTA, tile) piece is a segment, accumulated in TMEM (two
// accumulators, so the MMA runs ahead of the epilogue) and written as fp32 partials to
// a global scratch slot. Once every contributor of a tile has written its piece (per-tile
// counter), contributor j of the tile's nc reduces rows [j R / nc, (j+1) R / nc) over the
// partials in contributor order (deterministic), applies the epilogue and stores the
// output. A stage is complete when every slice is stored (per-stage counter); the
// producer of every CTA waits for that count before loading the next stage's activation
// tiles. Counters are zeroed by the last CTA to leave, so each launch starts from zero.
//
// Roles (256 threads): warp 0 lane 0 = TMA producer (weights ahead as far as the ring
// allows, activations when their stage's input is complete); warp 1 = TMEM owner, lane 0
// = MMA issuer; warps 2-3 = row sums of squares of the activation tiles (folded RMSNorm);
// warps 4-7 = epilogue (TMEM lanes = the tile's 128 weight rows). Every wait is bounded.
#include "common.cuh"
#include "host.cuh"

#include <string.h>

using namespace q3t;

namespace {

constexpr int kTileN = 128;   // weight rows per tile (UMMA M)
constexpr int kTileK = 64;    // inputs per k-block (one 128-byte swizzled row)
constexpr int kABytes = kTileN * kTileK * 2;
constexpr int kThreads = 256;
constexpr int kMaxStages = Q3T_CHAIN_MAX_STAGES;
// sync block layout (unsigned words)
constexpr int kSyncExit = 0, kSyncAbort = 1, kSyncStage = 4, kSyncTiles = 16;
constexpr int kSyncWords = 2048;  // room for kSyncTiles + every stage's tile counters
constexpr int kMaxPieces = 4;     // tiles one CTA may touch in one stage (scratch slots per CTA)
// A stage runs on at most units / kMinUnits CTAs, so that no tile is cut into more than about
// kblocks / kMinUnits + 1 pieces: the reduction of a tile reads every piece, so a stage of few
// weight tiles is better served by fewer, longer pieces than by every SM.
constexpr int kMinUnits = 4;
constexpr int kMaxGrid = 256;     // contributor slots of one tile (shared memory)
// Weight tiles the producer pulls into L2 ahead of the ring: the HBM stream keeps going while a
// stage waits for its input (16 x 16 KB per CTA, ~38 MB in flight over 148 SMs).
constexpr int kPrefetchAhead = 16;

template <int BN>
struct ChainCfg {
  static constexpr int kBBytes = BN * kTileK * 2;
  static constexpr int kSlotBytes = kABytes + kBBytes;   // a multiple of 1024 (swizzle atoms)
  static constexpr int kSlots = (200 * 1024) / kSlotBytes;
  static constexpr int kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  // ring, then 512 bytes of barriers and flags, the contributor slots of the tile being reduced,
  // and 1 KB of alignment slack
  static constexpr int kSmem = kSlots * kSlotBytes + 512 + kMaxGrid * 4 + 1024;
};

struct Stage {
  const uint8_t* tiles;               // [n_tiles][kblocks] 16 KB swizzled weight tiles
  void* out;
  const __nv_bfloat16* residual;      // may alias out (elementwise in place)
  const __nv_bfloat16* bias;
  int64_t out_stride, res_stride;
  int in_features, out_features, kblocks, n_tiles, units;
  int epilogue, out_f32, row_norm;
  float norm_eps;
  int segments;                       // (CTA, tile) pieces: stored slices per launch
  int ctas;                           // CTAs [0, ctas) split this stage's units
  int tile_base;                      // first tile counter of this stage in the sync block
  int depends;                        // stage whose completion gates this stage's activations (-1: none)
};

struct ChainParams {
  CUtensorMap x[kMaxStages];          // activation operand of each stage: {in_features, rows}, box {64, BN}
  Stage st[kMaxStages];
  int stages, rows, counters;         // counters: words of the sync block zeroed at exit
  int pieces;                         // scratch slots per CTA: the most tiles one CTA touches in a stage
  unsigned* sync;
  float* partials;                    // [grid * pieces][BN][128]
  float* sumsq;                       // [grid * pieces][BN]
  unsigned* status;
};

Q3T_DEV int range_start(int c, int units, int grid) { return int((int64_t(c) * units) / grid); }
// CTA whose unit range holds unit u (ranges are non-empty: units >= grid)
Q3T_DEV int owner_of(int u, int units, int grid) { return int(((int64_t(u) + 1) * grid - 1) / units); }
// scratch slot of CTA c's piece of tile t: CTA c owns slots [c * pieces, (c + 1) * pieces),
// one per tile its unit range touches, in tile order
Q3T_DEV int piece_slot(const Stage& s, int c, int t, int grid, int pieces) {
  return c * pieces + (t - range_start(c, s.units, grid) / s.kblocks);
}

Q3T_DEV unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
Q3T_DEV unsigned ld_volatile(const unsigned* p) {
  unsigned v;
  asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Non-blocking phase test (the producer polls two conditions and must not be suspended on one).
Q3T_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
Q3T_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
Q3T_DEV void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Bounded wait until *p >= target (both counted from zero in this launch). On timeout or
// when another CTA aborted, raises the abort flag / status and returns false.
Q3T_DEV bool wait_count(const unsigned* p, unsigned target, unsigned* sync, unsigned* status) {
  if (ld_acquire(p) >= target) return true;
  const uint64_t start = global_ns();
  for (int spin = 0;; ++spin) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i) {
      if (ld_acquire(p) >= target) return true;
      if (spin >= 64) __nanosleep(64);   // tight polling first: the wait is normally short
    }
    if (ld_volatile(sync + kSyncAbort)) return false;
    if (global_ns() - start > kWaitLimitNs) {
      atomicExch(sync + kSyncAbort, 1u);
      raise_status(status, kStatusFlagTimeout);
      return false;
    }
  }
}

// The CTA's sequence of k-blocks over all stages: stage s, tile t, k-block kb; `i` counts items.
struct Items {
  const ChainParams* p;
  int c, grid, i, s, t, kb, kb_end, t_last, u0, u1;
  bool done;
  Q3T_DEV void start(const ChainParams* params, int cta, int g) {
    p = params;
    c = cta;
    grid = g;
    i = 0;
    s = -1;
    done = false;
    next_stage();
  }
  Q3T_DEV void next_stage() {
    do {   // skip the stages this CTA takes no part in
      if (++s >= p->stages) {
        done = true;
        return;
      }
    } while (c >= p->st[s].ctas);
    const Stage& st = p->st[s];
    u0 = range_start(c, st.units, st.ctas);
    u1 = range_start(c + 1, st.units, st.ctas);
    t = u0 / st.kblocks;
    t_last = (u1 - 1) / st.kblocks;
    set_tile();
  }
  Q3T_DEV void set_tile() {
    const int K = p->st[s].kblocks;
    kb = (u0 > t * K ? u0 : t * K) - t * K;
    kb_end = (u1 < (t + 1) * K ? u1 : (t + 1) * K) - t * K;
  }
  // true when the item just left was the last of its segment
  Q3T_DEV bool advance() {
    ++i;
    if (++kb < kb_end) return false;
    if (++t <= t_last) {
      set_tile();
    } else {
      next_stage();
    }
    return true;
  }
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const __grid_constant__ ChainParams a) {
  using C = ChainCfg<BN>;
  constexpr int S = C::kSlots;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_a = reinterpret_cast<uint64_t*>(smem + S * C::kSlotBytes);
  uint64_t* full_b = full_a + S;
  uint64_t* empty = full_b + S;
  uint64_t* tmem_full = empty + S;     // [2]
  uint64_t* tmem_empty = tmem_full + 2;  // [2]
  uint64_t* mma_done = tmem_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* rs_done = reinterpret_cast<volatile int*>(tmem_slot + 1);   // row-sum pieces written (x2 warps)
  volatile int* consumed = rs_done + 1;                                      // items the MMA has taken
  volatile int* issued_a = consumed + 1;
  volatile int* issued_b = issued_a + 1;
  volatile int* last_flag = issued_b + 1;
  int* tile_slots = reinterpret_cast<int*>(smem + S * C::kSlotBytes + 512);   // [kMaxGrid]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x, grid = gridDim.x;
  unsigned* sync = a.sync;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full_a[s], 1);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 3);   // the MMA commit and the two row-sum warps
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tmem_full[b], 1);
      mbar_init(&tmem_empty[b], 1);
    }
    mbar_init(mma_done, 1);
    *rs_done = 0;
    *consumed = 0;
    *issued_a = 0;
    *issued_b = 0;
    *last_flag = 0;
    fence_mbar_init();
    for (int s = 0; s < a.stages; ++s) prefetch_tmap(&a.x[s]);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer: weights as far ahead as the ring allows (the first S before the
      // dependency wait), activations once their stage's input is complete
      const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
      Items A, B, P;
      A.start(&a, c, grid);
      B.start(&a, c, grid);
      P.start(&a, c, grid);
      auto tile_of = [&](const Items& it) {
        const Stage& st = a.st[it.s];
        return st.tiles + (size_t(it.t) * size_t(st.kblocks) + size_t(it.kb)) * size_t(kABytes);
      };
      auto prefetch_ahead = [&]() {   // L2 prefetch of the weight tiles after the ring's
        bool any = false;
        while (!P.done && P.i < A.i + S + kPrefetchAhead) {
          if (P.i >= A.i + S) prefetch_l2(tile_of(P), uint32_t(kABytes));
          P.advance();
          any = true;
        }
        return any;
      };
      auto issue_a = [&]() {
        const int slot = A.i % S;
        const Stage& st = a.st[A.s];
        (void)st;
        mbar_expect_tx(&full_a[slot], uint32_t(kABytes));
        bulk_load_hint(smem + slot * C::kSlotBytes, tile_of(A), uint32_t(kABytes), &full_a[slot], pol_w);
        A.advance();
        *issued_a = A.i;
      };
      while (!A.done && A.i < S) issue_a();
      prefetch_ahead();
      grid_dependency_wait();
      int ready_stage = 0;   // stages [0, ready_stage) may load activations
      bool ok = true;
      uint64_t idle_since = 0;
      while (ok && !B.done) {
        bool progress = false;
        if (!A.done && A.i < B.i + S) {
          const int slot = A.i % S;
          if (mbar_test_wait(&empty[slot], ((A.i / S) & 1) ^ 1)) {
            issue_a();
            progress = true;
          }
        }
        if (B.i < A.i) {
          if (B.s >= ready_stage) {
            const int dep = a.st[B.s].depends;
            if (dep < 0 || ld_acquire(sync + kSyncStage + dep) >= unsigned(a.st[dep].segments)) {
              fence_proxy_async_global();   // generic-proxy stores of other CTAs, then async-proxy loads
              ready_stage = B.s + 1;
            }
          }
          if (B.s < ready_stage) {
            const int slot = B.i % S;
            mbar_expect_tx(&full_b[slot], uint32_t(C::kBBytes));
            tma_load_2d(smem + slot * C::kSlotBytes + kABytes, &a.x[B.s], &full_b[slot], B.kb * kTileK, 0, pol_x);
            B.advance();
            *issued_b = B.i;
            progress = true;
          }
        }
        if (prefetch_ahead()) progress = true;
        if (progress) {
          idle_since = 0;
        } else {
          const uint64_t now = global_ns();
          if (idle_since == 0) idle_since = now;
          if (ld_volatile(sync + kSyncAbort)) ok = false;
          if (now - idle_since > kWaitLimitNs) {
            atomicExch(sync + kSyncAbort, 1u);
            raise_status(a.status, kStatusFlagTimeout);
            ok = false;
          }
          __nanosleep(32);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    grid_dependency_wait();
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16(kTileN, BN);
      Items it;
      it.start(&a, c, grid);
      int seg = 0;
      bool ok = true, first = true;
      while (ok && !it.done) {
        const int buf = seg & 1;
        if (first) {
          if (seg >= 2 && !mbar_wait(&tmem_empty[buf], ((seg >> 1) & 1) ^ 1, a.status, kStatusMmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        const int slot = it.i % S;
        const uint32_t parity = (it.i / S) & 1;
        if (!mbar_wait(&full_a[slot], parity, a.status, kStatusTmaTimeout) ||
            !mbar_wait(&full_b[slot], parity, a.status, kStatusTmaTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128(smem_u32(smem + slot * C::kSlotBytes));
        const uint64_t bd = umma_desc_sw128(smem_u32(smem + slot * C::kSlotBytes + kABytes));
        const uint32_t d = tmem + uint32_t(buf * BN);
#pragma unroll
        for (int k = 0; k < kTileK / 16; ++k) umma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (!first || k > 0) ? 1u : 0u);
        umma_commit(&empty[slot]);
        first = it.advance();
        *consumed = it.i;
        if (first) {
          umma_commit(&tmem_full[buf]);
          ++seg;
        }
      }
      if (!ok) atomicExch(sync + kSyncAbort, 1u);
      umma_commit(mma_done);   // every MMA issued so far has finished when this arrives
    }
    __syncwarp();
  } else if (warp == 2 || warp == 3) {
    // ---------------- row sums of squares of the activation tiles (folded RMSNorm), per piece
    grid_dependency_wait();
    const int m = threadIdx.x - 64;   // activation row (BN <= 64)
    Items it;
    it.start(&a, c, grid);
    float ss = 0.f;
    bool ok = true;
    while (ok && !it.done) {
      const int slot = it.i % S;
      const Stage& st = a.st[it.s];
      const int s_now = it.s, t_now = it.t;
      if (!mbar_wait(&full_b[slot], (it.i / S) & 1, a.status, kStatusTmaTimeout)) {
        ok = false;
        break;
      }
      if (st.row_norm && m < BN) {
        const uint4* row = reinterpret_cast<const uint4*>(smem + slot * C::kSlotBytes + kABytes + m * 128);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 v = row[q];
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = __uint_as_float(w4[e] << 16), hi = __uint_as_float(w4[e] & 0xFFFF0000u);
            ss += lo * lo + hi * hi;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (it.advance()) {   // piece complete: its row sums go to the piece's scratch slot
        if (st.row_norm && m < BN)
          __stcg(a.sumsq + size_t(piece_slot(st, c, t_now, st.ctas, a.pieces)) * BN + m, ss);
        (void)s_now;
        ss = 0.f;
        __threadfence();
        __syncwarp();
        if (lane == 0) atomicAdd(const_cast<int*>(rs_done), 1);
      }
    }
    if (!ok) atomicExch(sync + kSyncAbort, 1u);
  } else {
    // ---------------- epilogue: warps 4-7, thread r = TMEM lane = weight row of the tile
    grid_dependency_wait();
    const int r = threadIdx.x - 128;
    const int quad = warp & 3;
    const bool leader = threadIdx.x == 128;
    const int R = a.rows;
    int seg = 0;
    bool ok = true;
    for (int s = 0; s < a.stages && ok; ++s) {
      const Stage& st = a.st[s];
      if (c >= st.ctas) continue;
      const int K = st.kblocks, G = st.ctas;
      const int u0 = range_start(c, st.units, G), u1 = range_start(c + 1, st.units, G);
      const int t0 = u0 / K, t1 = (u1 - 1) / K;
      // (1) drain every piece of this stage into its scratch slot and count it at its tile
      for (int t = t0; t <= t1 && ok; ++t, ++seg) {
        const int buf = seg & 1;
        if (!mbar_wait(&tmem_full[buf], (seg >> 1) & 1, a.status, kStatusMmaTimeout)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float* part = a.partials + size_t(piece_slot(st, c, t, G, a.pieces)) * BN * kTileN;
        const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16) + uint32_t(buf * BN);
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
          tmem_ld16(taddr + c0, v);
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < R) __stcg(part + (c0 + j) * kTileN + r, v[j]);
        }
        tc_fence_before();
        epilogue_sync();
        if (leader) {
          mbar_arrive(&tmem_empty[buf]);
          // the row-sum warps have written this piece's sums (two arrivals per piece)
          const uint64_t begin = global_ns();
          while (*rs_done < 2 * (seg + 1)) {
            if (global_ns() - begin > kWaitLimitNs) {
              raise_status(a.status, kStatusFlagTimeout);
              atomicExch(sync + kSyncAbort, 1u);
              break;
            }
          }
          __threadfence();
          atomicAdd(sync + kSyncTiles + st.tile_base + t, 1u);
        }
      }
      if (!ok) break;
      // (2) reduce this CTA's row slice of every tile it touched, once all its pieces are in
      for (int t = t0; t <= t1 && ok; ++t) {
        const int c_lo = owner_of(t * K, st.units, G), c_hi = owner_of((t + 1) * K - 1, st.units, G);
        const int nc = c_hi - c_lo + 1, j = c - c_lo;
        for (int k = r; k < nc; k += kTileN) tile_slots[k] = piece_slot(st, c_lo + k, t, G, a.pieces);
        if (leader && !wait_count(sync + kSyncTiles + st.tile_base + t, unsigned(nc), sync, a.status))
          atomicExch(sync + kSyncAbort, 1u);
        epilogue_sync();   // the tile's pieces are in; tile_slots is visible to every thread
        if (ld_volatile(sync + kSyncAbort)) {
          ok = false;
          break;
        }
        const int m0 = int((int64_t(j) * R) / nc), m1 = int((int64_t(j + 1) * R) / nc);
        const int n0 = t * kTileN;
        // Every piece of the tile is summed in contributor order (deterministic). A thread owns
        // four consecutive features (one float4 of each partial row) and a fixed set of rows; the
        // loads of up to eight contributors x its rows are issued together, so a slice costs about
        // one L2 round trip.
        if (st.epilogue == Q3T_EPI_SWIGLU_PAIRED) {
          // tile rows are [64 gate; 64 up] of features n0/2 .. n0/2 + 63: thread = 4 gate features
          // (f4) x every 8th row of the slice
          const int f4 = r & 15, sub = r >> 4;
          for (int mb = m0 + sub; mb < m1; mb += 16) {
            float4 g[2], u[2];
            float ssum[2] = {0.f, 0.f};
#pragma unroll
            for (int q = 0; q < 2; ++q) g[q] = u[q] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k0 = 0; k0 < nc; k0 += 8) {
              float4 gv[8][2], uv[8][2];
              float sv[8][2];
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const bool kin = k0 + kk < nc;
                const int slot = kin ? tile_slots[k0 + kk] : 0;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  const int m = mb + 8 * q;
                  const bool in = kin && m < m1;
                  const float4* pp = reinterpret_cast<const float4*>(a.partials + (size_t(slot) * BN + (in ? m : 0)) * kTileN);
                  gv[kk][q] = in ? __ldcg(pp + f4) : make_float4(0.f, 0.f, 0.f, 0.f);
                  uv[kk][q] = in ? __ldcg(pp + 16 + f4) : make_float4(0.f, 0.f, 0.f, 0.f);
                  sv[kk][q] = in && st.row_norm ? __ldcg(a.sumsq + size_t(slot) * BN + m) : 0.f;
                }
              }
#pragma unroll
              for (int kk = 0; kk < 8; ++kk)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  g[q].x += gv[kk][q].x; g[q].y += gv[kk][q].y; g[q].z += gv[kk][q].z; g[q].w += gv[kk][q].w;
                  u[q].x += uv[kk][q].x; u[q].y += uv[kk][q].y; u[q].z += uv[kk][q].z; u[q].w += uv[kk][q].w;
                  ssum[q] += sv[kk][q];
                }
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int m = mb + 8 * q;
              if (m >= m1) continue;
              const float rs = st.row_norm ? 1.0f / sqrtf(ssum[q] / float(st.in_features) + st.norm_eps) : 1.f;
              const float gs[4] = {g[q].x, g[q].y, g[q].z, g[q].w}, us[4] = {u[q].x, u[q].y, u[q].z, u[q].w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int f = 4 * f4 + e;
                if (n0 + 64 + f >= st.out_features) continue;
                const float gr = bf16r(st.row_norm ? gs[e] * rs : gs[e]), ur = bf16r(st.row_norm ? us[e] * rs : us[e]);
                const float v = bf16r(bf16r(gr / (1.0f + expf(-gr))) * ur);
                static_cast<__nv_bfloat16*>(st.out)[int64_t(m) * st.out_stride + n0 / 2 + f] = __float2bfloat16_rn(v);
              }
            }
          }
        } else {
          // thread = 4 features (n4) x every 4th row of the slice
          const int n4 = r & 31, sub = r >> 5;
          const int nb = n0 + 4 * n4;
          float bias[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            bias[e] = (nb + e < st.out_features && st.bias != nullptr) ? __bfloat162float(st.bias[nb + e]) : 0.f;
          for (int mb = m0 + sub; mb < m1; mb += 8) {
            float4 acc[2];
            float ssum[2] = {0.f, 0.f};
            acc[0] = acc[1] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int k0 = 0; k0 < nc; k0 += 8) {
              float4 v[8][2];
              float sv[8][2];
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const bool kin = k0 + kk < nc;
                const int slot = kin ? tile_slots[k0 + kk] : 0;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  const int m = mb + 4 * q;
                  const bool in = kin && m < m1;
                  v[kk][q] = in ? __ldcg(reinterpret_cast<const float4*>(a.partials + (size_t(slot) * BN + m) * kTileN) + n4)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
                  sv[kk][q] = in && st.row_norm ? __ldcg(a.sumsq + size_t(slot) * BN + m) : 0.f;
                }
              }
#pragma unroll
              for (int kk = 0; kk < 8; ++kk)
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                  acc[q].x += v[kk][q].x; acc[q].y += v[kk][q].y; acc[q].z += v[kk][q].z; acc[q].w += v[kk][q].w;
                  ssum[q] += sv[kk][q];
                }
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int m = mb + 4 * q;
              if (m >= m1) continue;
              const float rs = st.row_norm ? 1.0f / sqrtf(ssum[q] / float(st.in_features) + st.norm_eps) : 1.f;
              const float vals[4] = {acc[q].x, acc[q].y, acc[q].z, acc[q].w};
              float res[4];
#pragma unroll
              for (int e = 0; e < 4; ++e)
                res[e] = (st.epilogue == Q3T_EPI_RESIDUAL && nb + e < st.out_features)
                             ? __bfloat162float(__ldcg(st.residual + int64_t(m) * st.res_stride + nb + e))
                             : 0.f;
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int n = nb + e;
                if (n >= st.out_features) continue;
                float val = st.row_norm ? vals[e] * rs : vals[e];
                val += bias[e];
                if (st.epilogue == Q3T_EPI_RESIDUAL) {
                  static_cast<__nv_bfloat16*>(st.out)[int64_t(m) * st.out_stride + n] =
                      __float2bfloat16_rn(res[e] + bf16r(val));
                } else if (st.out_f32) {
                  static_cast<float*>(st.out)[int64_t(m) * st.out_stride + n] = bf16r(val);
                } else {
                  static_cast<__nv_bfloat16*>(st.out)[int64_t(m) * st.out_stride + n] = __float2bfloat16_rn(val);
                }
              }
            }
          }
        }
        epilogue_sync();   // every output of the slice is stored (and tile_slots may be rewritten)
        if (leader) {
          __threadfence();
          atomicAdd(sync + kSyncStage + s, 1u);
        }
      }
    }
    if (!ok && leader) atomicExch(sync + kSyncAbort, 1u);
  }

  // ---------------- teardown: every MMA finished, every load landed, TMEM released; the last
  // CTA out zeroes the counters for the next launch
  __syncthreads();
  if (threadIdx.x == 32) mbar_wait(mma_done, 0, a.status, kStatusMmaTimeout);
  if (threadIdx.x == 0) {
    // loads issued but never consumed (an aborted launch) land before the ring goes away
    for (int j = *consumed; j < *issued_a; ++j) mbar_wait(&full_a[j % S], (j / S) & 1, a.status, kStatusTmaTimeout);
    for (int j = *consumed; j < *issued_b; ++j) mbar_wait(&full_b[j % S], (j / S) & 1, a.status, kStatusTmaTimeout);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
  if (threadIdx.x == 0) {
    __threadfence();
    *last_flag = atomicAdd(sync + kSyncExit, 1u) == unsigned(grid - 1) ? 1 : 0;
  }
  __syncthreads();
  if (*last_flag) {
    __threadfence();
    for (int w = threadIdx.x; w < a.counters; w += blockDim.x)
      if (w >= kSyncStage && w != kSyncAbort) sync[w] = 0u;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sync[kSyncExit] = 0u;
  }
}

// ---------------------------------------------------------------- host side
int rows_tile(int64_t rows) { return rows <= 16 ? 16 : rows <= 32 ? 32 : 64; }

template <int BN>
int launch_chain(const ChainParams& p, int grid, void* stream) {
  using C = ChainCfg<BN>;
  static PerDevice smem_once;
  if (const int rc = smem_limit(smem_once, chain_kernel<BN>, C::kSmem, "linear_chain: set smem")) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = size_t(C::kSmem);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, chain_kernel<BN>, p);
  if (err != cudaSuccess) return fail(Q3T_ECUDA, "linear_chain launch failed: %s", cudaGetErrorString(err));
  note_launch();
  return Q3T_OK;
}

// scratch: the counter block, then kMaxPieces partial tiles [BN][128] and row sums [BN] per CTA
size_t scratch_bytes(int bn, int grid) {
  return size_t(kSyncWords) * 4 + size_t(grid) * kMaxPieces * size_t(bn) * (kTileN + 1) * sizeof(float);
}

}  // namespace

extern "C" size_t q3t_linear_chain_workspace_bytes(int64_t rows) {
  if (rows < 1 || rows > 64) return 0;
  return scratch_bytes(rows_tile(rows), sm_count());
}

extern "C" int q3t_linear_chain(const q3t_chain_stage* stages, int count, int64_t rows, void* workspace,
                                size_t workspace_bytes, unsigned* status, void* stream) {
  if (stages == nullptr || count < 1 || count > kMaxStages) return fail(Q3T_EINVAL, "linear_chain: 1..%d stages", kMaxStages);
  if (rows < 1 || rows > 64) return fail(Q3T_EUNSUPPORTED, "linear_chain: rows must be 1..64");
  const int bn = rows_tile(rows);
  ChainParams p;
  memset(&p, 0, sizeof(p));
  int grid = sm_count();
  int tile_base = 0;
  for (int s = 0; s < count; ++s) {
    const q3t_chain_stage& q = stages[s];
    if (!q.x || !q.weight_tiles || !q.out) return fail(Q3T_EINVAL, "linear_chain: stage %d: null pointer", s);
    if (q.in_features < 8 || q.in_features % 8 || q.out_features < 1 || q.x_stride < q.in_features ||
        q.x_stride % 8 || !aligned16(q.x) || !aligned16(q.weight_tiles))
      return fail(Q3T_EINVAL, "linear_chain: stage %d: shape, stride or alignment", s);
    const bool swiglu = q.epilogue == Q3T_EPI_SWIGLU_PAIRED;
    if (q.epilogue != Q3T_EPI_STORE && q.epilogue != Q3T_EPI_RESIDUAL && !swiglu)
      return fail(Q3T_EINVAL, "linear_chain: stage %d: epilogue must be STORE, RESIDUAL or SWIGLU_PAIRED", s);
    if (q.out_stride < (swiglu ? q.out_features / 2 : q.out_features))
      return fail(Q3T_EINVAL, "linear_chain: stage %d: out_stride too small", s);
    if (q.out_dtype != Q3T_BF16 && (q.out_dtype != Q3T_F32 || q.epilogue != Q3T_EPI_STORE))
      return fail(Q3T_EINVAL, "linear_chain: stage %d: fp32 output only with the STORE epilogue", s);
    if (q.epilogue == Q3T_EPI_RESIDUAL && (q.residual == nullptr || q.residual_stride < q.out_features))
      return fail(Q3T_EINVAL, "linear_chain: stage %d: residual epilogue needs a residual", s);
    if (swiglu && (q.out_features % kTileN || q.bias != nullptr))
      return fail(Q3T_EINVAL, "linear_chain: stage %d: paired SwiGLU needs out_features %% 128 == 0, no bias", s);
    if (!(q.row_norm_eps >= 0.f)) return fail(Q3T_EINVAL, "linear_chain: stage %d: row-norm eps must be >= 0", s);
    if (q.depends < -1 || q.depends >= s) return fail(Q3T_EINVAL, "linear_chain: stage %d: depends on a later stage", s);
    Stage& st = p.st[s];
    st.tiles = static_cast<const uint8_t*>(q.weight_tiles);
    st.out = q.out;
    st.residual = static_cast<const __nv_bfloat16*>(q.residual);
    st.bias = static_cast<const __nv_bfloat16*>(q.bias);
    st.out_stride = q.out_stride;
    st.res_stride = q.residual_stride;
    st.in_features = int(q.in_features);
    st.out_features = int(q.out_features);
    st.kblocks = int((q.in_features + kTileK - 1) / kTileK);
    st.n_tiles = int((q.out_features + kTileN - 1) / kTileN);
    st.units = st.kblocks * st.n_tiles;
    st.epilogue = q.epilogue;
    st.out_f32 = q.out_dtype == Q3T_F32;
    st.row_norm = q.row_norm_eps > 0.f;
    st.norm_eps = q.row_norm_eps;
    st.tile_base = tile_base;
    st.depends = q.depends;
    tile_base += st.n_tiles;
    st.ctas = st.units / kMinUnits < grid ? st.units / kMinUnits : grid;
    if (st.ctas < 1) st.ctas = 1;
    const int rc = make_map_bf16(&p.x[s], q.x, rows, q.in_features, q.x_stride, kTileK, bn);
    if (rc) return rc;
  }
  if (kSyncTiles + tile_base > kSyncWords) return fail(Q3T_EUNSUPPORTED, "linear_chain: too many output tiles");
  {
    int widest = 1;
    for (int s = 0; s < count; ++s) widest = p.st[s].ctas > widest ? p.st[s].ctas : widest;
    grid = widest;   // every CTA works in at least one stage
  }
  if (grid > kMaxGrid) return fail(Q3T_EUNSUPPORTED, "linear_chain: more than %d SMs", kMaxGrid);
  // pieces per stage: every CTA touches tiles [u0 / K, (u1 - 1) / K]
  int per_cta = 1;
  for (int s = 0; s < count; ++s) {
    Stage& st = p.st[s];
    int pieces = 0;
    for (int c = 0; c < st.ctas; ++c) {
      const int u0 = int((int64_t(c) * st.units) / st.ctas), u1 = int((int64_t(c + 1) * st.units) / st.ctas);
      const int touched = (u1 - 1) / st.kblocks - u0 / st.kblocks + 1;
      pieces += touched;
      if (touched > per_cta) per_cta = touched;
    }
    st.segments = pieces;
  }
  if (per_cta > kMaxPieces)
    return fail(Q3T_EUNSUPPORTED, "linear_chain: a CTA would touch %d tiles of one stage (at most %d)", per_cta,
                kMaxPieces);
  const size_t need = scratch_bytes(bn, grid);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))
    return fail(Q3T_ESPACE, "linear_chain: workspace needs %zu bytes", need);
  p.stages = count;
  p.rows = int(rows);
  p.counters = kSyncTiles + tile_base;
  p.sync = static_cast<unsigned*>(workspace);
  p.pieces = per_cta;
  p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + size_t(kSyncWords) * 4);
  p.sumsq = p.partials + size_t(grid) * per_cta * bn * kTileN;
  p.status = status;
  switch (bn) {
    case 16: return launch_chain<16>(p, grid, stream);
    case 32: return launch_chain<32>(p, grid, stream);
    default: return launch_chain<64>(p, grid, stream);
  }
}
