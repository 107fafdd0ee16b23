// Dense projections (QKV, O, gate/up, down, LM heads) as tcgen05 GEMMs.
//
// Decode GEMMs have few rows (the batch, 1..64) against thousands of output
// features, so they are weight-streaming, HBM-bound problems. The kernel
// therefore puts the WEIGHTS in the 128-row UMMA A operand and the activation
// rows in the N dimension ("swap-AB"): one CTA owns 128 output features x BN
// rows, streams its 128 x K weight slab through a TMA/mbarrier ring into
// 128-byte-swizzled shared memory and accumulates in TMEM. K is split across
// the CTAs of a thread-block cluster (1..8 splits) so that ~2 CTAs per SM
// stream weights. Each CTA finalises 128 / splits of the tile's features: the
// other CTAs' fp32 partials of them reach it through distributed shared memory
// (tiles of <= 64 rows: a dedicated inbox filled by one bulk copy per source;
// 128-row tiles: stores into its idle ring), and it reduces them in fixed rank
// order (deterministic, no global scratch) and applies the fused epilogue.
//
// Roles (256 threads): warp0.lane0 = TMA producer, warp1 = TMEM owner and
// lane0 = MMA issuer, warps 2-7 = row sums of the folded RMSNorm, all eight
// warps = epilogue (warp w reads TMEM lanes 32(w%4)..+31, i.e. output features).
// Eight epilogue warps keep enough work in flight for the latency-bound
// epilogues (SnakeBeta, split-K partial loads). Weight tiles of the first ring
// slots are requested before griddepcontrol.wait, so with programmatic dependent
// launch the weight stream starts while the previous kernel is still finishing.
#include "common.cuh"
#include "host.cuh"

#include <mutex>
#include <string.h>

using namespace q3t;

namespace {

constexpr int kTileN = 128;   // weight rows per CTA (UMMA M)
constexpr int kThreads = 256;
constexpr int kTileK = 64;    // bf16 elements per 128-byte swizzled row
constexpr int kABytes = kTileN * kTileK * 2;

template <int BN>
struct Cfg {
  // Ring depth: as deep as two CTAs per SM allow; tiles of <= 64 rows also hold a split-K inbox
  // beside the ring.
  static constexpr int kStages = BN <= 16 ? 5 : BN <= 32 ? 4 : BN <= 128 ? 3 : 2;
  static constexpr int kBBytes = BN * kTileK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int kRing = kStages * kStageBytes;
  // split-K reduce buffer: column-major [BN][128 + 4] fp32 (rows of one batch column contiguous)
  static constexpr int kRedStride = kTileN + 4;
  static constexpr int kRedBytes = BN * kRedStride * 4;
  static constexpr int kMain = kRing > kRedBytes ? kRing : kRedBytes;
  static constexpr int kNormRows = (BN + 5) / 6;          // activation rows per norm warp (warps 2-7)
  static constexpr int kNormGroups = (kNormRows + 3) / 4;  // four rows per warp load
  // Split-K exchange (tiles of <= 64 rows): the owner of a feature receives every cluster peer's
  // fp32 partials of it in a dedicated inbox, [source rank][W + 1][BN + 4] floats (feature-major,
  // rows contiguous; row W of a source holds its partial row sums), at most (128 + 8)(BN + 4)
  // floats for any split count. Larger tiles exchange through the idle ring.
  static constexpr bool kAsyncExchange = BN <= 64;
  static constexpr int kInboxRow = BN + 4;
  static constexpr int kInboxBytes = kAsyncExchange ? (kTileN + 8) * kInboxRow * 4 : 0;
  // main area, inbox, barriers (2 per stage + done + 2) + tmem slot + flags, row scales [BN] of the
  // folded RMSNorm, plus 1 KB alignment slack
  static constexpr int kSmem = kMain + kInboxBytes + 256 + 1024 + 1024;
};

struct GemmArgs {
  int rows, in_features, out_features, kblocks, splits;
  // Q3T_WEIGHTS_TILED: weight tile (n-tile, k-block) is the contiguous 16 KB
  // swizzled shared-memory image at tiles + (n-tile * kblocks + k-block) * 16 KB
  const uint8_t* tiles;
  const __nv_bfloat16* bias;
  void* out;
  int64_t out_stride;
  int out_f32;
  const __nv_bfloat16* residual;
  int64_t res_stride;
  const __nv_bfloat16* scale;  // per-feature scale of Q3T_EPI_RESIDUAL_SCALED
  int row_norm;                // scale row m by 1/sqrt(mean_k x[m,k]^2 + norm_eps) (folded RMSNorm)
  float norm_eps;
  // L2 prefetch hint: bytes the NEXT kernel of the chain will stream (its weights),
  // split evenly over this grid's CTAs and requested at kernel start
  const uint8_t* prefetch;
  uint64_t prefetch_bytes;
  // L2 priority of the weight tiles: 0 = normal (several row tiles read each weight tile),
  // 1 = evict-first (one row tile: streamed once), 2 = evict-last (Q3T_LINEAR_KEEP_WEIGHTS:
  // weights a chain re-reads soon, the code predictor's layers once per codebook step).
  int weight_policy;
  // Implicit causal convolution (conv_taps > 0): the activations are a padded buffer
  // [batch, pad + frames, channels] (3-D tensor map); k-block kb covers tap j = kb / conv_cblocks,
  // channels (kb % conv_cblocks) * 64 + [0, 64), and reads frames t + shift(j) of the stream, with
  // shift(j) = j * dilation, or (taps - 1 - j) * dilation when conv_reverse. The m-tiles of a stream
  // (conv_tiles of them) cover its frames; output row = stream * conv_frames + frame.
  int conv_taps, conv_dil, conv_reverse, conv_cblocks, conv_frames, conv_tiles;
  const float* snake_alpha;  // per-feature SnakeBeta parameters of Q3T_EPI_SNAKE
  const float* snake_inv;
  // Staged epilogue (one-CTA tiles, bf16 output): the residual tile arrives by one TMA load
  // (tmr) and the finished [BN x 128] tile leaves by one TMA store (tmo), both through the
  // idle ring; 3-D maps {features, frames, streams} in conv mode, so stores clip per stream.
  int tma_out;
  unsigned* status;
};

__device__ __forceinline__ float silu_gate(float g, float u) {
  return bf16r(bf16r(g / (1.0f + expf(-g))) * u);
}

__host__ __device__ constexpr bool has_residual(int epi) { return epi == Q3T_EPI_RESIDUAL || epi == Q3T_EPI_RESIDUAL_SCALED; }

// Final value of one output element (non-SwiGLU epilogues) from its accumulator
// (bias already added), its residual input r and its per-feature scale g.
template <int EPI>
__device__ __forceinline__ float epilogue_value(float acc, float r, float g) {
  if constexpr (EPI == Q3T_EPI_RESIDUAL) {
    return r + bf16r(acc);
  } else if constexpr (EPI == Q3T_EPI_RESIDUAL_SCALED) {
    return r + bf16r(g * bf16r(acc));
  } else if constexpr (EPI == Q3T_EPI_GELU) {
    const float v = bf16r(acc);
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752f));
  } else if constexpr (EPI == Q3T_EPI_SILU) {
    const float v = bf16r(acc);
    return v / (1.0f + expf(-v));
  } else if constexpr (EPI == Q3T_EPI_SNAKE) {  // r = alpha[n], g = 1 / beta[n]
    return snake_bf16(bf16r(acc), r, g);
  } else {
    return acc;
  }
}

template <int EPI>
__device__ __forceinline__ void store_value(const GemmArgs& a, int m, int n, float v) {
  if (EPI == Q3T_EPI_STORE && a.out_f32)
    static_cast<float*>(a.out)[int64_t(m) * a.out_stride + n] = bf16r(v);
  else
    static_cast<__nv_bfloat16*>(a.out)[int64_t(m) * a.out_stride + n] = __float2bfloat16_rn(v);
}

// Output elements (m_first + j, n), j < 16, of one feature n. All residual inputs
// are loaded before the first store: the residual may alias the output, and
// interleaved load/store pairs would serialise one memory round trip per element.
template <int EPI>
__device__ __forceinline__ void store_rows16(const GemmArgs& a, int m_first, int m_end, int n, const float* v,
                                             const float* rscale) {
  const bool hb = a.bias != nullptr;
  const float bias = hb ? __bfloat162float(a.bias[n]) : 0.f;
  const float g = EPI == Q3T_EPI_RESIDUAL_SCALED ? __bfloat162float(a.scale[n])
                  : EPI == Q3T_EPI_SNAKE         ? a.snake_inv[n]
                                                 : 0.f;
  const float alpha = EPI == Q3T_EPI_SNAKE ? a.snake_alpha[n] : 0.f;
  float r[16];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    r[j] = (has_residual(EPI) && m_first + j < m_end)
               ? __bfloat162float(a.residual[int64_t(m_first + j) * a.res_stride + n])
               : alpha;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    if (m_first + j >= m_end) break;
    float acc = rscale != nullptr ? v[j] * rscale[j] : v[j];
    if (hb) acc += bias;
    store_value<EPI>(a, m_first + j, n, epilogue_value<EPI>(acc, r[j], g));
  }
}

// Epilogue inputs of output elements (m, n_first + j), j < 4: residual, bias and per-feature
// scale, loaded up front so that their latency overlaps the split-K partial loads.
struct Inputs4 {
  float r[4], bias[4], g[4];
};
template <int EPI>
__device__ __forceinline__ Inputs4 load_inputs4(const GemmArgs& a, int m, int n_first) {
  Inputs4 in;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const bool live = n_first + j < a.out_features;
    in.r[j] = (has_residual(EPI) && live) ? __bfloat162float(a.residual[int64_t(m) * a.res_stride + n_first + j])
                                          : 0.f;
    in.bias[j] = (a.bias != nullptr && live) ? __bfloat162float(a.bias[n_first + j]) : 0.f;
    in.g[j] = (EPI == Q3T_EPI_RESIDUAL_SCALED && live) ? __bfloat162float(a.scale[n_first + j]) : 0.f;
    if (EPI == Q3T_EPI_SNAKE && live) {
      in.r[j] = a.snake_alpha[n_first + j];
      in.g[j] = a.snake_inv[n_first + j];
    }
  }
  return in;
}

// Output elements (m, n_first + j), j < 4, of one activation row (features bounded by out_features).
template <int EPI>
__device__ __forceinline__ void store_features4(const GemmArgs& a, int m, int n_first, const float* v,
                                                const Inputs4& in) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (n_first + j >= a.out_features) break;
    float acc = v[j];
    if (a.bias != nullptr) acc += in.bias[j];
    store_value<EPI>(a, m, n_first + j, epilogue_value<EPI>(acc, in.r[j], in.g[j]));
  }
}

// Weight tile (k-block kb, rows n0..n0+127) into a ring slot: one contiguous
// 16 KB bulk copy from the pre-swizzled tile layout, or a 2-D TMA tile load.
Q3T_DEV void load_weights(uint8_t* dst, const CUtensorMap* tmw, const GemmArgs& a, uint64_t* bar, int kb, int n0,
                          uint64_t pol) {
  if (a.tiles != nullptr) {
    const size_t tile = size_t(n0 / kTileN) * size_t(a.kblocks) + size_t(kb);
    if (a.weight_policy != 0)
      bulk_load_hint(dst, a.tiles + tile * size_t(kABytes), uint32_t(kABytes), bar, pol);
    else
      bulk_load(dst, a.tiles + tile * size_t(kABytes), uint32_t(kABytes), bar);
  } else {
    tma_load_2d(dst, tmw, bar, kb * kTileK, n0, pol);
  }
}

Q3T_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
Q3T_DEV uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
Q3T_DEV uint32_t map_peer(uint32_t local_smem, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_smem), "r"(rank));
  return remote;
}
Q3T_DEV void st_peer1(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
Q3T_DEV void cluster_arrive() { asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory"); }
// Bulk copy of `bytes` from this CTA's shared memory to a cluster peer's (dst and the peer's
// mbarrier are shared::cluster addresses from map_peer); completion is counted on that
// mbarrier (complete_tx). Both addresses 16-byte aligned, bytes a multiple of 16.
Q3T_DEV void bulk_copy_peer(uint32_t dst, const void* src, uint32_t bytes, uint32_t peer_bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(peer_bar)
               : "memory");
}
Q3T_DEV void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;" ::: "memory"); }

// One CTA = 128 weight rows x BN activation rows x one K slice. The CTAs of
// the K slices of one tile form a thread-block cluster (gridDim.y = splits,
// 1..8) and reduce their fp32 accumulators through
// distributed shared memory: each writes its tile column-major into its own
// shared memory, then CTA of cluster rank r sums its share of the tile's
// feature quads over all peers in rank order (deterministic) and applies the
// epilogue.
template <int BN, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                  const __grid_constant__ CUtensorMap tmo, const __grid_constant__ CUtensorMap tmr, GemmArgs a) {
  using C = Cfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* inbox_area = reinterpret_cast<float*>(smem + C::kMain);  // split-K inbox (kAsyncExchange)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kMain + C::kInboxBytes);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint64_t* epi_bar = done + 1;  // residual tile of the staged epilogue
  uint64_t* inbox_bar = epi_bar + 1;  // split-K partials of this CTA's features have landed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(inbox_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;  // ring slots the MMA issuer has taken
  float* red = reinterpret_cast<float*>(smem);
  // folded RMSNorm: per activation row its sum of squares over this CTA's K slice, later turned
  // into the row scale in place
  float* rnorm = reinterpret_cast<float*>(smem + C::kMain + C::kInboxBytes + 256);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTileN;
  const int split = blockIdx.y;
  // activation tile: rows [m0, m0 + BN) of a plain GEMM, or frames [t0, t0 + BN) of stream
  // conv_b of an implicit conv; output rows below m_end exist
  const int conv_b = a.conv_taps ? int(blockIdx.z) / a.conv_tiles : 0;
  const int t0 = a.conv_taps ? (int(blockIdx.z) % a.conv_tiles) * BN : 0;
  const int m0 = a.conv_taps ? conv_b * a.conv_frames + t0 : int(blockIdx.z) * BN;
  const int m_end = a.conv_taps ? conv_b * a.conv_frames + (a.conv_frames < t0 + BN ? a.conv_frames : t0 + BN)
                                : a.rows;
  const int kb0 = int(int64_t(split) * a.kblocks / a.splits);
  const int kb1 = int(int64_t(split + 1) * a.kblocks / a.splits);
  const int nk = kb1 - kb0;
  const bool clustered = a.splits > 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      // a slot is free once the MMAs read it and, with row_norm, each of the six norm warps summed it
      mbar_init(&empty[s], a.row_norm ? 7 : 1);
    }
    mbar_init(done, 1);
    mbar_init(epi_bar, 1);
    mbar_init(inbox_bar, 1);
    if (C::kAsyncExchange && clustered) {
      // every cluster peer copies W feature rows of partials (+ its row sums with row_norm)
      const int W = kTileN / a.splits;
      mbar_expect_tx(inbox_bar, uint32_t((a.splits - 1) * (W + (a.row_norm ? 1 : 0)) * C::kInboxRow * 4));
    }
    *abort_flag = 0;
    *consumed = 0;
    fence_mbar_init();
    if (a.tiles == nullptr) prefetch_tmap(&tmw);
    prefetch_tmap(&tmx);
    if (a.tma_out) {
      prefetch_tmap(&tmo);
      if (has_residual(EPI)) prefetch_tmap(&tmr);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // peers send into this CTA's inbox only after its barrier is initialised and armed: this arrive
  // pairs with the cluster wait before the sends
  if (C::kAsyncExchange && clustered) cluster_arrive();
  const uint32_t tmem = *tmem_slot;
  int issued = 0;  // producer only
  if (a.prefetch != nullptr && threadIdx.x == 64) {
    // this CTA's share of the next kernel's weights, in 16-byte units, pulled into L2
    const uint64_t ctas = uint64_t(gridDim.x) * gridDim.y * gridDim.z;
    const uint64_t id = blockIdx.x + uint64_t(gridDim.x) * (blockIdx.y + uint64_t(gridDim.y) * blockIdx.z);
    prefetch_l2_share(a.prefetch, a.prefetch_bytes, id, ctas);
  }

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: weight tiles of the first ring slots go out before the
      // dependency wait (weights never depend on the previous kernel), activations after it.
      const uint64_t pol_w = a.weight_policy == 2 ? policy_evict_last() : policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      auto load_act = [&](uint8_t* dst, uint64_t* bar, int kb) {
        if (a.conv_taps) {
          const int j = kb / a.conv_cblocks, cb = kb - j * a.conv_cblocks;
          const int shift = (a.conv_reverse ? a.conv_taps - 1 - j : j) * a.conv_dil;
          tma_load_3d(dst, &tmx, bar, cb * kTileK, t0 + shift, conv_b, pol_x);
        } else {
          tma_load_2d(dst, &tmx, bar, kb * kTileK, m0, pol_x);
        }
      };
      const int pre = nk < S ? nk : S;
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], C::kStageBytes);
        load_weights(smem + i * C::kStageBytes, &tmw, a, &full[i], kb0 + i, n0, pol_w);
      }
      issued = pre;
      grid_dependency_wait();
      for (int i = 0; i < pre; ++i)
        load_act(smem + i * C::kStageBytes + kABytes, &full[i], kb0 + i);
      for (int i = pre; i < nk; ++i) {
        const int s = i % S;
        if (*abort_flag || !mbar_wait(&empty[s], ((i / S) & 1) ^ 1, a.status, kStatusMmaTimeout)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&full[s], C::kStageBytes);
        load_weights(smem + s * C::kStageBytes, &tmw, a, &full[s], kb0 + i, n0, pol_w);
        load_act(smem + s * C::kStageBytes + kABytes, &full[s], kb0 + i);
        issued = i + 1;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16(kTileN, BN);
      for (int i = 0; i < nk; ++i) {
        const int s = i % S;
        if (!mbar_wait(&full[s], (i / S) & 1, a.status, kStatusTmaTimeout)) {
          *abort_flag = 1;
          break;
        }
        *consumed = i + 1;
        tc_fence_after();
        const uint64_t ad = umma_desc_sw128(smem_u32(smem + s * C::kStageBytes));
        const uint64_t bd = umma_desc_sw128(smem_u32(smem + s * C::kStageBytes + kABytes));
#pragma unroll
        for (int k = 0; k < kTileK / 16; ++k) umma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (i > 0 || k > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      umma_commit(done);
    }
    __syncwarp();
  }

  // ---------------- folded RMSNorm: warps 2-7 (idle during the main loop) sum the squares of
  // every activation row from the ring slots as they land, over this CTA's K slice. Warp w owns
  // rows [(w - 2) R, (w - 1) R) (R = ceil(BN / 6)); in each stage lane l reads 16-byte chunk
  // l % 8 of row l / 8 of a group of four rows (one conflict-free 512-byte wavefront set), so a
  // stage costs each warp a few loads and a slot is released (empty barrier: MMA commit + one
  // arrival per norm warp) right after it lands. The eight chunk lanes of a row are added by a
  // fixed butterfly at the end, and rnorm[m] holds the row's sum over this K slice.
  if (a.row_norm && warp >= 2) {
    const int nw = warp - 2;
    const int row_lo = nw * C::kNormRows;
    const int chunk = lane & 7, sub = lane >> 3;
    float acc[C::kNormGroups];
#pragma unroll
    for (int j = 0; j < C::kNormGroups; ++j) acc[j] = 0.f;
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!mbar_wait(&full[s], (i / S) & 1, a.status, kStatusTmaTimeout)) {
        *abort_flag = 1;
        break;
      }
      const uint8_t* xb = smem + s * C::kStageBytes + kABytes;
#pragma unroll
      for (int j = 0; j < C::kNormGroups; ++j) {
        const int m = row_lo + 4 * j + sub;
        if (4 * j + sub < C::kNormRows && m < BN) {
          const uint4 v = *reinterpret_cast<const uint4*>(xb + m * 128 + chunk * 16);
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = __uint_as_float(w4[e] << 16), hi = __uint_as_float(w4[e] & 0xFFFF0000u);
            acc[j] += lo * lo + hi * hi;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
#pragma unroll
    for (int j = 0; j < C::kNormGroups; ++j) {
      float v = acc[j];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      const int m = row_lo + 4 * j + sub;
      if (chunk == 0 && 4 * j + sub < C::kNormRows && m < BN) rnorm[m] = v;
    }
  }
  grid_dependency_wait();

  // ---------------- split-K epilogue inputs (inbox form), loaded while the MMAs still run: the
  // output quads of this thread are feature fq x rows 4q..4q+3, q = (thread + i * 256) / nf
  const int xr_cs = a.splits;
  const int xr_rank = clustered ? int(cluster_rank()) : 0;
  const int xr_W = kTileN / xr_cs;
  const int nf = EPI == Q3T_EPI_SWIGLU_PAIRED ? xr_W / 2 : xr_W;
  const int units = nf * (BN / 4);
  // at most 64 features per owner (two or more splits): nf divides the block, so a thread's quads
  // all belong to one feature
  constexpr int kU = BN / 16 > 0 ? BN / 16 : 1;
  const int fq = int(threadIdx.x) % nf, nq = n0 + xr_rank * xr_W + fq;
  const bool nlive = nq < a.out_features;
  float pre_r[kU][4];
  float pre_b = 0.f, pre_g = 0.f;
  if constexpr (C::kAsyncExchange && EPI != Q3T_EPI_SWIGLU_PAIRED) {
    if (clustered) {
      pre_b = (nlive && a.bias != nullptr) ? __bfloat162float(a.bias[nq]) : 0.f;
      pre_g = !nlive                          ? 0.f
              : EPI == Q3T_EPI_RESIDUAL_SCALED ? __bfloat162float(a.scale[nq])
              : EPI == Q3T_EPI_SNAKE           ? a.snake_inv[nq]
                                               : 0.f;
#pragma unroll
      for (int i = 0; i < kU; ++i) {
        const int u = threadIdx.x + i * kThreads, q = u / nf;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int m = m0 + 4 * q + e;
          pre_r[i][e] = (has_residual(EPI) && nlive && u < units && m < m_end)
                            ? __bfloat162float(a.residual[int64_t(m) * a.res_stride + nq])
                            : (EPI == Q3T_EPI_SNAKE && nlive ? a.snake_alpha[nq] : 0.f);
        }
      }
    }
  }

  // ---------------- TMEM -> registers
  const bool ok = mbar_wait(done, 0, a.status, kStatusMmaTimeout);
  tc_fence_after();
  const int quad = warp & 3, half = warp >> 2;
  const int r = quad * 32 + lane;  // tile row (output feature n0 + r)
  const uint32_t taddr = tmem + (uint32_t(quad * 32) << 16);
  if (!clustered && EPI != Q3T_EPI_SWIGLU_PAIRED) {
    const int n = n0 + r;
    if (a.row_norm) {
      __syncthreads();  // every row's sum is in rnorm
      if (threadIdx.x < BN) rnorm[threadIdx.x] = 1.0f / sqrtf(rnorm[threadIdx.x] / float(a.in_features) + a.norm_eps);
      __syncthreads();
    }
    // block-uniform: every thread saw the accumulator complete and no load was abandoned
    if (a.tma_out && __syncthreads_and(ok && !*abort_flag)) {
      // Staged epilogue: the ring is idle (every load was consumed by the MMAs), so it holds
      // the [BN rows x 128 features] bf16 tile; thread r owns feature n0 + r of every row.
      __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(smem);
      bool res_ok = true;
      if constexpr (has_residual(EPI)) {
        if (threadIdx.x == 0) {
          mbar_expect_tx(epi_bar, uint32_t(BN * kTileN * 2));
          if (a.conv_taps)
            tma_load_3d(stage, &tmr, epi_bar, n0, t0, conv_b, policy_evict_first());
          else
            tma_load_2d(stage, &tmr, epi_bar, n0, m0, policy_evict_first());
        }
        res_ok = mbar_wait(epi_bar, 0, a.status, kStatusTmaTimeout);
      }
      const bool live = n < a.out_features;
      const bool hb = a.bias != nullptr;
      const float bias = hb && live ? __bfloat162float(a.bias[n]) : 0.f;
      const float g = !live                             ? 0.f
                      : EPI == Q3T_EPI_RESIDUAL_SCALED ? __bfloat162float(a.scale[n])
                      : EPI == Q3T_EPI_SNAKE           ? a.snake_inv[n]
                                                       : 0.f;
      const float alpha = EPI == Q3T_EPI_SNAKE && live ? a.snake_alpha[n] : 0.f;
#pragma unroll 1
      for (int c0 = 16 * half; c0 < BN; c0 += 32) {
        float v[16];
        tmem_ld16(taddr + c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          __nv_bfloat16* slot = stage + (c0 + j) * kTileN + r;
          const float rr = has_residual(EPI) ? __bfloat162float(*slot) : alpha;
          float acc = a.row_norm ? v[j] * rnorm[c0 + j] : v[j];
          if (hb) acc += bias;
          *slot = __float2bfloat16_rn(epilogue_value<EPI>(acc, rr, g));
        }
      }
      fence_async_shared();  // the tile's generic-proxy writes, before the TMA store reads them
      tc_fence_before();
      __syncthreads();
      if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
      if (threadIdx.x == 0 && res_ok) {
        if (a.conv_taps)
          tma_store_3d(&tmo, stage, n0, t0, conv_b);
        else
          tma_store_2d(&tmo, stage, n0, m0);
        bulk_commit_group();
        bulk_wait_read0();  // the tile must stay until the store engine has read it
      } else if (threadIdx.x == 0 && has_residual(EPI)) {
        mbar_wait(epi_bar, 0, a.status, kStatusTmaTimeout);  // a late residual load lands before exit
      }
      return;
    }
#pragma unroll 1
    for (int c0 = 16 * half; c0 < BN; c0 += 32) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (ok && n < a.out_features) store_rows16<EPI>(a, m0 + c0, m_end, n, v, a.row_norm ? rnorm + c0 : nullptr);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
  } else if (clustered) {
    // ---------------- split-K reduction across the cluster. The CTA that finalises a feature
    // (its owner) receives every peer's fp32 partials of it and sums them in rank order
    // (deterministic).
    if (threadIdx.x == 0 && *abort_flag)  // outstanding ring loads land before the ring is reused
      for (int j = *consumed; j < issued; ++j) mbar_wait(&full[j % S], (j / S) & 1, a.status, kStatusTmaTimeout);
    __syncthreads();
    const int cs = a.splits;
    const int rank = int(cluster_rank());
    const int W = kTileN / cs;  // features this CTA finalises (cs is a power of two <= 8)
    int owner, fl;
    if constexpr (EPI == Q3T_EPI_SWIGLU_PAIRED) {  // tile rows are [64 gate; 64 up]
      const int hw = W / 2, rr = r < 64 ? r : r - 64;
      owner = rr / hw;
      fl = (r < 64 ? 0 : hw) + rr - owner * hw;
    } else {
      owner = r / W;
      fl = r - owner * W;
    }
    const int mcount = (m_end - m0) < BN ? (m_end - m0) : BN;
    if constexpr (C::kAsyncExchange) {
      // Inbox form (tiles of <= 64 rows): every thread writes its half of its feature's rows from
      // the accumulator registers into this CTA's idle ring, grouped by owner in the owner's inbox
      // slot layout (its own features straight into its own inbox), and one thread copies each
      // owner's slot into that owner's dedicated inbox with a bulk shared::cluster copy counted on
      // the owner's inbox barrier (armed with the expected bytes at kernel start). No cluster
      // barrier follows the MMAs: the inbox is not shared with the ring, and the cluster barrier
      // begun at kernel start (waited before the first copy) only orders the copies after every
      // peer armed its barrier. The owner reduces once its inbox is complete; a second split
      // cluster barrier (arrive then, wait before exit) keeps every CTA resident until all copies
      // out of its staging have landed.
      constexpr int R4 = C::kInboxRow;
      const int slot_floats = (W + 1) * R4;  // one source's slot: W feature rows + the row sums
      cluster_wait();  // every peer's inbox barrier is initialised and armed
      float* staging = reinterpret_cast<float*>(smem);  // the idle ring: [cs][slot_floats], by owner
      {
        // this thread's BN / 2 rows of feature r (half 0: the first half of the rows), one TMEM load
        constexpr int NC = BN / 2;
        float v[NC];
        const int c0 = half * NC;
        tmem_ld<NC>(taddr + c0, v);
        if (!ok) {
#pragma unroll
          for (int j = 0; j < NC; ++j) v[j] = 0.f;
        }
        // owner `rank`: straight into this CTA's inbox; other owners: this CTA's idle ring
        // (staging, one slot per owner in the inbox slot layout), copied out below
        float* dst = (owner == rank ? inbox_area + rank * slot_floats : staging + owner * slot_floats) + fl * R4 + c0;
#pragma unroll
        for (int j = 0; j < NC; j += 4)
          *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
      if (a.row_norm && threadIdx.x < cs * (BN / 4)) {  // this CTA's partial row sums go to every owner
        const int o = threadIdx.x / (BN / 4), k = threadIdx.x % (BN / 4);  // owner o, rows 4k..4k+3
        float* dst = (o == rank ? inbox_area + rank * slot_floats : staging + o * slot_floats) + W * R4 + 4 * k;
        *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(rnorm + 4 * k);
      }
      fence_async_shared();  // the staging writes, before the bulk copies read them
      tc_fence_before();
      __syncthreads();  // staging and this CTA's own slot are written, every TMEM read is done
      if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
      if (threadIdx.x == 0) {
        const uint32_t bytes = uint32_t((W + (a.row_norm ? 1 : 0)) * R4 * 4);
        for (int o = 0; o < cs; ++o)
          if (o != rank)
            bulk_copy_peer(map_peer(smem_u32(inbox_area + rank * slot_floats), uint32_t(o)), staging + o * slot_floats,
                           bytes, map_peer(smem_u32(inbox_bar), uint32_t(o)));
      }
      const bool got = mbar_wait(inbox_bar, 0, a.status, kStatusTmaTimeout);  // peers' partials
      cluster_arrive();  // this CTA's inbox is complete; it leaves once every inbox is (its staging is read)
      if (!got) {
        cluster_wait();
        return;
      }
      // folded RMSNorm: one scale per row (sum of every source's partial row sums in rank order),
      // over this CTA's own row sums (already copied into its inbox and staging; the ring may
      // still be read by copies in flight)
      float* rscale = rnorm;
      if (a.row_norm) {
        if (threadIdx.x < BN) {
          float t = 0.f;
          for (int j = 0; j < cs; ++j) t += inbox_area[j * slot_floats + W * R4 + threadIdx.x];
          rscale[threadIdx.x] = 1.0f / sqrtf(t / float(a.in_features) + a.norm_eps);
        }
        __syncthreads();
      }
      // the sums of this thread's quads, every quad's partials loaded before any is used
      const int lg = __ffs(nf) - 1;
      float4 acc[kU], upv[kU];
      int qs[kU];
      bool live[kU];
#pragma unroll
      for (int i = 0; i < kU; ++i) {
        const int u = threadIdx.x + i * kThreads;
        const int q = u >> lg;
        live[i] = u < units && 4 * q < mcount;
        qs[i] = live[i] ? q : 0;
        acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        upv[i] = acc[i];
      }
      for (int j = 0; j < cs; ++j) {
        const float* src = inbox_area + j * slot_floats + fq * R4;
#pragma unroll
        for (int i = 0; i < kU; ++i) {
          const float4 p = *reinterpret_cast<const float4*>(src + 4 * qs[i]);
          acc[i].x += p.x; acc[i].y += p.y; acc[i].z += p.z; acc[i].w += p.w;
          if constexpr (EPI == Q3T_EPI_SWIGLU_PAIRED) {
            const float4 w = *reinterpret_cast<const float4*>(src + nf * R4 + 4 * qs[i]);
            upv[i].x += w.x; upv[i].y += w.y; upv[i].z += w.z; upv[i].w += w.w;
          }
        }
      }
#pragma unroll
      for (int i = 0; i < kU; ++i) {
        if (!live[i]) continue;
        const int q = qs[i];
        float av[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
        float uv[4] = {upv[i].x, upv[i].y, upv[i].z, upv[i].w};
        if (a.row_norm) {
          const float4 rn = *reinterpret_cast<const float4*>(rscale + 4 * q);
          const float rv[4] = {rn.x, rn.y, rn.z, rn.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            av[e] *= rv[e];
            uv[e] *= rv[e];
          }
        }
        if constexpr (EPI == Q3T_EPI_SWIGLU_PAIRED) {
          const int ft = rank * nf + fq;  // gate feature within the tile
          if (n0 + 64 + ft < a.out_features) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int m = m0 + 4 * q + e;
              if (m < m_end)
                static_cast<__nv_bfloat16*>(a.out)[int64_t(m) * a.out_stride + (n0 / 2 + ft)] =
                    __float2bfloat16_rn(silu_gate(bf16r(av[e]), bf16r(uv[e])));
            }
          }
        } else if (nlive) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int m = m0 + 4 * q + e;
            if (m < m_end) store_value<EPI>(a, m, nq, epilogue_value<EPI>(av[e] + pre_b, pre_r[i][e], pre_g));
          }
        }
      }
      cluster_wait();  // every inbox of the cluster is complete: no copy still reads this CTA's staging
    } else {
      // Ring form (128-row tiles): after one cluster barrier (every ring idle) each thread stores
      // its partials into the owner's shared memory, then a second cluster barrier; the owner
      // reduces its inbox in rank order.
      const int rs = W + 4;  // inbox row stride in floats; column W holds the partial row sums
      float* inbox = reinterpret_cast<float*>(smem);  // [cs][BN][rs]
      cluster_sync();
      const uint32_t inbox_u32 = smem_u32(inbox);
      const uint32_t dst = map_peer(inbox_u32, uint32_t(owner)) + uint32_t(rank * BN * rs + fl) * 4u;
#pragma unroll 1
      for (int c0 = 16 * half; c0 < BN; c0 += 32) {
        float v[16];
        tmem_ld16(taddr + c0, v);
#pragma unroll
        for (int j = 0; j < 16; ++j) st_peer1(dst + uint32_t((c0 + j) * rs) * 4u, ok ? v[j] : 0.f);
      }
      if (a.row_norm && threadIdx.x < BN)  // this CTA's partial row sums go to every owner
        for (int o = 0; o < cs; ++o)
          st_peer1(map_peer(inbox_u32, uint32_t(o)) + uint32_t((rank * BN + threadIdx.x) * rs + W) * 4u,
                   rnorm[threadIdx.x]);
      tc_fence_before();
      __syncthreads();
      if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
      cluster_sync();  // every partial has landed in its owner's inbox
      auto row_scale = [&](int c) -> float {
        float total = 0.f;
        for (int j = 0; j < cs; ++j) total += inbox[(j * BN + c) * rs + W];
        return 1.0f / sqrtf(total / float(a.in_features) + a.norm_eps);
      };
      if constexpr (EPI == Q3T_EPI_SWIGLU_PAIRED) {
        const int hw = W / 2, nq = hw / 4;
        const int units = mcount * nq;
        for (int u = threadIdx.x; u < units; u += blockDim.x) {
          const int c = u / nq;
          const int f = (u % nq) * 4;  // local gate feature; its up partner sits at hw + f
          float4 g = make_float4(0.f, 0.f, 0.f, 0.f), up = g;
          for (int j = 0; j < cs; ++j) {
            const float* row = inbox + (j * BN + c) * rs;
            const float4 gv = *reinterpret_cast<const float4*>(row + f);
            const float4 uv = *reinterpret_cast<const float4*>(row + hw + f);
            g.x += gv.x; g.y += gv.y; g.z += gv.z; g.w += gv.w;
            up.x += uv.x; up.y += uv.y; up.z += uv.z; up.w += uv.w;
          }
          if (a.row_norm) {
            const float rn = row_scale(c);
            g.x *= rn; g.y *= rn; g.z *= rn; g.w *= rn;
            up.x *= rn; up.y *= rn; up.z *= rn; up.w *= rn;
          }
          const int ft = rank * hw + f;  // gate feature within the tile
          __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + int64_t(m0 + c) * a.out_stride + (n0 / 2 + ft);
          const float gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {up.x, up.y, up.z, up.w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (n0 + 64 + ft + j < a.out_features) o[j] = __float2bfloat16_rn(silu_gate(bf16r(gs[j]), bf16r(us[j])));
        }
      } else {
        const int nq = W / 4;
        const int units = mcount * nq;
        for (int u = threadIdx.x; u < units; u += blockDim.x) {
          const int c = u / nq;
          const int f = (u % nq) * 4;
          const int n = n0 + rank * W + f;
          const Inputs4 in = load_inputs4<EPI>(a, m0 + c, n);
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int j = 0; j < cs; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(inbox + (j * BN + c) * rs + f);
            acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
          }
          float vals[4] = {acc.x, acc.y, acc.z, acc.w};
          if (a.row_norm) {
            const float rn = row_scale(c);
#pragma unroll
            for (int j = 0; j < 4; ++j) vals[j] *= rn;
          }
          store_features4<EPI>(a, m0 + c, n, vals, in);
        }
      }
    }
  } else if constexpr (EPI == Q3T_EPI_SWIGLU_PAIRED) {
    // ---------------- one CTA per tile, paired SwiGLU: the tile goes through shared memory so
    // that each thread finalises whole gate/up quad pairs
    if (threadIdx.x == 0 && *abort_flag)
      for (int j = *consumed; j < issued; ++j) mbar_wait(&full[j % S], (j / S) & 1, a.status, kStatusTmaTimeout);
    __syncthreads();
#pragma unroll 1
    for (int c0 = 16 * half; c0 < BN; c0 += 32) {
      float v[16];
      tmem_ld16(taddr + c0, v);
#pragma unroll
      for (int j = 0; j < 16; ++j) red[(c0 + j) * C::kRedStride + r] = ok ? v[j] : 0.f;
    }
    if (a.row_norm && threadIdx.x < BN)
      rnorm[threadIdx.x] = 1.0f / sqrtf(rnorm[threadIdx.x] / float(a.in_features) + a.norm_eps);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
    const int mcount = (m_end - m0) < BN ? (m_end - m0) : BN;
    const int units = mcount * 16;
    for (int u = threadIdx.x; u < units; u += blockDim.x) {
      const int c = u / 16;
      const int f = (u % 16) * 4;
      float4 g = *reinterpret_cast<const float4*>(red + c * C::kRedStride + f);
      float4 up = *reinterpret_cast<const float4*>(red + c * C::kRedStride + 64 + f);
      if (a.row_norm) {
        const float rn = rnorm[c];
        g.x *= rn; g.y *= rn; g.z *= rn; g.w *= rn;
        up.x *= rn; up.y *= rn; up.z *= rn; up.w *= rn;
      }
      __nv_bfloat16* o = static_cast<__nv_bfloat16*>(a.out) + int64_t(m0 + c) * a.out_stride + (n0 / 2 + f);
      const float gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {up.x, up.y, up.z, up.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (n0 + 64 + f + j < a.out_features) o[j] = __float2bfloat16_rn(silu_gate(bf16r(gs[j]), bf16r(us[j])));
    }
  }
}

// ---------------------------------------------------------------- wide tiles
// Row counts in the thousands (a packed prefill's prompt rows) make the projections
// tensor-bound rather than weight-streaming. linear_wide_kernel is persistent, one CTA per SM:
// CTA c walks tiles c, c + grid, ... of 128 output features x 256 rows over the whole K (no
// split), with one k-block ring across its tiles and TWO TMEM accumulators of 256 columns, so
// the epilogue of tile j (TMEM -> registers -> bf16 staging -> TMA store, in 64-row chunks)
// runs while the MMAs of tile j + 1 fill the other accumulator. Tiles are numbered
// feature-block-major (consecutive CTAs share a weight tile; every operand stays in L2).
// Roles (320 threads): warp 0 lane 0 = TMA producer, warp 1 = TMEM owner, lane 0 the MMA
// issuer, warps 2-9 = epilogue (warp w reads TMEM lanes 32(w%4)..+31 = output features, and
// the first (w < 6) or second 32 rows of each 64-row chunk).
// Epilogue decisions that follow a bounded wait are taken together (barrier reduction), so a
// timeout never splits the epilogue warps across barriers.
constexpr int kWideRows = 256;                            // activation rows per tile (UMMA N)
constexpr int kWideStages = 4;
constexpr int kWideStageBytes = kABytes + kWideRows * kTileK * 2;  // 16 KB weights + 32 KB rows
constexpr int kWideRing = kWideStages * kWideStageBytes;
constexpr int kWideChunk = 64;                            // rows per staged output chunk
constexpr int kWideStaging = kWideChunk * kTileN * 2;     // 16 KB
constexpr int kWideThreads = 320;
constexpr int kWideEpiThreads = kWideThreads - 64;
constexpr int kWideSmem = kWideRing + kWideStaging + 256 + 1024;
static_assert(kWideSmem <= 232448, "wide GEMM shared memory");

struct WideArgs {
  int rows, out_features, kblocks, n_tiles, m_tiles;
  const uint8_t* tiles;        // pre-swizzled weight tiles (Q3T_WEIGHTS_TILED layout)
  const __nv_bfloat16* bias;
  const __nv_bfloat16* scale;  // per-feature scale of Q3T_EPI_RESIDUAL_SCALED
  unsigned* status;
};

Q3T_DEV void epi_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Barrier of the 256 epilogue threads that also ANDs `pred` over them.
Q3T_DEV bool epi_bar_and(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.pred q, 1, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(uint32_t(pred))
      : "memory");
  return r != 0;
}
// 16 TMEM columns of this warp's lanes without the completion wait (tmem_wait_ld follows).
Q3T_DEV void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
Q3T_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

template <int EPI>
__global__ void __launch_bounds__(kWideThreads, 1)
    linear_wide_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmo,
                       const __grid_constant__ CUtensorMap tmr, WideArgs a) {
  constexpr int S = kWideStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + kWideRing;
  uint64_t* full = reinterpret_cast<uint64_t*>(staging + kWideStaging);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;    // [2] accumulator b complete
  uint64_t* tempty = tfull + 2;   // [2] accumulator b read out by the 8 epilogue warps
  uint64_t* res_bar = tempty + 2; // residual chunk landed in the staging buffer
  uint64_t* mma_done = res_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = a.n_tiles * a.m_tiles;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kWideEpiThreads / 32);
    }
    mbar_init(res_bar, 1);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    prefetch_tmap(&tmx);
    prefetch_tmap(&tmo);
    if (has_residual(EPI)) prefetch_tmap(&tmr);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * kWideRows);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      const uint64_t pol_x = policy_evict_last();
      int it = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x) {
        const int nt = t / a.m_tiles, mt = t - nt * a.m_tiles;
        for (int kb = 0; kb < a.kblocks; ++kb) {
          const int s = it % S;
          if (*abort_flag || !mbar_wait(&empty[s], ((it / S) & 1) ^ 1, a.status, kStatusMmaTimeout)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* dst = smem + s * kWideStageBytes;
          mbar_expect_tx(&full[s], kWideStageBytes);
          bulk_load(dst, a.tiles + (size_t(nt) * size_t(a.kblocks) + size_t(kb)) * size_t(kABytes), kABytes,
                    &full[s]);
          tma_load_2d(dst + kABytes, &tmx, &full[s], kb * kTileK, mt * kWideRows, pol_x);
          ++it;
        }
      }
      // loads still in flight land before the CTA can exit (the last load of each slot)
      if (*abort_flag)
        for (int i = it > S ? it - S : 0; i < it; ++i) mbar_wait(&full[i % S], (i / S) & 1, a.status, kStatusTmaTimeout);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc = umma_idesc_bf16(kTileN, kWideRows);
      int it = 0, j = 0;
      for (int t = blockIdx.x; t < tiles && !*abort_flag; t += gridDim.x, ++j) {
        const int b = j & 1;
        if (!mbar_wait(&tempty[b], ((j >> 1) & 1) ^ 1, a.status, kStatusMmaTimeout)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + uint32_t(b * kWideRows);
        bool ok = true;
        for (int kb = 0; kb < a.kblocks; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1, a.status, kStatusTmaTimeout)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = umma_desc_sw128(smem_u32(smem + s * kWideStageBytes));
          const uint64_t bd = umma_desc_sw128(smem_u32(smem + s * kWideStageBytes + kABytes));
#pragma unroll
          for (int k = 0; k < kTileK / 16; ++k) umma_bf16(d, ad + 2 * k, bd + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        umma_commit(&tfull[b]);
      }
      // every MMA of this CTA has completed before TMEM is released
      umma_commit(mma_done);
      mbar_wait(mma_done, 0, a.status, kStatusMmaTimeout);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: warps 2-9
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;      // rows 32*half .. +31 of each chunk
    const int r = quad * 32 + lane;        // tile row = output feature n0 + r
    const int et = threadIdx.x - 64;       // 0 .. 255
    const bool leader = et == 0;
    __nv_bfloat16* stage = reinterpret_cast<__nv_bfloat16*>(staging);
    int j = 0, chunks = 0;
    bool res_pending = false;  // leader: a residual load whose landing nobody saw
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++j) {
      const int b = j & 1;
      const int nt = t / a.m_tiles, mt = t - nt * a.m_tiles;
      const int n0 = nt * kTileN, m0 = mt * kWideRows;
      const bool ready = mbar_wait(&tfull[b], (j >> 1) & 1, a.status, kStatusMmaTimeout);
      if (!epi_bar_and(ready && !*abort_flag)) {
        if (leader) *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t tbase = tmem + (uint32_t(quad * 32) << 16) + uint32_t(b * kWideRows + 32 * half);
      const int n = n0 + r;
      const bool live = n < a.out_features;
      const float bias = (a.bias != nullptr && live) ? __bfloat162float(a.bias[n]) : 0.f;
      const float g = (EPI == Q3T_EPI_RESIDUAL_SCALED && live) ? __bfloat162float(a.scale[n]) : 0.f;
      bool ok = true;
      for (int h = 0; h < kWideRows / kWideChunk && ok; ++h) {
        const int mc = m0 + h * kWideChunk;
        if (mc >= a.rows) break;
        // the staging buffer is free once the previous chunk's store has read it
        if (leader) {
          bulk_wait_read0();
          if constexpr (has_residual(EPI)) {
            mbar_expect_tx(res_bar, uint32_t(kWideStaging));
            tma_load_2d(stage, &tmr, res_bar, n0, mc, policy_evict_first());
            res_pending = true;
          }
        }
        if constexpr (has_residual(EPI)) {
          const bool landed = mbar_wait(res_bar, uint32_t(chunks & 1), a.status, kStatusTmaTimeout);
          if (leader && landed) res_pending = false;
          ok = epi_bar_and(landed);
          if (!ok) {
            if (leader) *abort_flag = 1;
            break;
          }
        } else {
          epi_bar_sync();
        }
        ++chunks;
        uint32_t raw[2][16];
        tmem_ld16_async(tbase + uint32_t(h * kWideChunk), raw[0]);
        tmem_ld16_async(tbase + uint32_t(h * kWideChunk + 16), raw[1]);
        tmem_wait_ld();
        int store_col = n0;
        if constexpr (EPI == Q3T_EPI_SWIGLU_PAIRED) {
          // tile rows are [64 gate; 64 up] of output features n0/2 .. n0/2 + 63. The chunk goes
          // through shared memory as bf16 (silu_gate rounds both inputs to bf16 first), then every
          // epilogue thread finalises 16 rows of one feature.
#pragma unroll
          for (int i = 0; i < 32; ++i)
            stage[(32 * half + i) * kTileN + r] = __float2bfloat16_rn(__uint_as_float(raw[i >> 4][i & 15]));
          epi_bar_sync();
          const int f = et & 63, r0 = (et >> 6) * 16;
          float o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            o[i] = silu_gate(__bfloat162float(stage[(r0 + i) * kTileN + f]),
                             __bfloat162float(stage[(r0 + i) * kTileN + 64 + f]));
          epi_bar_sync();  // every gate/up value is read before the outputs overwrite them
#pragma unroll
          for (int i = 0; i < 16; ++i) stage[(r0 + i) * 64 + f] = __float2bfloat16_rn(o[i]);
          store_col = n0 / 2;
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            __nv_bfloat16* slot = stage + (32 * half + i) * kTileN + r;
            const float rr = has_residual(EPI) ? __bfloat162float(*slot) : 0.f;
            *slot = __float2bfloat16_rn(epilogue_value<EPI>(__uint_as_float(raw[i >> 4][i & 15]) + bias, rr, g));
          }
        }
        fence_async_shared();  // generic-proxy writes of the chunk, before the TMA store reads them
        epi_bar_sync();
        if (leader) {
          tma_store_2d(&tmo, stage, store_col, mc);
          bulk_commit_group();
        }
      }
      // accumulator b is read out (every tcgen05.ld above has completed)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[b]);
      if (!ok) break;
    }
    if (leader) {
      bulk_wait_read0();  // the staging buffer stays until the last store has read it
      if (res_pending) mbar_wait(res_bar, uint32_t(chunks & 1), a.status, kStatusTmaTimeout);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, 2 * kWideRows);
}

// Weight [N, K] row-major -> tiles [ceil(N/128)][ceil(K/64)] of the 128-byte-swizzled
// shared-memory image (row r, 16-byte chunk j stored at chunk j ^ (r % 8)); padding is zero.
__global__ void pack_tiles_kernel(const __nv_bfloat16* __restrict__ w, int64_t n, int64_t k, int64_t kblocks,
                                  int64_t total_chunks, uint4* __restrict__ tiles) {
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total_chunks;
       i += int64_t(gridDim.x) * blockDim.x) {
    // i enumerates destination 16-byte chunks in storage order
    const int64_t tile = i / (kTileN * 8), within = i % (kTileN * 8);
    const int r = int(within / 8), pos = int(within % 8);
    const int j = pos ^ (r & 7);  // logical chunk stored at this position
    const int64_t nt = tile / kblocks, kb = tile % kblocks;
    const int64_t row = nt * kTileN + r, col = kb * kTileK + int64_t(j) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < n) {
      if (col + 8 <= k) {
        v = *reinterpret_cast<const uint4*>(w + row * k + col);
      } else {
        __nv_bfloat16 e[8];
        for (int q = 0; q < 8; ++q) e[q] = (col + q < k) ? w[row * k + col + q] : __float2bfloat16_rn(0.f);
        v = *reinterpret_cast<const uint4*>(e);
      }
    }
    tiles[i] = v;
  }
}

// ---------------------------------------------------------------- host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// 2-D bf16 K-major map: dims {cols, rows}, box {64, box_rows}, 128-byte swizzle.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t stride_elems, int box_rows) {
  EncodeTiled enc = encoder();
  if (enc == nullptr) return fail(Q3T_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(stride_elems) * 2};
  cuuint32_t box[2] = {cuuint32_t(kTileK), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q3T_EINVAL, "tensor map encode failed (%d)", int(r));
  return Q3T_OK;
}

// 3-D bf16 map over a padded conv buffer [batch, frames, channels]: box {64, box_rows, 1}, 128-byte swizzle.
int make_map_3d(CUtensorMap* map, const void* base, int64_t batch, int64_t frames, int64_t channels, int box_rows) {
  EncodeTiled enc = encoder();
  if (enc == nullptr) return fail(Q3T_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {cuuint64_t(channels), cuuint64_t(frames), cuuint64_t(batch)};
  cuuint64_t strides[2] = {cuuint64_t(channels) * 2, cuuint64_t(frames) * cuuint64_t(channels) * 2};
  cuuint32_t box[3] = {cuuint32_t(kTileK), cuuint32_t(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q3T_EINVAL, "tensor map encode failed (%d)", int(r));
  return Q3T_OK;
}

// Activation rows per CTA. Large row counts (codec convolutions, prefill) use 128-row tiles:
// two CTAs (16 warps) per SM keep the latency-bound epilogues busy (measured on the codec's
// 61,440-row convolutions: 1.5x faster than 256-row tiles at one CTA per SM).
int pick_bn(int64_t rows) {
  if (rows <= 16) return 16;
  if (rows <= 32) return 32;
  if (rows <= 64) return 64;
  return 128;
}

struct Plan {
  int bn, n_tiles, m_tiles, kblocks, splits;
};

// Tensor maps of one launch: weights (row-major path only), activations, and the staged
// epilogue's output and residual (zeroed when unused).
struct Maps {
  CUtensorMap w, x, o, r;
};

// Maps of the staged epilogue: out (and the residual) as bf16 {features, rows} (frames == 0) or
// {features, frames, streams} maps with a {128, bn} box, no swizzle. False = not eligible
// (alignment, stride or encode), and the kernel then stores element by element.
bool staged_maps(Maps& m, int bn, int64_t out_features, const void* out, int64_t out_stride, const void* residual,
                 int64_t res_stride, int64_t rows, int64_t batch, int64_t frames) {
  EncodeTiled enc = encoder();
  if (enc == nullptr) return false;
  auto make = [&](CUtensorMap* map, const void* base, int64_t stride) -> bool {
    if (!aligned16(base) || stride % 8 || stride < out_features) return false;
    cuuint64_t dims[3] = {cuuint64_t(out_features), cuuint64_t(frames ? frames : rows), cuuint64_t(batch)};
    cuuint64_t strides[2] = {cuuint64_t(stride) * 2, cuuint64_t(frames) * cuuint64_t(stride) * 2};
    cuuint32_t box[3] = {cuuint32_t(kTileN), cuuint32_t(bn), 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, frames ? 3 : 2, const_cast<void*>(base), dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  };
  if (!make(&m.o, out, out_stride)) return false;
  if (residual != nullptr && !make(&m.r, residual, res_stride)) return false;
  return true;
}


// K splits: a power of two <= 8 (one thread-block cluster per tile) with at most
// ~1.33 CTAs per SM in total and at least two k-blocks per split; grids beyond 64
// CTAs need four k-blocks per split, beyond 128 CTAs sixteen, and 8-CTA clusters
// (the costliest reduction) six unless the grid has at most 64 CTAs. (Measured in
// dependent launch chains of every talker, predictor and codec projection at 8-128
// rows, splits 1-8: this pick is the fastest power of two or within 5% of it;
// 3-, 5- and 6-CTA clusters were no faster, 16-CTA clusters 1.6-2x slower.)
void choose_splits(Plan& p) {
  const int base = p.n_tiles * p.m_tiles;
  const int target = sm_count() + sm_count() / 3;
  int splits = 1;
  while (splits < 8) {
    const int next = splits * 2, ctas = base * next, per_split = p.kblocks / next;
    if (ctas > target || per_split < 2 || (ctas > 64 && per_split < 4) || (ctas > 128 && per_split < 16) ||
        (next == 8 && ctas > 64 && per_split < 6))
      break;
    splits = next;
  }
  p.splits = splits;
}

Plan plan(int64_t rows, int64_t in_features, int64_t out_features) {
  Plan p;
  p.bn = pick_bn(rows);
  p.n_tiles = int((out_features + kTileN - 1) / kTileN);
  p.m_tiles = int((rows + p.bn - 1) / p.bn);
  p.kblocks = int((in_features + kTileK - 1) / kTileK);
  choose_splits(p);
  return p;
}

template <int BN, int EPI>
int launch_linear(const Plan& p, const Maps& m, const GemmArgs& args, void* stream) {
  using C = Cfg<BN>;
  static PerDevice smem_once;
  if (const int rc = smem_limit(smem_once, linear_kernel<BN, EPI>, C::kSmem, "linear: set smem")) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_tiles, p.splits, p.m_tiles);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = size_t(C::kSmem);
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = unsigned(p.splits);
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, linear_kernel<BN, EPI>, m.w, m.x, m.o, m.r, args);
  if (err != cudaSuccess) return fail(Q3T_ECUDA, "linear launch failed: %s", cudaGetErrorString(err));
  note_launch();
  return Q3T_OK;
}

// 2-D bf16 map of an output (or residual) matrix {features, rows} with a {box_cols, 64}
// box and no swizzle: one staged chunk of the wide kernel.
bool chunk_map(CUtensorMap* map, const void* base, int64_t rows, int64_t features, int64_t stride, int box_cols) {
  EncodeTiled enc = encoder();
  if (enc == nullptr || !aligned16(base) || stride % 8 || stride < features) return false;
  cuuint64_t dims[2] = {cuuint64_t(features), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(stride) * 2};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(kWideChunk)};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The wide kernel pays once the 256-row tiles fill every SM (measured on the talker prefill
// projections: the split-K kernel's 128-row tiles are faster below that).
bool wide_pays(int64_t rows, int64_t out_features) {
  const int64_t tiles = ((rows + kWideRows - 1) / kWideRows) * ((out_features + kTileN - 1) / kTileN);
  return rows >= 1024 && tiles >= sm_count();
}

template <int EPI>
int launch_wide(const CUtensorMap& x, const CUtensorMap& o, const CUtensorMap& r, const WideArgs& a, void* stream) {
  static PerDevice smem_once;
  if (const int rc = smem_limit(smem_once, linear_wide_kernel<EPI>, kWideSmem, "linear_wide: set smem")) return rc;
  const int tiles = a.n_tiles * a.m_tiles;
  return launch(linear_wide_kernel<EPI>, dim3(unsigned(tiles < sm_count() ? tiles : sm_count())), dim3(kWideThreads),
                size_t(kWideSmem), stream, true, "linear_wide", x, o, r, a);
}

// Returns Q3T_OK / an error code (negative), or kNotWide when the maps cannot be encoded
// (the caller then runs the split-K kernel).
constexpr int kNotWide = 1;
int linear_wide(const void* x, int64_t x_stride, int64_t rows, int64_t in_features, const void* tiles,
                int64_t out_features, const void* bias, void* out, int64_t out_stride, int epilogue,
                const void* residual, int64_t residual_stride, const void* scale, unsigned* status, void* stream) {
  CUtensorMap mx, mo, mr;
  memset(&mr, 0, sizeof(mr));
  const bool paired = epilogue == Q3T_EPI_SWIGLU_PAIRED;
  if (make_map(&mx, x, rows, in_features, x_stride, kWideRows) != Q3T_OK) return kNotWide;
  if (!chunk_map(&mo, out, rows, paired ? out_features / 2 : out_features, out_stride, paired ? 64 : kTileN))
    return kNotWide;
  if (has_residual(epilogue) && !chunk_map(&mr, residual, rows, out_features, residual_stride, kTileN))
    return kNotWide;
  WideArgs a = {};
  a.rows = int(rows);
  a.out_features = int(out_features);
  a.kblocks = int((in_features + kTileK - 1) / kTileK);
  a.n_tiles = int((out_features + kTileN - 1) / kTileN);
  a.m_tiles = int((rows + kWideRows - 1) / kWideRows);
  a.tiles = static_cast<const uint8_t*>(tiles);
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.status = status;
  switch (epilogue) {
    case Q3T_EPI_STORE: return launch_wide<Q3T_EPI_STORE>(mx, mo, mr, a, stream);
    case Q3T_EPI_RESIDUAL: return launch_wide<Q3T_EPI_RESIDUAL>(mx, mo, mr, a, stream);
    case Q3T_EPI_RESIDUAL_SCALED: return launch_wide<Q3T_EPI_RESIDUAL_SCALED>(mx, mo, mr, a, stream);
    case Q3T_EPI_GELU: return launch_wide<Q3T_EPI_GELU>(mx, mo, mr, a, stream);
    case Q3T_EPI_SILU: return launch_wide<Q3T_EPI_SILU>(mx, mo, mr, a, stream);
    default: return launch_wide<Q3T_EPI_SWIGLU_PAIRED>(mx, mo, mr, a, stream);
  }
}

template <int EPI>
int dispatch_bn(const Plan& p, const Maps& m, const GemmArgs& args, void* stream) {
  switch (p.bn) {
    case 16: return launch_linear<16, EPI>(p, m, args, stream);
    case 32: return launch_linear<32, EPI>(p, m, args, stream);
    case 64: return launch_linear<64, EPI>(p, m, args, stream);
    default: return launch_linear<128, EPI>(p, m, args, stream);
  }
}

}  // namespace

extern "C" size_t q3t_weight_tiles_bytes(int64_t out_features, int64_t in_features) {
  if (out_features < 1 || in_features < 1) return 0;
  return size_t((out_features + kTileN - 1) / kTileN) * size_t((in_features + kTileK - 1) / kTileK) * kABytes;
}

extern "C" int q3t_pack_weight_tiles(const void* weight, int64_t out_features, int64_t in_features, void* tiles,
                                     void* stream) {
  if (!weight || !tiles || out_features < 1 || in_features < 8 || in_features % 8 || !aligned16(weight) ||
      !aligned16(tiles))
    return fail(Q3T_EINVAL, "pack_weight_tiles: invalid arguments");
  const int64_t kblocks = (in_features + kTileK - 1) / kTileK;
  const int64_t chunks = int64_t(q3t_weight_tiles_bytes(out_features, in_features) / 16);
  int64_t blocks = (chunks + 255) / 256;
  if (blocks > int64_t(sm_count()) * 16) blocks = int64_t(sm_count()) * 16;
  return launch(pack_tiles_kernel, dim3(unsigned(blocks)), dim3(256), 0, stream, false, "pack_weight_tiles",
                static_cast<const __nv_bfloat16*>(weight), out_features, in_features, kblocks, chunks,
                static_cast<uint4*>(tiles));
}

// The split-K reduction runs through distributed shared memory: no scratch.
extern "C" size_t q3t_linear_workspace_bytes(int64_t rows, int64_t in_features, int64_t out_features) {
  (void)rows;
  (void)in_features;
  (void)out_features;
  return 0;
}

namespace {

int linear_impl(const void* x, int64_t x_stride, int64_t rows, int64_t in_features, const void* weight,
                int64_t out_features, const void* bias, void* out, int64_t out_stride, int out_dtype, int epilogue,
                const void* residual, int64_t residual_stride, const void* scale, float row_norm_eps,
                const void* weight_tiles, const void* prefetch, size_t prefetch_bytes, int flags, unsigned* status,
                void* stream) {
  if (!x || (!weight && !weight_tiles) || !out) return fail(Q3T_EINVAL, "linear: null pointer");
  if (prefetch != nullptr && (!aligned16(prefetch) || prefetch_bytes % 16))
    return fail(Q3T_EINVAL, "linear: prefetch range needs 16-byte alignment and size");
  if (!(row_norm_eps >= 0.f)) return fail(Q3T_EINVAL, "linear: row-norm eps must be >= 0");
  if (rows < 1 || rows > (int64_t(1) << 24) || in_features < 8 || in_features % 8 || out_features < 1 || out_features > (1 << 24))
    return fail(Q3T_EINVAL, "linear: unsupported shape rows=%lld in=%lld out=%lld", (long long)rows,
                (long long)in_features, (long long)out_features);
  if (x_stride < in_features || x_stride % 8 || !aligned16(x) || (weight && !aligned16(weight)) ||
      (weight_tiles && !aligned16(weight_tiles)))
    return fail(Q3T_EINVAL, "linear: x/weight need 16-byte aligned rows");
  if (out_stride < (epilogue == Q3T_EPI_SWIGLU_PAIRED ? out_features / 2 : out_features))
    return fail(Q3T_EINVAL, "linear: out_stride too small");
  if (out_dtype != Q3T_BF16 && out_dtype != Q3T_F32) return fail(Q3T_EINVAL, "linear: out dtype");
  if ((epilogue == Q3T_EPI_RESIDUAL || epilogue == Q3T_EPI_RESIDUAL_SCALED) &&
      (residual == nullptr || out_dtype != Q3T_BF16))
    return fail(Q3T_EINVAL, "linear: residual epilogue needs a bf16 residual and bf16 output");
  if (epilogue == Q3T_EPI_RESIDUAL_SCALED && scale == nullptr)
    return fail(Q3T_EINVAL, "linear: scaled residual epilogue needs a scale vector");
  if ((epilogue == Q3T_EPI_GELU || epilogue == Q3T_EPI_SILU) && out_dtype != Q3T_BF16)
    return fail(Q3T_EINVAL, "linear: GELU/SiLU epilogues are bf16");
  if (epilogue == Q3T_EPI_SWIGLU_PAIRED && (out_features % kTileN || out_dtype != Q3T_BF16 || bias != nullptr))
    return fail(Q3T_EINVAL, "linear: paired SwiGLU needs out_features %% 128 == 0, bf16 output, no bias");
  if (epilogue < Q3T_EPI_STORE || epilogue > Q3T_EPI_SILU)
    return fail(Q3T_EINVAL, "linear: epilogue (the Snake epilogue needs q3t_conv_linear)");
  if (weight_tiles != nullptr && row_norm_eps == 0.f && out_dtype == Q3T_BF16 && prefetch == nullptr && flags == 0 &&
      wide_pays(rows, out_features)) {
    const int rc = linear_wide(x, x_stride, rows, in_features, weight_tiles, out_features, bias, out, out_stride,
                               epilogue, residual, residual_stride, scale, status, stream);
    if (rc != kNotWide) return rc;
  }
  const Plan p = plan(rows, in_features, out_features);
  if (p.m_tiles > 65535) return fail(Q3T_EINVAL, "linear: too many rows (%lld)", (long long)rows);
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  int rc = Q3T_OK;
  if (weight_tiles == nullptr) {
    rc = make_map(&maps.w, weight, out_features, in_features, in_features, kTileN);
    if (rc) return rc;
  }
  rc = make_map(&maps.x, x, rows, in_features, x_stride, p.bn);
  if (rc) return rc;
  GemmArgs a = {};
  a.rows = int(rows);
  a.in_features = int(in_features);
  a.out_features = int(out_features);
  a.kblocks = p.kblocks;
  a.splits = p.splits;
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.out = out;
  a.out_stride = out_stride;
  a.out_f32 = out_dtype == Q3T_F32;
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.res_stride = residual_stride;
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.tiles = static_cast<const uint8_t*>(weight_tiles);
  a.row_norm = row_norm_eps > 0.f ? 1 : 0;
  a.norm_eps = row_norm_eps;
  a.prefetch = prefetch_bytes ? static_cast<const uint8_t*>(prefetch) : nullptr;
  a.prefetch_bytes = prefetch_bytes;
  a.weight_policy = (flags & Q3T_LINEAR_KEEP_WEIGHTS) ? 2 : p.m_tiles == 1 ? 1 : 0;
  a.tma_out = p.splits == 1 && p.bn >= 64 && epilogue != Q3T_EPI_SWIGLU_PAIRED && out_dtype == Q3T_BF16 &&
              staged_maps(maps, p.bn, out_features, out, out_stride, residual, residual_stride, rows, 1, 0);
  a.status = status;
  switch (epilogue) {
    case Q3T_EPI_STORE: return dispatch_bn<Q3T_EPI_STORE>(p, maps, a, stream);
    case Q3T_EPI_RESIDUAL: return dispatch_bn<Q3T_EPI_RESIDUAL>(p, maps, a, stream);
    case Q3T_EPI_RESIDUAL_SCALED: return dispatch_bn<Q3T_EPI_RESIDUAL_SCALED>(p, maps, a, stream);
    case Q3T_EPI_GELU: return dispatch_bn<Q3T_EPI_GELU>(p, maps, a, stream);
    case Q3T_EPI_SILU: return dispatch_bn<Q3T_EPI_SILU>(p, maps, a, stream);
    default: return dispatch_bn<Q3T_EPI_SWIGLU_PAIRED>(p, maps, a, stream);
  }
}

}  // namespace

extern "C" int q3t_linear(const void* x, int64_t x_stride, int64_t rows, int64_t in_features, const void* weight,
                          int64_t out_features, const void* bias, void* out, int64_t out_stride, int out_dtype,
                          int epilogue, const void* residual, int64_t residual_stride, const void* scale,
                          const void* weight_tiles, void* workspace, size_t workspace_bytes, unsigned* status,
                          void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  return linear_impl(x, x_stride, rows, in_features, weight, out_features, bias, out, out_stride, out_dtype, epilogue,
                     residual, residual_stride, scale, 0.f, weight_tiles, nullptr, 0, 0, status, stream);
}

extern "C" int q3t_linear_rownorm(const void* x, int64_t x_stride, int64_t rows, int64_t in_features,
                                  const void* weight, int64_t out_features, const void* bias, void* out,
                                  int64_t out_stride, int out_dtype, int epilogue, const void* residual,
                                  int64_t residual_stride, const void* scale, float eps, const void* weight_tiles,
                                  unsigned* status, void* stream) {
  if (!(eps > 0.f)) return fail(Q3T_EINVAL, "linear_rownorm: eps must be positive");
  return linear_impl(x, x_stride, rows, in_features, weight, out_features, bias, out, out_stride, out_dtype, epilogue,
                     residual, residual_stride, scale, eps, weight_tiles, nullptr, 0, 0, status, stream);
}

extern "C" int q3t_linear_ex(const void* x, int64_t x_stride, int64_t rows, int64_t in_features, const void* weight,
                             int64_t out_features, const void* bias, void* out, int64_t out_stride, int out_dtype,
                             int epilogue, const void* residual, int64_t residual_stride, const void* scale,
                             float eps, const void* weight_tiles, const void* prefetch, size_t prefetch_bytes,
                             int flags, unsigned* status, void* stream) {
  if (!(eps >= 0.f)) return fail(Q3T_EINVAL, "linear_ex: eps must be >= 0");
  if (flags & ~(Q3T_LINEAR_KEEP_WEIGHTS | Q3T_LINEAR_NARROW)) return fail(Q3T_EINVAL, "linear_ex: unknown flags");
  return linear_impl(x, x_stride, rows, in_features, weight, out_features, bias, out, out_stride, out_dtype, epilogue,
                     residual, residual_stride, scale, eps, weight_tiles, prefetch, prefetch_bytes, flags, status,
                     stream);
}

extern "C" int q3t_conv_linear(const void* xs, int64_t batch, int64_t frames, int64_t pad, int64_t channels,
                               int64_t taps, int64_t dilation, int reverse, const void* weight_tiles,
                               int64_t out_features, const void* bias, void* out, int64_t out_stride, int epilogue,
                               const void* residual, int64_t residual_stride, const void* scale,
                               const float* snake_alpha, const float* snake_inv, unsigned* status, void* stream) {
  if (!xs || !weight_tiles || !out) return fail(Q3T_EINVAL, "conv_linear: null pointer");
  if (batch < 1 || batch > 65535 || frames < 1 || frames > (1 << 24) || channels < 8 || channels % 8 ||
      taps < 1 || taps > 64 || dilation < 1 || pad < 0 || out_features < 1 || out_features > (1 << 24))
    return fail(Q3T_EINVAL, "conv_linear: unsupported geometry");
  if (pad < (taps - 1) * dilation) return fail(Q3T_EINVAL, "conv_linear: pad must cover (taps - 1) * dilation");
  if (!aligned16(xs) || !aligned16(weight_tiles)) return fail(Q3T_EINVAL, "conv_linear: 16-byte alignment");
  if (out_stride < out_features) return fail(Q3T_EINVAL, "conv_linear: out_stride too small");
  if (has_residual(epilogue) && residual == nullptr)
    return fail(Q3T_EINVAL, "conv_linear: residual epilogue needs a residual");
  if (epilogue == Q3T_EPI_RESIDUAL_SCALED && scale == nullptr)
    return fail(Q3T_EINVAL, "conv_linear: scaled residual epilogue needs a scale vector");
  if (epilogue == Q3T_EPI_SNAKE && (snake_alpha == nullptr || snake_inv == nullptr))
    return fail(Q3T_EINVAL, "conv_linear: Snake epilogue needs alpha and inverse beta");
  if (epilogue == Q3T_EPI_SWIGLU_PAIRED || epilogue < Q3T_EPI_STORE || epilogue > Q3T_EPI_SNAKE)
    return fail(Q3T_EINVAL, "conv_linear: epilogue");
  Plan p;
  p.bn = pick_bn(frames);
  const int64_t tiles = (frames + p.bn - 1) / p.bn;
  p.n_tiles = int((out_features + kTileN - 1) / kTileN);
  p.m_tiles = int(batch * tiles);
  const int cblocks = int((channels + kTileK - 1) / kTileK);
  p.kblocks = int(taps) * cblocks;
  choose_splits(p);
  if (p.m_tiles > 65535) return fail(Q3T_EINVAL, "conv_linear: too many row tiles");
  Maps maps;
  memset(&maps, 0, sizeof(maps));
  int rc = make_map_3d(&maps.x, xs, batch, pad + frames, channels, p.bn);
  if (rc) return rc;
  GemmArgs a = {};
  a.rows = int(batch * frames);
  a.in_features = p.kblocks * kTileK;
  a.out_features = int(out_features);
  a.kblocks = p.kblocks;
  a.splits = p.splits;
  a.tiles = static_cast<const uint8_t*>(weight_tiles);
  a.bias = static_cast<const __nv_bfloat16*>(bias);
  a.out = out;
  a.out_stride = out_stride;
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.res_stride = residual_stride;
  a.scale = static_cast<const __nv_bfloat16*>(scale);
  a.conv_taps = int(taps);
  a.conv_dil = int(dilation);
  a.conv_reverse = reverse ? 1 : 0;
  a.conv_cblocks = cblocks;
  a.conv_frames = int(frames);
  a.conv_tiles = int(tiles);
  a.snake_alpha = snake_alpha;
  a.snake_inv = snake_inv;
  a.tma_out = p.splits == 1 && p.bn >= 64 &&
              staged_maps(maps, p.bn, out_features, out, out_stride, residual, residual_stride, batch * frames,
                          batch, frames);
  a.status = status;
  switch (epilogue) {
    case Q3T_EPI_STORE: return dispatch_bn<Q3T_EPI_STORE>(p, maps, a, stream);
    case Q3T_EPI_RESIDUAL: return dispatch_bn<Q3T_EPI_RESIDUAL>(p, maps, a, stream);
    case Q3T_EPI_RESIDUAL_SCALED: return dispatch_bn<Q3T_EPI_RESIDUAL_SCALED>(p, maps, a, stream);
    case Q3T_EPI_GELU: return dispatch_bn<Q3T_EPI_GELU>(p, maps, a, stream);
    case Q3T_EPI_SILU: return dispatch_bn<Q3T_EPI_SILU>(p, maps, a, stream);
    default: return dispatch_bn<Q3T_EPI_SNAKE>(p, maps, a, stream);
  }
}
