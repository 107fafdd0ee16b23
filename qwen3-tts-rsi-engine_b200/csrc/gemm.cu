// Dense projections (QKV, O, gate/up, down, LM heads) as tcgen05 GEMMs.
//
// Decode GEMMs have few rows (the batch, 1..64) against thousands of output
// features, so they are weight-streaming, HBM-bound problems. The kernel
// therefore puts the WEIGHTS in the 128-row UMMA A operand and the activation
// rows in the N dimension ("swap-AB"): one CTA owns 128 output features x BN
// rows, streams its 128 x K weight slab through a TMA/mbarrier ring into
// 128-byte-swizzled shared memory and accumulates in TMEM. K is split across
// CTAs so that ~2 CTAs per SM stream weights; each split writes fp32 partials
// and the last CTA of a tile (atomic ticket) sums them in fixed split order
// (deterministic) and applies the fused epilogue.
//
// Roles (128 threads): warp0.lane0 = TMA producer, warp1 = TMEM owner and
// lane0 = MMA issuer, all four warps = epilogue (warp w reads TMEM lanes
// 32w..32w+31). Weight tiles of the first ring slots are requested before
// griddepcontrol.wait, so with programmatic dependent launch the weight stream
// starts while the previous kernel is still finishing.
#include "common.cuh"
#include "host.cuh"

#include <mutex>

using namespace q3t;

namespace {

constexpr int kTileN = 128;   // weight rows per CTA (UMMA M)
constexpr int kTileK = 64;    // bf16 elements per 128-byte swizzled row
constexpr int kABytes = kTileN * kTileK * 2;

template <int BN>
struct Cfg {
  static constexpr int kStages = BN <= 16 ? 6 : BN <= 32 ? 5 : BN <= 64 ? 4 : BN <= 128 ? 3 : 2;
  static constexpr int kBBytes = BN * kTileK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemCols = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  // ring + barriers (2 per stage + done) + tmem slot + flags, plus 1 KB alignment slack
  static constexpr int kSmem = kStages * kStageBytes + 256 + 1024;
};

struct GemmArgs {
  int rows, in_features, out_features, kblocks, splits;
  const __nv_bfloat16* bias;
  void* out;
  int64_t out_stride;
  int out_f32;
  const __nv_bfloat16* residual;
  int64_t res_stride;
  float* partials;      // [splits][rows][out_features]
  unsigned* counters;   // [n_tiles * m_tiles]
  unsigned* status;
};

__device__ __forceinline__ float silu_gate(float g, float u) {
  return bf16r(bf16r(g / (1.0f + expf(-g))) * u);
}

// Stores one output element according to the epilogue (non-SwiGLU).
template <int EPI>
__device__ __forceinline__ void store_out(const GemmArgs& a, int m, int n, float acc) {
  if (a.bias != nullptr) acc += __bfloat162float(a.bias[n]);
  if constexpr (EPI == Q3T_EPI_RESIDUAL) {
    const float r = __bfloat162float(a.residual[int64_t(m) * a.res_stride + n]);
    static_cast<__nv_bfloat16*>(a.out)[int64_t(m) * a.out_stride + n] = __float2bfloat16_rn(r + bf16r(acc));
  } else {
    if (a.out_f32)
      static_cast<float*>(a.out)[int64_t(m) * a.out_stride + n] = bf16r(acc);
    else
      static_cast<__nv_bfloat16*>(a.out)[int64_t(m) * a.out_stride + n] = __float2bfloat16_rn(acc);
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(128, 1)
    linear_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx, GemmArgs a) {
  using C = Cfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* consumed = abort_flag + 1;  // ring slots the MMA issuer has taken
  int* ticket = const_cast<int*>(consumed + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTileN;
  const int split = blockIdx.y;
  const int m0 = blockIdx.z * BN;
  const int kb0 = int(int64_t(split) * a.kblocks / a.splits);
  const int kb1 = int(int64_t(split + 1) * a.kblocks / a.splits);
  const int nk = kb1 - kb0;

  grid_dependency_launch();
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    *consumed = 0;
    fence_mbar_init();
    prefetch_tmap(&tmw);
    prefetch_tmap(&tmx);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  int issued = 0;  // producer only

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
      const int pre = nk < S ? nk : S;
      for (int i = 0; i < pre; ++i) {
        mbar_expect_tx(&full[i], C::kStageBytes);
        tma_load_2d(smem + i * C::kStageBytes, &tmw, &full[i], (kb0 + i) * kTileK, n0, pol_w);
      }
      issued = pre;
      grid_dependency_wait();  // activations come from the previous kernel
      for (int i = 0; i < pre; ++i)
        tma_load_2d(smem + i * C::kStageBytes + kABytes, &tmx, &full[i], (kb0 + i) * kTileK, m0, pol_x);
      for (int i = pre; i < nk; ++i) {
        const int s = i % S;
        if (*abort_flag || !mbar_wait(&empty[s], ((i / S) & 1) ^ 1, a.status, kStatusMmaTimeout)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&full[s], C::kStageBytes);
        tma_load_2d(smem + s * C::kStageBytes, &tmw, &full[s], (kb0 + i) * kTileK, n0, pol_w);
        tma_load_2d(smem + s * C::kStageBytes + kABytes, &tmx, &full[s], (kb0 + i) * kTileK, m0, pol_x);
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
  grid_dependency_wait();

  // ---------------- epilogue: TMEM -> registers -> partials / output
  const bool ok = mbar_wait(done, 0, a.status, kStatusMmaTimeout);
  tc_fence_after();
  const int n = n0 + warp * 32 + lane;
  const uint32_t taddr = tmem + (uint32_t(warp * 32) << 16);
  if (a.splits == 1 && EPI != Q3T_EPI_SWIGLU_PAIRED) {
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (ok && n < a.out_features) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c0 + j;
          if (m < a.rows) store_out<EPI>(a, m, n, v[j]);
        }
      }
    }
  } else {
    float* part = a.partials + int64_t(split) * a.rows * a.out_features;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(taddr + c0, v);
      if (n < a.out_features) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c0 + j;
          if (m < a.rows) part[int64_t(m) * a.out_features + n] = ok ? v[j] : 0.f;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, C::kTmemCols);
  if (threadIdx.x == 0 && *abort_flag) {
    // Failure path: wait (bounded) for ring loads that were issued but never
    // consumed, so no TMA write lands after this CTA's shared memory is gone.
    for (int j = *consumed; j < issued; ++j) mbar_wait(&full[j % S], (j / S) & 1, a.status, kStatusTmaTimeout);
  }
  if (a.splits == 1 && EPI != Q3T_EPI_SWIGLU_PAIRED) return;

  // ---------------- split-K ticket: the last CTA of this tile reduces
  __threadfence();
  __syncthreads();
  const int tile = blockIdx.z * gridDim.x + blockIdx.x;
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&a.counters[tile], 1u);
    *ticket = (prev == unsigned(a.splits - 1)) ? 1 : 0;
  }
  __syncthreads();
  if (*ticket != 1) return;
  __threadfence();
  const int mcount = (a.rows - m0) < BN ? (a.rows - m0) : BN;
  const int64_t plane = int64_t(a.rows) * a.out_features;
  if constexpr (EPI == Q3T_EPI_SWIGLU_PAIRED) {
    const int width = a.out_features / 2;
    for (int e = threadIdx.x; e < mcount * 64; e += blockDim.x) {
      const int m = m0 + e / 64, f = e % 64;
      const int ng = n0 + f, nu = n0 + 64 + f;
      if (nu >= a.out_features) continue;
      float g = 0.f, u = 0.f;
      for (int s = 0; s < a.splits; ++s) {
        g += __ldcg(a.partials + s * plane + int64_t(m) * a.out_features + ng);
        u += __ldcg(a.partials + s * plane + int64_t(m) * a.out_features + nu);
      }
      g = bf16r(g);
      u = bf16r(u);
      static_cast<__nv_bfloat16*>(a.out)[int64_t(m) * a.out_stride + (n0 / 2 + f)] =
          __float2bfloat16_rn(silu_gate(g, u));
      (void)width;
    }
  } else {
    for (int e = threadIdx.x; e < mcount * kTileN; e += blockDim.x) {
      const int m = m0 + e / kTileN, nn = n0 + e % kTileN;
      if (nn >= a.out_features) continue;
      float acc = 0.f;
      for (int s = 0; s < a.splits; ++s) acc += __ldcg(a.partials + s * plane + int64_t(m) * a.out_features + nn);
      store_out<EPI>(a, m, nn, acc);
    }
  }
  if (threadIdx.x == 0) a.counters[tile] = 0u;
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

int pick_bn(int64_t rows) {
  if (rows <= 16) return 16;
  if (rows <= 32) return 32;
  if (rows <= 64) return 64;
  if (rows <= 128) return 128;
  return 256;
}

struct Plan {
  int bn, n_tiles, m_tiles, kblocks, splits;
};

Plan plan(int64_t rows, int64_t in_features, int64_t out_features) {
  Plan p;
  p.bn = pick_bn(rows);
  p.n_tiles = int((out_features + kTileN - 1) / kTileN);
  p.m_tiles = int((rows + p.bn - 1) / p.bn);
  p.kblocks = int((in_features + kTileK - 1) / kTileK);
  const int base = p.n_tiles * p.m_tiles;
  const int target = 2 * sm_count();
  int splits = (target + base / 2) / base;
  const int max_split = p.kblocks / 2 > 1 ? p.kblocks / 2 : 1;
  if (splits > max_split) splits = max_split;
  if (splits < 1) splits = 1;
  p.splits = splits;
  return p;
}

template <int BN, int EPI>
int launch_linear(const Plan& p, const CUtensorMap& tmw, const CUtensorMap& tmx, const GemmArgs& args, void* stream) {
  using C = Cfg<BN>;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(linear_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) !=
        cudaSuccess)
      return check_cuda("linear: set smem");
    configured[dev] = true;
  }
  return launch(linear_kernel<BN, EPI>, dim3(p.n_tiles, p.splits, p.m_tiles), dim3(128), size_t(C::kSmem), stream,
                true, "linear", tmw, tmx, args);
}

template <int EPI>
int dispatch_bn(const Plan& p, const CUtensorMap& tmw, const CUtensorMap& tmx, const GemmArgs& args, void* stream) {
  switch (p.bn) {
    case 16: return launch_linear<16, EPI>(p, tmw, tmx, args, stream);
    case 32: return launch_linear<32, EPI>(p, tmw, tmx, args, stream);
    case 64: return launch_linear<64, EPI>(p, tmw, tmx, args, stream);
    case 128: return launch_linear<128, EPI>(p, tmw, tmx, args, stream);
    default: return launch_linear<256, EPI>(p, tmw, tmx, args, stream);
  }
}

// Workspace layout: a fixed ticket region (kMaxTiles counters, zero between
// calls) followed by the fp32 partials. The ticket region never moves, so
// calls of different shapes sharing one workspace cannot see each other's
// partials as tickets.
constexpr size_t kMaxTiles = 16384;
constexpr size_t kTicketBytes = kMaxTiles * sizeof(unsigned);

size_t workspace_for(const Plan& p, int64_t rows, int64_t out_features) {
  const size_t partial = size_t(p.splits) * size_t(rows) * size_t(out_features) * sizeof(float);
  return kTicketBytes + partial;
}

}  // namespace

extern "C" size_t q3t_linear_workspace_bytes(int64_t rows, int64_t in_features, int64_t out_features) {
  if (rows < 1 || in_features < 1 || out_features < 1) return 0;
  return workspace_for(plan(rows, in_features, out_features), rows, out_features);
}

extern "C" int q3t_linear(const void* x, int64_t x_stride, int64_t rows, int64_t in_features, const void* weight,
                          int64_t out_features, const void* bias, void* out, int64_t out_stride, int out_dtype,
                          int epilogue, const void* residual, int64_t residual_stride, void* workspace,
                          size_t workspace_bytes, unsigned* status, void* stream) {
  if (!x || !weight || !out) return fail(Q3T_EINVAL, "linear: null pointer");
  if (rows < 1 || rows > 65536 || in_features < 8 || in_features % 8 || out_features < 1 || out_features > (1 << 24))
    return fail(Q3T_EINVAL, "linear: unsupported shape rows=%lld in=%lld out=%lld", (long long)rows,
                (long long)in_features, (long long)out_features);
  if (x_stride < in_features || x_stride % 8 || !aligned16(x) || !aligned16(weight))
    return fail(Q3T_EINVAL, "linear: x/weight need 16-byte aligned rows");
  if (out_stride < (epilogue == Q3T_EPI_SWIGLU_PAIRED ? out_features / 2 : out_features))
    return fail(Q3T_EINVAL, "linear: out_stride too small");
  if (out_dtype != Q3T_BF16 && out_dtype != Q3T_F32) return fail(Q3T_EINVAL, "linear: out dtype");
  if (epilogue == Q3T_EPI_RESIDUAL && (residual == nullptr || out_dtype != Q3T_BF16))
    return fail(Q3T_EINVAL, "linear: residual epilogue needs a bf16 residual and bf16 output");
  if (epilogue == Q3T_EPI_SWIGLU_PAIRED && (out_features % kTileN || out_dtype != Q3T_BF16 || bias != nullptr))
    return fail(Q3T_EINVAL, "linear: paired SwiGLU needs out_features %% 128 == 0, bf16 output, no bias");
  if (epilogue < Q3T_EPI_STORE || epilogue > Q3T_EPI_SWIGLU_PAIRED) return fail(Q3T_EINVAL, "linear: epilogue");
  const Plan p = plan(rows, in_features, out_features);
  const bool needs_ws = p.splits > 1 || epilogue == Q3T_EPI_SWIGLU_PAIRED;
  const size_t need = workspace_for(p, rows, out_features);
  if (needs_ws && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)))
    return fail(Q3T_ESPACE, "linear: workspace needs %zu bytes", need);
  CUtensorMap tmw, tmx;
  int rc = make_map(&tmw, weight, out_features, in_features, in_features, kTileN);
  if (rc) return rc;
  rc = make_map(&tmx, x, rows, in_features, x_stride, p.bn);
  if (rc) return rc;
  GemmArgs a;
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
  if (size_t(p.n_tiles) * p.m_tiles > kMaxTiles) return fail(Q3T_EUNSUPPORTED, "linear: more than 16384 tiles");
  a.counters = static_cast<unsigned*>(workspace);
  a.partials = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kTicketBytes) : nullptr;
  a.status = status;
  switch (epilogue) {
    case Q3T_EPI_STORE: return dispatch_bn<Q3T_EPI_STORE>(p, tmw, tmx, a, stream);
    case Q3T_EPI_RESIDUAL: return dispatch_bn<Q3T_EPI_RESIDUAL>(p, tmw, tmx, a, stream);
    default: return dispatch_bn<Q3T_EPI_SWIGLU_PAIRED>(p, tmw, tmx, a, stream);
  }
}
