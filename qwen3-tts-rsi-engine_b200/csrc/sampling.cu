// Fused token sampling: repetition penalty, vocabulary mask, minimum-step EOS
// gate, temperature, top-k (exact radix select, ties kept), softmax, optional
// top-p, vocabulary-order CDF and inverse-CDF selection, plus the `seen`
// update - one CTA per row, everything in shared memory.
//
// Arithmetic follows the reference's fp32 torch path (sampling.py:5-14,
// continuous.py:365-370): true fp32 division by the scalar penalty and
// temperature, softmax as exp(x - max) * (1 / sum), cumsum accumulated in
// double and rounded to fp32 per prefix, IEEE division cdf / cdf[-1].
// Uniforms come from the caller's table (sampling.py:17-19 random_table) or
// from a Philox4x32-10 stream (Salmon et al., SC'11) keyed by `seed`.
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

constexpr int kThreads = 512;
constexpr int kMaxWidth = 4096;
constexpr int kPer = kMaxWidth / kThreads;  // elements per thread (contiguous)

// ---------------------------------------------------------------- Philox4x32-10
struct U4 {
  uint32_t x, y, z, w;
};
__host__ __device__ inline void mulhilo(uint32_t a, uint32_t b, uint32_t& hi, uint32_t& lo) {
  const uint64_t p = uint64_t(a) * uint64_t(b);
  hi = uint32_t(p >> 32);
  lo = uint32_t(p);
}
__host__ __device__ inline U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0, lo0, hi1, lo1;
    mulhilo(0xD2511F53u, c.x, hi0, lo0);
    mulhilo(0xCD9E8D57u, c.z, hi1, lo1);
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}
__host__ __device__ inline float u01(uint32_t x) { return float(x >> 8) * (1.0f / 16777216.0f); }

// ---------------------------------------------------------------- block helpers
__device__ inline uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ inline float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

template <typename T>
__device__ T block_reduce_sum(T v, T* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  T t = l < (kThreads / 32) ? scratch[l] : T(0);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  return t;
}
__device__ float block_reduce_max(float v, float* scratch) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) scratch[w] = v;
  __syncthreads();
  float t = l < (kThreads / 32) ? scratch[l] : -INFINITY;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}
// Exclusive scan of one double per thread across the block (thread order).
__device__ double block_exclusive_scan(double v, double* scratch) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  double incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double n = __shfl_up_sync(0xffffffffu, incl, o);
    if (l >= o) incl += n;
  }
  __syncthreads();
  if (l == 31) scratch[w] = incl;
  __syncthreads();
  if (w == 0) {
    double t = l < (kThreads / 32) ? scratch[l] : 0.0;
    double ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, ti, o);
      if (l >= o) ti += n;
    }
    if (l < (kThreads / 32)) scratch[l] = ti - t;  // exclusive warp offsets
  }
  __syncthreads();
  return scratch[w] + (incl - v);
}

struct SampleArgs {
  const void* logits;
  int logits_bf16;
  int64_t logits_stride;
  const uint8_t* seen;
  int64_t seen_stride;
  const uint8_t* allowed;
  const int64_t* steps;
  int64_t eos, min_steps;
  float penalty, temperature, top_p;
  int top_k;
  const float* uniforms;
  int64_t uniform_stride;
  uint64_t seed;
  const int64_t* offsets;
  int64_t offset_add;
  int64_t* tokens;
  int64_t token_stride;
  uint8_t* seen_out;
  int64_t seen_out_stride;
  int width;
};

__global__ void __launch_bounds__(kThreads) sample_kernel(SampleArgs a) {
  __shared__ unsigned hist[256];
  __shared__ float fscratch[32];
  __shared__ double dscratch[32];
  __shared__ int iscratch[32];
  __shared__ uint32_t sel_prefix;
  __shared__ int sel_remaining;
  __shared__ float cand_p[kMaxWidth];
  __shared__ int cand_i[kMaxWidth];
  __shared__ int cand_n;
  __shared__ uint8_t removed[kMaxWidth];
  grid_dependency_wait();

  const int64_t r = blockIdx.x;
  const int W = a.width;
  const int base = threadIdx.x * kPer;
  float x[kPer];
  // ---- 1. scores with semantic preprocessing
  const int64_t step = a.steps ? a.steps[r] : 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = base + j;
    float v = -INFINITY;
    if (i < W) {
      v = a.logits_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.logits)[r * a.logits_stride + i])
                        : static_cast<const float*>(a.logits)[r * a.logits_stride + i];
      if (a.seen != nullptr && a.seen[r * a.seen_stride + i]) v = v < 0.f ? v * a.penalty : v / a.penalty;
      if (a.allowed != nullptr && !a.allowed[i]) v = -INFINITY;
      if (a.steps != nullptr && i == a.eos && step < a.min_steps) v = -INFINITY;
      v = v / a.temperature;
    }
    x[j] = v;
  }

  // ---- 2. k-th largest score (radix select on order-preserving keys)
  float thr = -INFINITY;
  const int k = a.top_k;
  if (k > 0 && k < W) {
    if (threadIdx.x == 0) {
      sel_prefix = 0u;
      sel_remaining = k;
    }
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (threadIdx.x < 256) hist[threadIdx.x] = 0u;
      __syncthreads();
      const uint32_t prefix = sel_prefix;
      const uint32_t mask = shift == 24 ? 0u : (0xFFFFFFFFu << (shift + 8));
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        if (base + j < W) {
          const uint32_t key = order_key(x[j]);
          if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 0xFFu], 1u);
        }
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        // The digit is the first bin, from the top, at which the cumulative count
        // reaches `remaining`. Lane l holds bins 255-8l .. 248-8l; a warp scan finds
        // the lane, which then walks its eight bins.
        const int lane = threadIdx.x;
        const int rem = sel_remaining;
        const int top = 255 - 8 * lane;
        int cnt[8], local = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          cnt[q] = int(hist[top - q]);
          local += cnt[q];
        }
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += v;
        }
        const int excl = incl - local;
        __syncwarp();
        if (excl < rem && rem <= incl) {
          int r2 = rem - excl, d = top - 7;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (cnt[q] >= r2) {
              d = top - q;
              break;
            }
            r2 -= cnt[q];
          }
          sel_prefix = prefix | (uint32_t(d) << shift);
          sel_remaining = r2;
        }
      }
      __syncthreads();
    }
    thr = key_float(sel_prefix);
  }
  // ---- 3. softmax over the kept scores
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (x[j] >= thr) mx = fmaxf(mx, x[j]);
  mx = block_reduce_max(mx, fscratch);
  float e[kPer];
  float local = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    e[j] = (base + j < W && x[j] >= thr && x[j] != -INFINITY) ? expf(x[j] - mx) : 0.f;
    local += e[j];
  }
  float total = block_reduce_sum(local, fscratch);
  float inv = 1.0f / total;

  // ---- 4. optional top-p over the kept candidates
  if (a.top_p < 1.0f) {
    if (threadIdx.x == 0) cand_n = 0;
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (e[j] > 0.f) {
        const int slot = atomicAdd(&cand_n, 1);
        cand_p[slot] = e[j] * inv;
        cand_i[slot] = base + j;
      }
    }
    __syncthreads();
    const int n = cand_n;
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    for (int i = n + threadIdx.x; i < n2; i += kThreads) {
      cand_p[i] = INFINITY;
      cand_i[i] = 0x7FFFFFFF;
    }
    __syncthreads();
    // bitonic sort ascending by (p, index)
    for (int size = 2; size <= n2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = threadIdx.x; i < n2; i += kThreads) {
          const int j = i ^ stride;
          if (j > i) {
            const bool asc = (i & size) == 0;
            const float pi = cand_p[i], pj = cand_p[j];
            const int ii = cand_i[i], ij = cand_i[j];
            const bool greater = pi > pj || (pi == pj && ii > ij);
            if (greater == asc) {
              cand_p[i] = pj;
              cand_p[j] = pi;
              cand_i[i] = ij;
              cand_i[j] = ii;
            }
          }
        }
        __syncthreads();
      }
    }
    if (threadIdx.x == 0) {
      // drop the low-probability tail whose cumulative mass <= 1 - top_p; always keep the largest
      float cum = 0.f;
      const float cut = 1.0f - a.top_p;
      for (int i = 0; i < n; ++i) {
        cum += cand_p[i];
        if (cum <= cut && i < n - 1) cand_p[i] = -1.f;
      }
    }
    for (int i = threadIdx.x; i < kMaxWidth; i += kThreads) removed[i] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += kThreads)
      if (cand_p[i] < 0.f) removed[cand_i[i]] = 1;
    __syncthreads();
    local = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      if (base + j < W && removed[base + j]) e[j] = 0.f;
      local += e[j];
    }
    total = block_reduce_sum(local, fscratch);
    inv = 1.0f / total;
  }

  // ---- 5. vocabulary-order CDF (double accumulation) and selection
  float p[kPer];
  double dl = 0.0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    p[j] = e[j] * inv;
    dl += double(p[j]);
  }
  double run = block_exclusive_scan(dl, dscratch);
  float cdf[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    run += double(p[j]);
    cdf[j] = float(run);
  }
  // cdf[W - 1] lives in the thread owning index W - 1
  __shared__ float last;
  if (base <= W - 1 && W - 1 < base + kPer) last = cdf[(W - 1) - base];
  float u;
  if (a.uniforms != nullptr) {
    u = a.uniforms[r * a.uniform_stride];
  } else {
    const uint64_t off = (a.offsets ? uint64_t(a.offsets[r]) : uint64_t(r)) + uint64_t(a.offset_add);
    const U4 o = philox4x32_10(U4{uint32_t(off), uint32_t(off >> 32), 0u, 0u}, uint32_t(a.seed), uint32_t(a.seed >> 32));
    u = u01(o.x);
  }
  __syncthreads();
  const float denom = last;
  int count = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (base + j < W && cdf[j] / denom <= u) ++count;
  const int token = block_reduce_sum(count, iscratch);
  if (threadIdx.x == 0) a.tokens[r * a.token_stride] = token;
  if (a.seen_out != nullptr) {
    const int tok = token < W ? token : W - 1;
    for (int i = threadIdx.x; i < W; i += kThreads) {
      const uint8_t s = a.seen ? a.seen[r * a.seen_stride + i] : uint8_t(0);
      a.seen_out[r * a.seen_out_stride + i] = (i == tok) ? uint8_t(1) : s;
    }
  }
}

// token[r] = #{ j : cdf[r, j] / cdf[r, W-1] <= u[r] }   (cdf_triton_ascend.py:8-17)
__global__ void cdf_select_kernel(const float* __restrict__ cdf, const float* __restrict__ u, int64_t* __restrict__ out,
                                  int width) {
  __shared__ int iscratch[32];
  grid_dependency_wait();
  const int64_t r = blockIdx.x;
  const float total = cdf[r * width + width - 1];
  const float ur = u[r];
  int count = 0;
  for (int i = threadIdx.x; i < width; i += kThreads)
    if (__fdiv_rn(cdf[r * width + i], total) <= ur) ++count;
  const int t = block_reduce_sum(count, iscratch);
  if (threadIdx.x == 0) out[r] = t;
}

__global__ void philox_kernel(uint64_t seed, uint64_t offset, float* out, int64_t count) {
  grid_dependency_wait();
  const int64_t groups = (count + 3) / 4;
  for (int64_t g = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; g < groups; g += int64_t(gridDim.x) * blockDim.x) {
    const uint64_t c = offset + uint64_t(g);
    const U4 o = philox4x32_10(U4{uint32_t(c), uint32_t(c >> 32), 0u, 0u}, uint32_t(seed), uint32_t(seed >> 32));
    const uint32_t v[4] = {o.x, o.y, o.z, o.w};
    for (int j = 0; j < 4 && g * 4 + j < count; ++j) out[g * 4 + j] = u01(v[j]);
  }
}

}  // namespace

extern "C" int q3t_cdf_select(const float* cdf, const float* uniforms, int64_t* tokens, int64_t rows, int64_t width,
                              void* stream) {
  if (!cdf || width < 1 || width > kMaxWidth) return fail(Q3T_EINVAL, "CDF must be contiguous FP32 rows of width 1..4096");
  if (!uniforms) return fail(Q3T_EINVAL, "Uniforms must be one contiguous FP32 value per CDF row");
  if (rows < 1) return fail(Q3T_EINVAL, "Empty CDF batch");
  if (!tokens) return fail(Q3T_EINVAL, "cdf_select: null output");
  return launch(cdf_select_kernel, dim3(unsigned(rows)), dim3(kThreads), 0, stream, true, "cdf_select", cdf, uniforms,
                tokens, int(width));
}

extern "C" int q3t_sample(const void* logits, int logits_dtype, int64_t logits_stride, const uint8_t* seen,
                          int64_t seen_stride, const uint8_t* allowed, const int64_t* steps, int64_t eos,
                          int64_t min_steps, float penalty, float temperature, int64_t top_k, float top_p,
                          const float* uniforms, int64_t uniform_stride, uint64_t seed, const int64_t* philox_offsets,
                          int64_t philox_add, int64_t* tokens, int64_t token_stride, uint8_t* seen_out, int64_t seen_out_stride,
                          int64_t rows, int64_t width, void* stream) {
  if (!logits || !tokens || rows < 1 || width < 1 || width > kMaxWidth)
    return fail(Q3T_EINVAL, "sample: rows >= 1 and width in 1..4096 required");
  if (logits_dtype != Q3T_BF16 && logits_dtype != Q3T_F32) return fail(Q3T_EINVAL, "sample: logits dtype");
  if (!(temperature > 0.f) || !(top_p > 0.f) || top_p > 1.f || !(penalty > 0.f))
    return fail(Q3T_EINVAL, "sample: temperature, penalty and top_p must be positive (top_p <= 1)");
  if (steps && (eos < 0 || eos >= width)) return fail(Q3T_EINVAL, "sample: eos outside the vocabulary");
  if (top_k > width) return fail(Q3T_EINVAL, "sample: top_k exceeds the vocabulary");
  SampleArgs a;
  a.logits = logits;
  a.logits_bf16 = logits_dtype == Q3T_BF16;
  a.logits_stride = logits_stride;
  a.seen = seen;
  a.seen_stride = seen_stride;
  a.allowed = allowed;
  a.steps = steps;
  a.eos = eos;
  a.min_steps = min_steps;
  a.penalty = penalty;
  a.temperature = temperature;
  a.top_p = top_p;
  a.top_k = int(top_k);
  a.uniforms = uniforms;
  a.uniform_stride = uniform_stride;
  a.seed = seed;
  a.offsets = philox_offsets;
  a.offset_add = philox_add;
  a.tokens = tokens;
  a.token_stride = token_stride;
  a.seen_out = seen_out;
  a.seen_out_stride = seen_out_stride;
  a.width = int(width);
  return launch(sample_kernel, dim3(unsigned(rows)), dim3(kThreads), 0, stream, true, "sample", a);
}

extern "C" int q3t_philox_uniforms(uint64_t seed, uint64_t offset, float* out, int64_t count, void* stream) {
  if (!out || count < 1) return fail(Q3T_EINVAL, "philox_uniforms: invalid arguments");
  const int64_t groups = (count + 3) / 4;
  int blocks = int((groups + 255) / 256);
  if (blocks > 4 * sm_count()) blocks = 4 * sm_count();
  return launch(philox_kernel, dim3(blocks), dim3(256), 0, stream, true, "philox", seed, offset, out, count);
}
