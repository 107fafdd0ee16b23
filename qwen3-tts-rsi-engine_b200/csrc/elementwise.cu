// HBM-bound copy and elementwise kernels of the decode path: slot-table KV
// writes, packed-prefix and slot copies, RMSNorm, rotary, SwiGLU, Snake,
// codec row scatter and embedding gathers.
//
// All are memory-bound: 16-byte vector accesses where the layout allows,
// one CTA per row where a row reduction is needed.
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

// ------------------------------------------------------------------ KV write
// kv_triton_ascend.py:25-36 `_write_row`: one CTA per batch row writes all
// heads of K and V at positions[row].
template <typename T, bool kVec>
__global__ void kv_write_kernel(const T* __restrict__ keys, int64_t kb, int64_t kh, int64_t kd,
                                const T* __restrict__ values, int64_t vb, int64_t vh, int64_t vd,
                                T* __restrict__ tk, T* __restrict__ tv, const int64_t* __restrict__ positions,
                                int heads, int width, int64_t capacity, unsigned* status) {
  grid_dependency_wait();
  const int b = blockIdx.x;
  const int64_t pos = positions[b];
  if (pos < 0 || pos >= capacity) {
    if (threadIdx.x == 0) raise_status(status, kStatusBadIndex);
    return;
  }
  constexpr int V = kVec ? int(16 / sizeof(T)) : 1;
  const int units = heads * width / V;
  for (int i = threadIdx.x; i < units; i += blockDim.x) {
    const int e = i * V;
    const int h = e / width;
    const int d = e - h * width;
    const size_t dst = ((size_t(b) * heads + h) * size_t(capacity) + size_t(pos)) * width + d;
    if constexpr (kVec) {
      *reinterpret_cast<uint4*>(tk + dst) = *reinterpret_cast<const uint4*>(keys + b * kb + h * kh + d);
      *reinterpret_cast<uint4*>(tv + dst) = *reinterpret_cast<const uint4*>(values + b * vb + h * vh + d);
    } else {
      tk[dst] = keys[b * kb + h * kh + d * kd];
      tv[dst] = values[b * vb + h * vh + d * vd];
    }
  }
}

// ------------------------------------------------------------------ strided 4-D copy
template <typename T>
__global__ void strided_copy4_kernel(T* __restrict__ dst, int64_t d0, int64_t d1, int64_t d2, int64_t d3,
                                     const T* __restrict__ src, int64_t s0, int64_t s1, int64_t s2, int64_t s3,
                                     int64_t n0, int64_t n1, int64_t n2, int64_t n3) {
  grid_dependency_wait();
  const int64_t total = n0 * n1 * n2 * n3;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    int64_t r = i;
    const int64_t i3 = r % n3;
    r /= n3;
    const int64_t i2 = r % n2;
    r /= n2;
    const int64_t i1 = r % n1;
    const int64_t i0 = r / n1;
    dst[i0 * d0 + i1 * d1 + i2 * d2 + i3 * d3] = src[i0 * s0 + i1 * s1 + i2 * s2 + i3 * s3];
  }
}

// ------------------------------------------------------------------ slot / row copies
template <typename T>
__global__ void plane_copy_kernel(T* __restrict__ base, int64_t planes, int64_t plane_stride, int64_t slot_elems,
                                  int64_t src_off, int64_t dst_off) {
  grid_dependency_wait();
  const int64_t total = planes * slot_elems;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = i / slot_elems;
    const int64_t e = i - p * slot_elems;
    base[p * plane_stride + dst_off + e] = base[p * plane_stride + src_off + e];
  }
}

template <typename T>
__global__ void plane_zero_kernel(T* __restrict__ base, int64_t planes, int64_t plane_stride, int64_t elems,
                                  int64_t off) {
  grid_dependency_wait();
  const int64_t total = planes * elems;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t p = i / elems;
    base[p * plane_stride + off + (i - p * elems)] = T{};
  }
}

template <typename T>
__global__ void rows_copy_kernel(char* __restrict__ dst, int64_t dst_pitch, const char* __restrict__ src,
                                 int64_t src_pitch, int64_t row_units, int64_t rows) {
  grid_dependency_wait();
  const int64_t total = row_units * rows;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / row_units;
    const int64_t u = i - r * row_units;
    reinterpret_cast<T*>(dst + r * dst_pitch)[u] = reinterpret_cast<const T*>(src + r * src_pitch)[u];
  }
}

// ------------------------------------------------------------------ RMSNorm
// operators.py:16-23 / HF Qwen3 RMSNorm. One CTA per row, 8 elements per
// thread-iteration; fp32 sum of squares; IEEE 1/sqrt.
__device__ float block_sum(float v, float* scratch) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? scratch[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();
  return t;
}

__global__ void rms_norm_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride,
                                const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int width,
                                float eps, int mode) {
  __shared__ float scratch[32];
  grid_dependency_wait();
  const int64_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * x_stride;
  __nv_bfloat16* yr = out + row * int64_t(width);
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < width; i += blockDim.x * 8) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + i), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
  }
  ss = block_sum(ss, scratch);
  const float r = 1.0f / sqrtf(ss / float(width) + eps);
  for (int i = threadIdx.x * 8; i < width; i += blockDim.x * 8) {
    float f[8], g[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + i), f);
    unpack8(*reinterpret_cast<const uint4*>(w + i), g);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = mode == Q3T_NORM_REFERENCE ? g[j] * bf16r(f[j] * r) : g[j] * (f[j] * r);
    *reinterpret_cast<uint4*>(yr + i) = pack8(f);
  }
}

__global__ void add_rms_norm_kernel(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* h,
                                    const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out,
                                    __nv_bfloat16* res_out, int width, float eps, int mode) {
  extern __shared__ float sums[];  // width floats
  __shared__ float scratch[32];
  grid_dependency_wait();
  const int64_t row = blockIdx.x;
  const int64_t base = row * int64_t(width);
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < width; i += blockDim.x * 8) {
    float fa[8], fh[8], s[8];
    unpack8(*reinterpret_cast<const uint4*>(a + base + i), fa);
    unpack8(*reinterpret_cast<const uint4*>(h + base + i), fh);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float raw = fa[j] + fh[j];
      const float v = mode == Q3T_NORM_NATIVE ? raw : bf16r(raw);
      s[j] = raw;
      sums[i + j] = v;
      ss += v * v;
    }
    *reinterpret_cast<uint4*>(res_out + base + i) = pack8(s);
  }
  ss = block_sum(ss, scratch);
  const float r = 1.0f / sqrtf(ss / float(width) + eps);
  for (int i = threadIdx.x * 8; i < width; i += blockDim.x * 8) {
    float g[8], y[8];
    unpack8(*reinterpret_cast<const uint4*>(w + i), g);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float v = sums[i + j];
      y[j] = mode == Q3T_NORM_REFERENCE ? g[j] * bf16r(v * r) : g[j] * (v * r);
    }
    *reinterpret_cast<uint4*>(out + base + i) = pack8(y);
  }
}

// ------------------------------------------------------------------ rotary (BSND)
// rotary_triton_ascend.py:7-26, bf16 rounding after every product and sum.
__global__ void rotary_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ c,
                              const __nv_bfloat16* __restrict__ s, __nv_bfloat16* __restrict__ y, int heads,
                              int width) {
  grid_dependency_wait();
  const int64_t row = blockIdx.x;  // batch * length
  const int half = width / 2;
  for (int i = threadIdx.x; i < heads * half; i += blockDim.x) {
    const int h = i / half, d = i - h * half;
    const int64_t base = (row * heads + h) * width;
    const float x1 = ld_bf16(x + base + d), x2 = ld_bf16(x + base + d + half);
    const float c1 = ld_bf16(c + row * width + d), c2 = ld_bf16(c + row * width + d + half);
    const float s1 = ld_bf16(s + row * width + d), s2 = ld_bf16(s + row * width + d + half);
    const float o1 = bf16r(x1 * c1) + bf16r(-x2 * s1);
    const float o2 = bf16r(x2 * c2) + bf16r(x1 * s2);
    y[base + d] = __float2bfloat16_rn(o1);
    y[base + d + half] = __float2bfloat16_rn(o2);
  }
}

// ------------------------------------------------------------------ SwiGLU
__global__ void swiglu_kernel(const __nv_bfloat16* __restrict__ packed, __nv_bfloat16* __restrict__ out,
                              int64_t rows, int64_t width) {
  grid_dependency_wait();
  const int64_t total = rows * width / 8;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t e = i * 8;
    const int64_t r = e / width, c = e - r * width;
    float g[8], u[8];
    unpack8(*reinterpret_cast<const uint4*>(packed + r * 2 * width + c), g);
    unpack8(*reinterpret_cast<const uint4*>(packed + r * 2 * width + width + c), u);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = bf16r(g[j] / (1.0f + expf(-g[j]))) * u[j];
    *reinterpret_cast<uint4*>(out + e) = pack8(g);
  }
}

// ------------------------------------------------------------------ Snake
// snake_triton_ascend.py:13-25 (bf16: round after every op) and
// incremental_codec.py:49 (fp32: x + inv_beta * sin(x * alpha)^2).
template <typename T, typename C>
__global__ void snake_kernel(const T* __restrict__ x, const C* __restrict__ alpha, const C* __restrict__ inv,
                             T* __restrict__ y, int64_t channels, int64_t length, int64_t total) {
  grid_dependency_wait();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t ch = (i / length) % channels;
    const float a = float(alpha[ch]);
    const float r = float(inv[ch]);
    const float v = float(x[i]);
    if constexpr (sizeof(T) == 2) {
      const float phase = bf16r(v * a);
      const float sine = bf16r(sinf(phase));
      const float square = bf16r(sine * sine);
      const float scaled = bf16r(r * square);
      y[i] = T(v + scaled);
    } else {
      const float sn = sinf(v * a);
      y[i] = T(v + r * (sn * sn));
    }
  }
}

// ------------------------------------------------------------------ row scatter
// codec_row_scatter.py:8-45: target[indices[row]] = source[row], source up to 4-D strided.
template <typename T>
__global__ void scatter_rows_kernel(T* __restrict__ target, int64_t target_rows, const int64_t* __restrict__ idx,
                                    const T* __restrict__ src, int64_t n, int64_t e1, int64_t e2, int64_t e3,
                                    int64_t s0, int64_t s1, int64_t s2, int64_t s3, unsigned* status) {
  grid_dependency_wait();
  const int64_t row = e1 * e2 * e3;
  const int64_t total = n * row;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / row;
    int64_t e = i - r * row;
    const int64_t dst_row = idx[r];
    if (dst_row < 0 || dst_row >= target_rows) {
      if (e == 0) raise_status(status, kStatusBadIndex);
      continue;
    }
    const int64_t i3 = e % e3;
    e /= e3;
    const int64_t i2 = e % e2;
    const int64_t i1 = e / e2;
    target[dst_row * row + (i - r * row)] = src[r * s0 + i1 * s1 + i2 * s2 + i3 * s3];
  }
}

// ------------------------------------------------------------------ embeddings
__global__ void embedding_kernel(const int64_t* __restrict__ ids, int64_t ids_stride,
                                 const __nv_bfloat16* __restrict__ table, int64_t vocab,
                                 __nv_bfloat16* __restrict__ out, int64_t out_stride, int hidden, unsigned* status) {
  grid_dependency_wait();
  const int64_t r = blockIdx.x;
  const int64_t id = ids[r * ids_stride];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0) raise_status(status, kStatusBadIndex);
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (ok) v = *reinterpret_cast<const uint4*>(table + id * hidden + i);
    *reinterpret_cast<uint4*>(out + r * out_stride + i) = v;
  }
}

// continuous.py:584-601: E_talker[codes0] + sum_g E_g[codes_g] (fp32 sum, one
// rounding) then + text (bf16 add).
__global__ void frame_embed_kernel(const int64_t* __restrict__ codes, int64_t codes_stride,
                                   const __nv_bfloat16* __restrict__ first, int64_t first_vocab,
                                   const __nv_bfloat16* __restrict__ groups_tab, int groups, int64_t group_vocab,
                                   const __nv_bfloat16* __restrict__ text, int64_t text_stride,
                                   __nv_bfloat16* __restrict__ out, int hidden, unsigned* status) {
  grid_dependency_wait();
  const int64_t b = blockIdx.x;
  __shared__ int64_t ids[32];
  if (threadIdx.x <= groups) {
    int64_t id = codes[b * codes_stride + threadIdx.x];
    const int64_t lim = threadIdx.x == 0 ? first_vocab : group_vocab;
    if (id < 0 || id >= lim) {
      raise_status(status, kStatusBadIndex);
      id = -1;
    }
    ids[threadIdx.x] = id;
  }
  __syncthreads();
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int g = 0; g <= groups; ++g) {
      const int64_t id = ids[g];
      if (id < 0) continue;
      const __nv_bfloat16* row =
          g == 0 ? first + id * hidden : groups_tab + ((int64_t(g) - 1) * group_vocab + id) * hidden;
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(row + i), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    if (text != nullptr) {
      float t[8];
      unpack8(*reinterpret_cast<const uint4*>(text + b * text_stride + i), t);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = bf16r(acc[j]) + t[j];
    }
    *reinterpret_cast<uint4*>(out + b * int64_t(hidden) + i) = pack8(acc);
  }
}

// values[i] += delta (device-side position / frame counters).
__global__ void advance_kernel(int64_t* __restrict__ values, int64_t n, int64_t delta) {
  grid_dependency_wait();
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
    values[i] += delta;
}

int grid_for(int64_t total, int threads) {
  const int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count()) * 16;
  return int(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

}  // namespace

// ====================================================================== entry points

extern "C" int q3t_kv_write(const void* keys, const int64_t* ks, const void* values, const int64_t* vs,
                            void* target_keys, void* target_values, const int64_t* positions, int64_t batch,
                            int64_t heads, int64_t width, int64_t capacity, int dtype, unsigned* status,
                            void* stream) {
  if (!keys || !values || !target_keys || !target_values || !positions || !ks || !vs)
    return fail(Q3T_EINVAL, "kv_write: null pointer");
  if (batch < 1 || heads < 1 || width < 1 || capacity < 1 || heads * width > (1 << 20))
    return fail(Q3T_EINVAL, "kv_write: invalid geometry");
  if (dtype != Q3T_BF16 && dtype != Q3T_F32) return fail(Q3T_EINVAL, "kv_write: dtype must be bf16 or f32");
  const int esz = dtype == Q3T_BF16 ? 2 : 4;
  const int vec = 16 / esz;
  const bool vector = ks[2] == 1 && vs[2] == 1 && width % vec == 0 && ks[0] % vec == 0 && ks[1] % vec == 0 &&
                      vs[0] % vec == 0 && vs[1] % vec == 0 && aligned16(keys) && aligned16(values) &&
                      aligned16(target_keys) && aligned16(target_values);
  const int threads = 128;
  if (esz == 2) {
    using T = uint16_t;
    auto k = vector ? kv_write_kernel<T, true> : kv_write_kernel<T, false>;
    return launch(k, dim3(unsigned(batch)), dim3(threads), 0, stream, true, "kv_write",
                  static_cast<const T*>(keys), ks[0], ks[1], ks[2], static_cast<const T*>(values), vs[0], vs[1],
                  vs[2], static_cast<T*>(target_keys), static_cast<T*>(target_values), positions, int(heads),
                  int(width), capacity, status);
  }
  using T = uint32_t;
  auto k = vector ? kv_write_kernel<T, true> : kv_write_kernel<T, false>;
  return launch(k, dim3(unsigned(batch)), dim3(threads), 0, stream, true, "kv_write", static_cast<const T*>(keys),
                ks[0], ks[1], ks[2], static_cast<const T*>(values), vs[0], vs[1], vs[2],
                static_cast<T*>(target_keys), static_cast<T*>(target_values), positions, int(heads), int(width),
                capacity, status);
}

namespace {
template <typename T>
int launch_strided4(void* dst, const int64_t* ds, const void* src, const int64_t* ss, const int64_t* n,
                    void* stream) {
  const int64_t total = n[0] * n[1] * n[2] * n[3];
  return launch(strided_copy4_kernel<T>, dim3(grid_for(total, 256)), dim3(256), 0, stream, true, "strided_copy",
                static_cast<T*>(dst), ds[0], ds[1], ds[2], ds[3], static_cast<const T*>(src), ss[0], ss[1], ss[2],
                ss[3], n[0], n[1], n[2], n[3]);
}
}  // namespace

extern "C" int q3t_copy_packed_prefix(void* target, const int64_t* tshape, const int64_t* tstr, const void* source,
                                      const int64_t* sshape, const int64_t* sstr, int elem_size, int64_t slot,
                                      int64_t row, int64_t length, void* stream) {
  if (!target || !source || !tshape || !tstr || !sshape || !sstr) return fail(Q3T_EINVAL, "copy_packed_prefix: null");
  for (int i = 0; i < 5; ++i)
    if (tshape[i] <= 0 || sshape[i] <= 0)
      return fail(Q3T_EINVAL, "Expected independent compatible packed KV tensors");
  if (tshape[0] != sshape[0] || tshape[2] != sshape[2] || tshape[4] != sshape[4] || target == source)
    return fail(Q3T_EINVAL, "Expected independent compatible packed KV tensors");
  if (slot < 0 || slot >= tshape[1] || row < 0 || row >= sshape[1] || length <= 0 || length > tshape[3] ||
      length > sshape[3])
    return fail(Q3T_EINVAL, "Expected a valid packed KV row and prefix length");
  if (elem_size != 2 && elem_size != 4 && elem_size != 8) return fail(Q3T_EINVAL, "copy_packed_prefix: elem_size");
  const int64_t n[4] = {tshape[0], tshape[2], length, tshape[4]};
  const int64_t ds[4] = {tstr[0], tstr[2], tstr[3], tstr[4]};
  const int64_t ss[4] = {sstr[0], sstr[2], sstr[3], sstr[4]};
  char* dst = static_cast<char*>(target) + slot * tstr[1] * elem_size;
  const char* src = static_cast<const char*>(source) + row * sstr[1] * elem_size;
  if (elem_size == 2) return launch_strided4<uint16_t>(dst, ds, src, ss, n, stream);
  if (elem_size == 4) return launch_strided4<uint32_t>(dst, ds, src, ss, n, stream);
  return launch_strided4<uint64_t>(dst, ds, src, ss, n, stream);
}

namespace {
// Picks the widest unit (16/8/4/2/1 bytes) that divides all offsets and sizes.
int unit_bytes(const void* base, int64_t a, int64_t b, int64_t c, int64_t d) {
  const uint64_t m = reinterpret_cast<uintptr_t>(base) | uint64_t(a) | uint64_t(b) | uint64_t(c) | uint64_t(d);
  for (int u = 16; u > 1; u >>= 1)
    if ((m & uint64_t(u - 1)) == 0) return u;
  return 1;
}
template <typename T>
int launch_plane_copy(void* base, int64_t planes, int64_t pstride, int64_t elems, int64_t so, int64_t dof,
                      void* stream) {
  return launch(plane_copy_kernel<T>, dim3(grid_for(planes * elems, 256)), dim3(256), 0, stream, true, "slot_move",
                static_cast<T*>(base), planes, pstride, elems, so, dof);
}
template <typename T>
int launch_plane_zero(void* base, int64_t planes, int64_t pstride, int64_t elems, int64_t off, void* stream) {
  return launch(plane_zero_kernel<T>, dim3(grid_for(planes * elems, 256)), dim3(256), 0, stream, true, "slot_zero",
                static_cast<T*>(base), planes, pstride, elems, off);
}
}  // namespace

extern "C" int q3t_slot_move(void* base, int64_t planes, int64_t plane_stride, int64_t slot_stride,
                             int64_t slot_elems, int elem_size, int64_t source, int64_t destination, void* stream) {
  if (!base || planes < 1 || slot_elems < 1 || elem_size < 1 || source < 0 || destination < 0)
    return fail(Q3T_EINVAL, "slot_move: invalid arguments");
  if (source == destination) return Q3T_OK;
  const int64_t pb = plane_stride * elem_size, sb = slot_stride * elem_size, eb = slot_elems * elem_size;
  const int u = unit_bytes(base, pb, sb, eb, 0);
  const int64_t ps = pb / u, so = source * sb / u, dof = destination * sb / u, n = eb / u;
  switch (u) {
    case 16: return launch_plane_copy<uint4>(base, planes, ps, n, so, dof, stream);
    case 8: return launch_plane_copy<uint64_t>(base, planes, ps, n, so, dof, stream);
    case 4: return launch_plane_copy<uint32_t>(base, planes, ps, n, so, dof, stream);
    case 2: return launch_plane_copy<uint16_t>(base, planes, ps, n, so, dof, stream);
    default: return launch_plane_copy<uint8_t>(base, planes, ps, n, so, dof, stream);
  }
}

extern "C" int q3t_slot_zero(void* base, int64_t planes, int64_t plane_stride, int64_t slot_stride,
                             int64_t slot_elems, int elem_size, int64_t start, int64_t count, void* stream) {
  if (!base || planes < 1 || slot_elems < 1 || elem_size < 1 || start < 0 || count < 0)
    return fail(Q3T_EINVAL, "slot_zero: invalid arguments");
  if (count == 0) return Q3T_OK;
  if (count > 1 && slot_stride != slot_elems) {
    for (int64_t s = start; s < start + count; ++s) {
      int rc = q3t_slot_zero(base, planes, plane_stride, slot_stride, slot_elems, elem_size, s, 1, stream);
      if (rc != Q3T_OK) return rc;
    }
    return Q3T_OK;
  }
  const int64_t pb = plane_stride * elem_size, off = start * slot_stride * elem_size,
                eb = slot_elems * count * elem_size;
  const int u = unit_bytes(base, pb, off, eb, 0);
  switch (u) {
    case 16: return launch_plane_zero<uint4>(base, planes, pb / u, eb / u, off / u, stream);
    case 8: return launch_plane_zero<uint64_t>(base, planes, pb / u, eb / u, off / u, stream);
    case 4: return launch_plane_zero<uint32_t>(base, planes, pb / u, eb / u, off / u, stream);
    case 2: return launch_plane_zero<uint16_t>(base, planes, pb / u, eb / u, off / u, stream);
    default: return launch_plane_zero<uint8_t>(base, planes, pb / u, eb / u, off / u, stream);
  }
}

extern "C" int q3t_copy_rows(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t row_bytes,
                             int64_t rows, void* stream) {
  if (!dst || !src || row_bytes < 0 || rows < 0 || dst_pitch < row_bytes || src_pitch < row_bytes)
    return fail(Q3T_EINVAL, "copy_rows: invalid arguments");
  if (rows == 0 || row_bytes == 0) return Q3T_OK;
  const int u = unit_bytes(dst, dst_pitch, src_pitch, row_bytes, reinterpret_cast<uintptr_t>(src));
  const int64_t n = row_bytes / u;
  const dim3 g(grid_for(n * rows, 256));
  char* d = static_cast<char*>(dst);
  const char* s = static_cast<const char*>(src);
  switch (u) {
    case 16: return launch(rows_copy_kernel<uint4>, g, dim3(256), 0, stream, true, "copy_rows", d, dst_pitch, s, src_pitch, n, rows);
    case 8: return launch(rows_copy_kernel<uint64_t>, g, dim3(256), 0, stream, true, "copy_rows", d, dst_pitch, s, src_pitch, n, rows);
    case 4: return launch(rows_copy_kernel<uint32_t>, g, dim3(256), 0, stream, true, "copy_rows", d, dst_pitch, s, src_pitch, n, rows);
    case 2: return launch(rows_copy_kernel<uint16_t>, g, dim3(256), 0, stream, true, "copy_rows", d, dst_pitch, s, src_pitch, n, rows);
    default: return launch(rows_copy_kernel<uint8_t>, g, dim3(256), 0, stream, true, "copy_rows", d, dst_pitch, s, src_pitch, n, rows);
  }
}

extern "C" int q3t_rms_norm(const void* x, int64_t x_stride, const void* weight, void* out, int64_t rows,
                            int64_t width, float eps, int mode, void* stream) {
  if (!x || !weight || !out || rows < 1 || width < 8 || width % 8 || x_stride % 8 || width > 65536)
    return fail(Q3T_EINVAL, "rms_norm: invalid arguments (width multiple of 8)");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out)) return fail(Q3T_EINVAL, "rms_norm: 16-byte alignment");
  if (mode != Q3T_NORM_REFERENCE && mode != Q3T_NORM_NATIVE) return fail(Q3T_EINVAL, "rms_norm: mode");
  int threads = int(width / 8);
  threads = threads > 256 ? 256 : ((threads + 31) / 32) * 32;
  return launch(rms_norm_kernel, dim3(unsigned(rows)), dim3(threads), 0, stream, true, "rms_norm",
                static_cast<const __nv_bfloat16*>(x), x_stride, static_cast<const __nv_bfloat16*>(weight),
                static_cast<__nv_bfloat16*>(out), int(width), eps, mode);
}

extern "C" int q3t_add_rms_norm(const void* a, const void* h, const void* weight, void* normalized,
                                void* residual_out, int64_t rows, int64_t width, float eps, int mode, void* stream) {
  if (!a || !h || !weight || !normalized || !residual_out || rows < 1 || width < 8 || width % 8 || width > 12288)
    return fail(Q3T_EINVAL, "add_rms_norm: invalid arguments");
  if (!aligned16(a) || !aligned16(h) || !aligned16(weight) || !aligned16(normalized) || !aligned16(residual_out))
    return fail(Q3T_EINVAL, "add_rms_norm: 16-byte alignment");
  if (mode != Q3T_NORM_REFERENCE && mode != Q3T_NORM_NATIVE) return fail(Q3T_EINVAL, "add_rms_norm: mode");
  int threads = int(width / 8);
  threads = threads > 256 ? 256 : ((threads + 31) / 32) * 32;
  return launch(add_rms_norm_kernel, dim3(unsigned(rows)), dim3(threads), size_t(width) * 4, stream, true,
                "add_rms_norm", static_cast<const __nv_bfloat16*>(a), static_cast<const __nv_bfloat16*>(h),
                static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(normalized),
                static_cast<__nv_bfloat16*>(residual_out), int(width), eps, mode);
}

extern "C" int q3t_rotary(const void* x, const void* cos, const void* sin, void* out, int64_t batch, int64_t length,
                          int64_t heads, int64_t width, void* stream) {
  if (!x || !cos || !sin || !out) return fail(Q3T_EINVAL, "Expected BF16 BSND input");
  if (heads < 1 || heads > 64 || width < 2 || width % 2 || width > 512 || batch * length < 1)
    return fail(Q3T_EINVAL, "Unsupported rotary shape");
  return launch(rotary_kernel, dim3(unsigned(batch * length)), dim3(128), 0, stream, true, "rotary",
                static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(cos),
                static_cast<const __nv_bfloat16*>(sin), static_cast<__nv_bfloat16*>(out), int(heads), int(width));
}

extern "C" int q3t_swiglu(const void* packed, void* out, int64_t rows, int64_t width, void* stream) {
  if (!packed || !out || rows < 1 || width < 8 || width % 8) return fail(Q3T_EINVAL, "swiglu: invalid arguments");
  if (!aligned16(packed) || !aligned16(out)) return fail(Q3T_EINVAL, "swiglu: 16-byte alignment");
  return launch(swiglu_kernel, dim3(grid_for(rows * width / 8, 256)), dim3(256), 0, stream, true, "swiglu",
                static_cast<const __nv_bfloat16*>(packed), static_cast<__nv_bfloat16*>(out), rows, width);
}

extern "C" int q3t_snake(const void* x, const void* alpha, const void* inverse_beta, void* out, int64_t batch,
                         int64_t channels, int64_t length, int dtype, int coef_dtype, void* stream) {
  if (!x || !alpha || !inverse_beta || !out || batch < 1 || channels < 1 || length < 1)
    return fail(Q3T_EINVAL, "Snake requires nonempty NCT input and per-channel coefficients");
  const int64_t total = batch * channels * length;
  const dim3 g(grid_for(total, 256));
  if (dtype == Q3T_BF16 && coef_dtype == Q3T_F32)
    return launch(snake_kernel<__nv_bfloat16, float>, g, dim3(256), 0, stream, true, "snake",
                  static_cast<const __nv_bfloat16*>(x), static_cast<const float*>(alpha),
                  static_cast<const float*>(inverse_beta), static_cast<__nv_bfloat16*>(out), channels, length, total);
  if (dtype == Q3T_BF16 && coef_dtype == Q3T_BF16)
    return launch(snake_kernel<__nv_bfloat16, __nv_bfloat16>, g, dim3(256), 0, stream, true, "snake",
                  static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(alpha),
                  static_cast<const __nv_bfloat16*>(inverse_beta), static_cast<__nv_bfloat16*>(out), channels, length,
                  total);
  if (dtype == Q3T_F32 && coef_dtype == Q3T_F32)
    return launch(snake_kernel<float, float>, g, dim3(256), 0, stream, true, "snake", static_cast<const float*>(x),
                  static_cast<const float*>(alpha), static_cast<const float*>(inverse_beta), static_cast<float*>(out),
                  channels, length, total);
  return fail(Q3T_EINVAL, "snake: unsupported dtype combination");
}

extern "C" int q3t_scatter_rows(void* target, int64_t target_rows, const int64_t* indices, const void* source,
                                int ndim, const int64_t* shape, const int64_t* strides, int elem_size,
                                unsigned* status, void* stream) {
  if (!target || !indices || !source || !shape || !strides || ndim < 1 || ndim > 4 || target_rows < 1)
    return fail(Q3T_EINVAL, "Expected independent source and contiguous selected-row target");
  int64_t e[4] = {1, 1, 1, 1}, s[4] = {0, 0, 0, 0};
  for (int i = 0; i < ndim; ++i) {
    if (shape[i] < 1) return fail(Q3T_EINVAL, "scatter_rows: empty source");
    e[i] = shape[i];
    s[i] = strides[i];
  }
  const int64_t total = e[0] * e[1] * e[2] * e[3];
  const dim3 g(grid_for(total, 256));
  switch (elem_size) {
    case 2:
      return launch(scatter_rows_kernel<uint16_t>, g, dim3(256), 0, stream, true, "scatter_rows",
                    static_cast<uint16_t*>(target), target_rows, indices, static_cast<const uint16_t*>(source), e[0],
                    e[1], e[2], e[3], s[0], s[1], s[2], s[3], status);
    case 4:
      return launch(scatter_rows_kernel<uint32_t>, g, dim3(256), 0, stream, true, "scatter_rows",
                    static_cast<uint32_t*>(target), target_rows, indices, static_cast<const uint32_t*>(source), e[0],
                    e[1], e[2], e[3], s[0], s[1], s[2], s[3], status);
    case 8:
      return launch(scatter_rows_kernel<uint64_t>, g, dim3(256), 0, stream, true, "scatter_rows",
                    static_cast<uint64_t*>(target), target_rows, indices, static_cast<const uint64_t*>(source), e[0],
                    e[1], e[2], e[3], s[0], s[1], s[2], s[3], status);
    default: return fail(Q3T_EINVAL, "scatter_rows: elem_size must be 2, 4 or 8");
  }
}

extern "C" int q3t_embedding(const int64_t* ids, int64_t ids_stride, const void* table, int64_t vocab, void* out,
                             int64_t out_stride, int64_t rows, int64_t hidden, unsigned* status, void* stream) {
  if (!ids || !table || !out || rows < 1 || vocab < 1 || hidden < 8 || hidden % 8 || out_stride % 8)
    return fail(Q3T_EINVAL, "embedding: invalid arguments");
  if (!aligned16(table) || !aligned16(out)) return fail(Q3T_EINVAL, "embedding: 16-byte alignment");
  int threads = int(hidden / 8);
  threads = threads > 256 ? 256 : ((threads + 31) / 32) * 32;
  return launch(embedding_kernel, dim3(unsigned(rows)), dim3(threads), 0, stream, true, "embedding", ids, ids_stride,
                static_cast<const __nv_bfloat16*>(table), vocab, static_cast<__nv_bfloat16*>(out), out_stride,
                int(hidden), status);
}

extern "C" int q3t_frame_embed(const int64_t* codes, int64_t codes_stride, const void* first_table,
                               int64_t first_vocab, const void* group_tables, int64_t groups, int64_t group_vocab,
                               const void* text, int64_t text_stride, void* out, int64_t batch, int64_t hidden,
                               unsigned* status, void* stream) {
  if (!codes || !first_table || !group_tables || !out || batch < 1 || hidden < 8 || hidden % 8 || groups < 0 ||
      groups > 31 || first_vocab < 1 || group_vocab < 1)
    return fail(Q3T_EINVAL, "frame_embed: invalid arguments");
  if (!aligned16(first_table) || !aligned16(group_tables) || !aligned16(out) || (text && !aligned16(text)) ||
      text_stride % 8)
    return fail(Q3T_EINVAL, "frame_embed: 16-byte alignment");
  int threads = int(hidden / 8);
  threads = threads > 256 ? 256 : ((threads + 31) / 32) * 32;
  if (threads < 32) threads = 32;
  return launch(frame_embed_kernel, dim3(unsigned(batch)), dim3(threads), 0, stream, true, "frame_embed", codes,
                codes_stride, static_cast<const __nv_bfloat16*>(first_table), first_vocab,
                static_cast<const __nv_bfloat16*>(group_tables), int(groups), group_vocab,
                static_cast<const __nv_bfloat16*>(text), text_stride, static_cast<__nv_bfloat16*>(out), int(hidden),
                status);
}

extern "C" int q3t_advance(int64_t* values, int64_t count, int64_t delta, void* stream) {
  if (!values || count < 1) return fail(Q3T_EINVAL, "advance: invalid arguments");
  return launch(advance_kernel, dim3(grid_for(count, 256)), dim3(256), 0, stream, true, "advance", values, count,
                delta);
}
