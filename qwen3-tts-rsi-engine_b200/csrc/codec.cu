// Incremental codec kernels: RVQ dequantisation, causal-conv im2col with
// per-slot history (and the SnakeBeta activation fused into the gather),
// history updates, depthwise conv + LayerNorm of the ConvNeXt blocks,
// codec frame positions and on-device PCM16 conversion.
//
// Codec activations are time-major [batch, time, channels] bf16, i.e. the
// row layout of the tcgen05 GEMM: a causal conv (kernel k, dilation d) is
// gather -> GEMM with K ordered (tap, channel); a transposed conv of kernel
// 2r and stride r is ONE GEMM over [x[t] | x[t-1]] whose r*C_out outputs per
// input frame are already the upsampled sequence in time-major order.
// Streams are addressed through a slot table, so per-request state (conv
// histories, frame counters) stays in place (codec_slots.py:15-39).
#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

int grid_for(int64_t total, int threads) {
  const int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = int64_t(sm_count()) * 16;
  return int(blocks < 1 ? 1 : (blocks > cap ? cap : blocks));
}

// ------------------------------------------------------------------ RVQ (cached_quantizer.py:17-30)
// out[row] = [ sum_{q < semantic} table_q[code_q] | sum_{q >= semantic} table_q[code_q] ]
// (fp32 sums in codebook order, one rounding each); the caller applies
// [W_first | W_rest] as one GEMM.
__global__ void rvq_gather_kernel(const int64_t* __restrict__ codes, int64_t cb_stride, int64_t t_stride,
                                  int64_t b_stride, const __nv_bfloat16* __restrict__ tables, int codebooks,
                                  int semantic, int64_t bins, int dim, int T, __nv_bfloat16* __restrict__ out,
                                  unsigned* status) {
  grid_dependency_wait();
  const int64_t row = blockIdx.x;  // b * T + t
  const int64_t b = row / T, t = row % T;
  for (int c = threadIdx.x * 8; c < dim; c += blockDim.x * 8) {
    float sem[8] = {0, 0, 0, 0, 0, 0, 0, 0}, rest[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int q = 0; q < codebooks; ++q) {
      int64_t code = codes[b * b_stride + q * cb_stride + t * t_stride];
      if (code < 0 || code >= bins) {
        if (c == threadIdx.x * 8) raise_status(status, kStatusBadIndex);
        continue;
      }
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(tables + (int64_t(q) * bins + code) * dim + c), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (q < semantic) sem[j] += f[j];
        else rest[j] += f[j];
      }
    }
    *reinterpret_cast<uint4*>(out + row * 2 * dim + c) = pack8(sem);
    *reinterpret_cast<uint4*>(out + row * 2 * dim + dim + c) = pack8(rest);
  }
}

// ------------------------------------------------------------------ im2col with history and Snake
// col[(b,t), j*C + c] = f(src(b, t - shift_j, c)); shift_j = (taps-1-j)*d (causal conv) or
// j*d (reverse: [x[t], x[t-1], ...] for transposed convs). Negative times read the
// slot's history [slots, H, C] at H + t'.
__global__ void conv_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T, int C,
                                   const __nv_bfloat16* __restrict__ hist, int H, const int64_t* __restrict__ slots,
                                   int taps, int dilation, int reverse, const float* __restrict__ alpha,
                                   const float* __restrict__ inv, __nv_bfloat16* __restrict__ col, int64_t rows) {
  grid_dependency_wait();
  const int cv = C / 8;
  const int64_t total = rows * taps * cv;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int c = int(i % cv) * 8;
    const int64_t rj = i / cv;
    const int j = int(rj % taps);
    const int64_t row = rj / taps;
    const int64_t b = row / T;
    const int t = int(row % T);
    const int shift = reverse ? j * dilation : (taps - 1 - j) * dilation;
    const int ts = t - shift;
    uint4 raw;
    if (ts >= 0) {
      raw = *reinterpret_cast<const uint4*>(x + (b * T + ts) * x_stride + c);
    } else if (hist != nullptr && H + ts >= 0) {
      const int64_t slot = slots ? slots[b] : b;
      raw = *reinterpret_cast<const uint4*>(hist + (slot * H + (H + ts)) * int64_t(C) + c);
    } else {
      raw = make_uint4(0, 0, 0, 0);
    }
    if (alpha != nullptr) {
      float f[8];
      unpack8(raw, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = snake_bf16(f[k], alpha[c + k], inv[c + k]);
      raw = pack8(f);
    }
    *reinterpret_cast<uint4*>(col + row * int64_t(taps) * C + int64_t(j) * C + c) = raw;
  }
}

// Padded input of an implicit causal conv (q3t_conv_linear):
// xs[b, p, c] = f(seq_b[p]), seq_b = [history[slot_b] (H frames) | x[b*T .. b*T + T)],
// f = SnakeBeta (alpha != null) or identity; one thread per (row, 8 channels).
__global__ void conv_pad_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int T, int C,
                                const __nv_bfloat16* __restrict__ hist, int H, const int64_t* __restrict__ slots,
                                const float* __restrict__ alpha, const float* __restrict__ inv,
                                __nv_bfloat16* __restrict__ xs, int64_t rows) {
  grid_dependency_wait();
  const int cv = C / 8;
  const int64_t total = rows * cv;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int c = int(i % cv) * 8;
    const int64_t row = i / cv;
    const int64_t b = row / (H + T);
    const int p = int(row % (H + T));
    uint4 raw;
    if (p >= H) {
      raw = *reinterpret_cast<const uint4*>(x + (b * T + (p - H)) * x_stride + c);
    } else if (hist != nullptr) {
      const int64_t slot = slots ? slots[b] : b;
      raw = *reinterpret_cast<const uint4*>(hist + (slot * H + p) * int64_t(C) + c);
    } else {
      raw = make_uint4(0, 0, 0, 0);
    }
    if (alpha != nullptr) {
      float f[8];
      unpack8(raw, f);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] = snake_bf16(f[k], alpha[c + k], inv[c + k]);
      raw = pack8(f);
    }
    *reinterpret_cast<uint4*>(xs + row * int64_t(C) + c) = raw;
  }
}

// new history = last H frames of [old history | x]. With T >= H every new frame comes from
// x: one thread per (stream, frame, 8 channels). Otherwise one thread per (stream, 8 channels)
// walks the frames in ascending order, so the in-place shift reads before it overwrites.
__global__ void conv_history_kernel(const __nv_bfloat16* __restrict__ x, int64_t x_stride, int B, int T, int C,
                                    __nv_bfloat16* __restrict__ hist, int H, const int64_t* __restrict__ slots) {
  grid_dependency_wait();
  const int cv = C / 8;
  if (T >= H) {
    const int64_t total = int64_t(B) * H * cv;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total;
         i += int64_t(gridDim.x) * blockDim.x) {
      const int c = int(i % cv) * 8;
      const int64_t bk = i / cv;
      const int64_t b = bk / H;
      const int k = int(bk % H);
      const int64_t slot = slots ? slots[b] : b;
      *reinterpret_cast<uint4*>(hist + (slot * H + k) * int64_t(C) + c) =
          *reinterpret_cast<const uint4*>(x + (b * T + (T - H + k)) * x_stride + c);
    }
    return;
  }
  const int64_t total = int64_t(B) * cv;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = i / cv;
    const int c = int(i % cv) * 8;
    const int64_t slot = slots ? slots[b] : b;
    __nv_bfloat16* h = hist + slot * H * int64_t(C) + c;
    for (int k = 0; k < H; ++k) {
      const int src = k + T;  // position in [old history (H) | x (T)]
      uint4 v;
      if (src < H)
        v = *reinterpret_cast<const uint4*>(h + int64_t(src) * C);
      else
        v = *reinterpret_cast<const uint4*>(x + (b * T + (src - H)) * x_stride + c);
      *reinterpret_cast<uint4*>(h + int64_t(k) * C) = v;
    }
  }
}

// ------------------------------------------------------------------ ConvNeXt depthwise conv + LayerNorm
// y_c = bias_c + sum_j w[c, j] x(t - 6 + j, c) (kernel 7, causal, history 6), rounded to bf16,
// then LayerNorm over channels (fp32 statistics) -> bf16 (incremental_codec.py:80-84).
__global__ void dwconv_layernorm_kernel(const __nv_bfloat16* __restrict__ x, int T, int C,
                                        const __nv_bfloat16* __restrict__ hist, int H,
                                        const int64_t* __restrict__ slots, const float* __restrict__ w,
                                        const float* __restrict__ bias, const float* __restrict__ ln_w,
                                        const float* __restrict__ ln_b, float eps, __nv_bfloat16* __restrict__ out) {
  extern __shared__ float y[];  // C floats
  __shared__ float red[64];
  grid_dependency_wait();
  const int64_t row = blockIdx.x;
  const int64_t b = row / T;
  const int t = int(row % T);
  const int64_t slot = slots ? slots[b] : b;
  float s = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    float acc = bias[c];
#pragma unroll
    for (int j = 0; j < 7; ++j) {
      const int ts = t - 6 + j;
      float v = 0.f;
      if (ts >= 0)
        v = __bfloat162float(x[(b * T + ts) * int64_t(C) + c]);
      else if (H + ts >= 0)
        v = __bfloat162float(hist[(slot * H + (H + ts)) * int64_t(C) + c]);
      acc = fmaf(w[c * 7 + j], v, acc);
    }
    acc = bf16r(acc);
    y[c] = acc;
    s += acc;
  }
  s = warp_sum(s);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[warp] = s;
  __syncthreads();
  float mean = 0.f;
  for (int k = 0; k < nw; ++k) mean += red[k];
  mean /= float(C);
  __syncthreads();
  float v2 = 0.f;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    const float d = y[c] - mean;
    v2 += d * d;
  }
  v2 = warp_sum(v2);
  if (lane == 0) red[32 + warp] = v2;
  __syncthreads();
  float var = 0.f;
  for (int k = 0; k < nw; ++k) var += red[32 + k];
  var /= float(C);
  const float r = 1.0f / sqrtf(var + eps);
  for (int c = threadIdx.x; c < C; c += blockDim.x)
    out[row * int64_t(C) + c] = __float2bfloat16_rn((y[c] - mean) * r * ln_w[c] + ln_b[c]);
}

// ------------------------------------------------------------------ frame positions (codec_slots.py:70-72, 98)
// rows (b, t): rotary position frames[slot_b] + t, cache row (frames[slot_b] + t) % ring;
// then frames[slot_b] += T (one thread per stream reads then writes its counter).
__global__ void codec_positions_kernel(int64_t* __restrict__ frames, const int64_t* __restrict__ slots, int B, int T,
                                       int64_t ring, int64_t* __restrict__ rot, int64_t* __restrict__ cache,
                                       int advance) {
  grid_dependency_wait();
  for (int b = blockIdx.x * blockDim.x + threadIdx.x; b < B; b += gridDim.x * blockDim.x) {
    const int64_t slot = slots ? slots[b] : b;
    const int64_t f = frames[slot];
    for (int t = 0; t < T; ++t) {
      rot[int64_t(b) * T + t] = f + t;
      cache[int64_t(b) * T + t] = ring > 0 ? (f + t) % ring : f + t;
    }
    if (advance) frames[slot] = f + T;
  }
}

// ------------------------------------------------------------------ PCM16 (continuous.py:535)
// pcm = int16(clip(x, -1, 1) * 32767) (truncation toward zero); wave = clip(x, -1, 1).
__global__ void pcm16_kernel(const __nv_bfloat16* __restrict__ x, int64_t n, float* __restrict__ wave,
                             int16_t* __restrict__ pcm, unsigned* status) {
  grid_dependency_wait();
  bool finite = true;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
    const float raw = __bfloat162float(x[i]);
    finite = finite && isfinite(raw);
    const float v = fminf(fmaxf(raw, -1.0f), 1.0f);
    if (wave) wave[i] = v;
    if (pcm) pcm[i] = int16_t(v * 32767.0f);
  }
  if (__any_sync(0xffffffffu, !finite) && (threadIdx.x & 31) == 0) raise_status(status, kStatusNonFinite);
}

}  // namespace

extern "C" int q3t_rvq_gather(const int64_t* codes, int64_t b_stride, int64_t cb_stride, int64_t t_stride,
                              const void* tables, int64_t codebooks, int64_t semantic, int64_t bins, int64_t dim,
                              int64_t batch, int64_t frames, void* out, unsigned* status, void* stream) {
  if (!codes || !tables || !out || batch < 1 || frames < 1 || codebooks < 1 || semantic < 0 || semantic > codebooks ||
      bins < 1 || dim < 8 || dim % 8)
    return fail(Q3T_EINVAL, "rvq_gather: invalid arguments");
  if (!aligned16(tables) || !aligned16(out)) return fail(Q3T_EINVAL, "rvq_gather: 16-byte alignment");
  int threads = int(dim / 8);
  threads = threads > 128 ? 128 : ((threads + 31) / 32) * 32;
  return launch(rvq_gather_kernel, dim3(unsigned(batch * frames)), dim3(threads), 0, stream, true, "rvq_gather", codes,
                cb_stride, t_stride, b_stride, static_cast<const __nv_bfloat16*>(tables), int(codebooks),
                int(semantic), bins, int(dim), int(frames), static_cast<__nv_bfloat16*>(out), status);
}

extern "C" int q3t_conv_gather(const void* x, int64_t x_stride, int64_t batch, int64_t frames, int64_t channels,
                               const void* history, int64_t history_len, const int64_t* slots, int64_t taps,
                               int64_t dilation, int reverse, const float* alpha, const float* inverse_beta,
                               void* col, void* stream) {
  if (!x || !col || batch < 1 || frames < 1 || channels < 8 || channels % 8 || taps < 1 || dilation < 1 ||
      x_stride % 8 || history_len < 0 || (history_len > 0 && !history) || ((alpha == nullptr) != (inverse_beta == nullptr)))
    return fail(Q3T_EINVAL, "conv_gather: invalid arguments");
  if ((taps - 1) * dilation > history_len && history != nullptr)
    return fail(Q3T_EINVAL, "conv_gather: history shorter than the receptive field");
  if (!aligned16(x) || !aligned16(col) || (history && !aligned16(history)))
    return fail(Q3T_EINVAL, "conv_gather: 16-byte alignment");
  const int64_t rows = batch * frames;
  return launch(conv_gather_kernel, dim3(grid_for(rows * taps * (channels / 8), 256)), dim3(256), 0, stream, true,
                "conv_gather", static_cast<const __nv_bfloat16*>(x), x_stride, int(frames), int(channels),
                static_cast<const __nv_bfloat16*>(history), int(history_len), slots, int(taps), int(dilation),
                reverse, alpha, inverse_beta, static_cast<__nv_bfloat16*>(col), rows);
}

extern "C" int q3t_conv_pad(const void* x, int64_t x_stride, int64_t batch, int64_t frames, int64_t channels,
                            const void* history, int64_t history_len, const int64_t* slots, const float* alpha,
                            const float* inverse_beta, void* xs, void* stream) {
  if (!x || !xs || batch < 1 || frames < 1 || channels < 8 || channels % 8 || x_stride % 8 || x_stride < channels ||
      history_len < 0 || ((alpha == nullptr) != (inverse_beta == nullptr)))
    return fail(Q3T_EINVAL, "conv_pad: invalid arguments");
  if (!aligned16(x) || !aligned16(xs) || (history && !aligned16(history)))
    return fail(Q3T_EINVAL, "conv_pad: 16-byte alignment");
  const int64_t rows = batch * (history_len + frames);
  return launch(conv_pad_kernel, dim3(grid_for(rows * (channels / 8), 256)), dim3(256), 0, stream, true, "conv_pad",
                static_cast<const __nv_bfloat16*>(x), x_stride, int(frames), int(channels),
                static_cast<const __nv_bfloat16*>(history), int(history_len), slots, alpha, inverse_beta,
                static_cast<__nv_bfloat16*>(xs), rows);
}

extern "C" int q3t_conv_history(const void* x, int64_t x_stride, int64_t batch, int64_t frames, int64_t channels,
                                void* history, int64_t history_len, const int64_t* slots, void* stream) {
  if (!x || !history || batch < 1 || frames < 1 || channels < 8 || channels % 8 || history_len < 1 || x_stride % 8)
    return fail(Q3T_EINVAL, "conv_history: invalid arguments");
  const int64_t work = frames >= history_len ? batch * history_len * (channels / 8) : batch * (channels / 8);
  return launch(conv_history_kernel, dim3(grid_for(work, 128)), dim3(128), 0, stream, true,
                "conv_history", static_cast<const __nv_bfloat16*>(x), x_stride, int(batch), int(frames),
                int(channels), static_cast<__nv_bfloat16*>(history), int(history_len), slots);
}

extern "C" int q3t_dwconv_layernorm(const void* x, int64_t batch, int64_t frames, int64_t channels,
                                    const void* history, int64_t history_len, const int64_t* slots,
                                    const float* weight, const float* bias, const float* ln_weight,
                                    const float* ln_bias, float eps, void* out, void* stream) {
  if (!x || !weight || !bias || !ln_weight || !ln_bias || !out || batch < 1 || frames < 1 || channels < 1 ||
      channels > 16384 || (history_len > 0 && !history))
    return fail(Q3T_EINVAL, "dwconv_layernorm: invalid arguments");
  return launch(dwconv_layernorm_kernel, dim3(unsigned(batch * frames)), dim3(256), size_t(channels) * 4, stream,
                true, "dwconv_layernorm", static_cast<const __nv_bfloat16*>(x), int(frames), int(channels),
                static_cast<const __nv_bfloat16*>(history), int(history_len), slots, weight, bias, ln_weight, ln_bias,
                eps, static_cast<__nv_bfloat16*>(out));
}

extern "C" int q3t_codec_positions(int64_t* frames_by_slot, const int64_t* slots, int64_t batch, int64_t frames,
                                   int64_t ring, int64_t* rotary_positions, int64_t* cache_positions, int advance,
                                   void* stream) {
  if (!frames_by_slot || !rotary_positions || !cache_positions || batch < 1 || frames < 1 || ring < 0)
    return fail(Q3T_EINVAL, "codec_positions: invalid arguments");
  return launch(codec_positions_kernel, dim3(1), dim3(128), 0, stream, true, "codec_positions", frames_by_slot, slots,
                int(batch), int(frames), ring, rotary_positions, cache_positions, advance);
}

extern "C" int q3t_pcm16(const void* x, int64_t count, float* wave, int16_t* pcm, unsigned* status, void* stream) {
  if (!x || count < 1 || (!wave && !pcm)) return fail(Q3T_EINVAL, "pcm16: invalid arguments");
  return launch(pcm16_kernel, dim3(grid_for(count, 256)), dim3(256), 0, stream, true, "pcm16",
                static_cast<const __nv_bfloat16*>(x), count, wave, pcm, status);
}
