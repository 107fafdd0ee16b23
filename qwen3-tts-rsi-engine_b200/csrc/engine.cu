// Per-tick slot bookkeeping of the continuous-batching engine, on the device.
//
// The reference keeps every request's decode state in a Python RequestState
// (continuous.py:232-247) and assembles each tick's inputs with torch.cat /
// torch.stack over the active states (continuous.py:575-606), then writes the
// results back one state at a time (continuous.py:620-640). Here that state is
// dense device arrays indexed by slot (slot i = the i-th active request), so
// the whole tick replays as one CUDA graph:
//
//   tick_gather  : state arrays -> the predictor/talker step inputs
//   (predictor chain, talker step, semantic sampling: other kernels)
//   tick_commit  : step outputs -> state arrays (code ring, hidden, counters)
//
// Rows at or beyond the device scalar `*active` are graph padding and get the
// reference's padding values (token 0, zero hidden/text, draws 0.5,
// position 0; continuous.py:580-583, 599-604); tick_commit leaves them alone.
//
// The code ring is CodecCodeBuffer (codec_code_buffer.py:5-31) with a
// configurable depth: frame f of slot s lives in row s * depth + f % depth.

#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"
#include "host.cuh"

using namespace q3t;

namespace {

constexpr int kDraws = 16;

__device__ __forceinline__ void copy_row_bf16(__nv_bfloat16* dst, const __nv_bfloat16* src, int hidden, bool zero) {
  for (int i = threadIdx.x * 8; i < hidden; i += blockDim.x * 8) {
    uint4 v = make_uint4(0, 0, 0, 0);
    if (!zero) v = *reinterpret_cast<const uint4*>(src + i);
    *reinterpret_cast<uint4*>(dst + i) = v;
  }
}

__global__ void tick_gather_kernel(const int64_t* __restrict__ active, const int64_t* __restrict__ tokens,
                                   const __nv_bfloat16* __restrict__ hidden_state,
                                   const __nv_bfloat16* __restrict__ codec_embedding, int64_t vocab,
                                   const float* __restrict__ tables, int64_t table_rows,
                                   const int64_t* __restrict__ frames, const __nv_bfloat16* __restrict__ trailing,
                                   int64_t trailing_rows, const int64_t* __restrict__ trailing_len,
                                   const __nv_bfloat16* __restrict__ pad, const int64_t* __restrict__ positions,
                                   const int64_t* __restrict__ rotary, __nv_bfloat16* __restrict__ pred_inputs,
                                   int64_t* __restrict__ codes, int64_t codes_stride, float* __restrict__ draws,
                                   float* __restrict__ talker_uniform, int64_t* __restrict__ steps,
                                   __nv_bfloat16* __restrict__ text, int64_t* __restrict__ step_positions,
                                   int64_t* __restrict__ step_rotary, int hidden, unsigned* status) {
  grid_dependency_wait();
  const int64_t b = blockIdx.x;
  const bool live = b < *active;
  int64_t token = live ? tokens[b] : 0;
  int64_t frame = live ? frames[b] : 0;
  bool ok = token >= 0 && token < vocab && frame >= 0 && frame + 1 < table_rows;
  if (!ok) {
    if (threadIdx.x == 0) raise_status(status, kStatusBadIndex);
    token = 0;
    frame = 0;
  }
  __nv_bfloat16* in = pred_inputs + b * 2 * hidden;
  copy_row_bf16(in, hidden_state + b * hidden, hidden, !live);
  copy_row_bf16(in + hidden, codec_embedding + token * hidden, hidden, false);
  const int64_t tlen = live ? trailing_len[b] : 0;
  const bool from_trailing = live && frame < tlen && frame < trailing_rows;
  copy_row_bf16(text + b * hidden, from_trailing ? trailing + (b * trailing_rows + frame) * hidden : pad + b * hidden,
                hidden, !live);
  const float* row = tables + (b * table_rows + frame) * kDraws;
  if (threadIdx.x < kDraws) draws[b * kDraws + threadIdx.x] = live ? row[threadIdx.x] : 0.5f;
  if (threadIdx.x == 0) {
    talker_uniform[b] = live ? row[kDraws] : 0.5f;   // column 0 of the next frame's row
    steps[b] = live ? frame + 1 : 0;
    codes[b * codes_stride] = token;
    step_positions[b] = live ? positions[b] : 0;
    step_rotary[b] = live ? rotary[b] : 0;
  }
}

__global__ void tick_commit_kernel(const int64_t* __restrict__ active, const int64_t* __restrict__ codes,
                                   int64_t codes_stride, int codebooks, const __nv_bfloat16* __restrict__ step_hidden,
                                   __nv_bfloat16* __restrict__ hidden_state, int64_t* __restrict__ ring,
                                   int64_t ring_depth, int64_t* __restrict__ frames, int64_t* __restrict__ positions,
                                   int64_t* __restrict__ rotary, int hidden) {
  grid_dependency_wait();
  const int64_t b = blockIdx.x;
  if (b >= *active) return;
  const int64_t frame = frames[b];
  int64_t* dst = ring + (b * ring_depth + (frame % ring_depth)) * codebooks;
  for (int c = threadIdx.x; c < codebooks; c += blockDim.x) dst[c] = codes[b * codes_stride + c];
  copy_row_bf16(hidden_state + b * hidden, step_hidden + b * hidden, hidden, false);
  __syncthreads();   // every thread has read frames[b] before it advances
  if (threadIdx.x == 0) {
    frames[b] = frame + 1;
    positions[b] += 1;
    rotary[b] += 1;
  }
}

__global__ void ring_write_kernel(const int64_t* __restrict__ codes, int64_t codes_stride,
                                  const int64_t* __restrict__ frame_indices, int64_t* __restrict__ ring,
                                  int64_t ring_depth, int codebooks) {
  grid_dependency_wait();
  const int64_t b = blockIdx.x;
  const int64_t f = frame_indices[b];
  const int64_t row = ((f % ring_depth) + ring_depth) % ring_depth;
  for (int c = threadIdx.x; c < codebooks; c += blockDim.x)
    ring[(b * ring_depth + row) * codebooks + c] = codes[b * codes_stride + c];
}

// out[i, c, t] = ring[slots[i], (starts[i] + t) % depth, c]
__global__ void ring_read_kernel(const int64_t* __restrict__ ring, int64_t slots, int64_t ring_depth, int codebooks,
                                 const int64_t* __restrict__ indices, const int64_t* __restrict__ starts,
                                 int64_t length, int64_t* __restrict__ out, unsigned* status) {
  grid_dependency_wait();
  const int64_t i = blockIdx.x;
  const int64_t slot = indices[i];
  const int64_t start = starts[i];
  const bool ok = slot >= 0 && slot < slots && start >= 0;
  if (!ok && threadIdx.x == 0) raise_status(status, kStatusBadIndex);
  for (int64_t e = threadIdx.x; e < codebooks * length; e += blockDim.x) {
    const int64_t c = e / length, t = e % length;
    out[(i * codebooks + c) * length + t] =
        ok ? ring[(slot * ring_depth + (start + t) % ring_depth) * codebooks + c] : int64_t(0);
  }
}

}  // namespace

extern "C" int q3t_tick_gather(const int64_t* active, const int64_t* tokens, const void* hidden_state,
                               const void* codec_embedding, int64_t vocab, const float* tables, int64_t table_rows,
                               const int64_t* frames, const void* trailing, int64_t trailing_rows,
                               const int64_t* trailing_len, const void* pad, const int64_t* positions,
                               const int64_t* rotary, void* pred_inputs, int64_t* codes, int64_t codes_stride,
                               float* draws, float* talker_uniform, int64_t* steps, void* text,
                               int64_t* step_positions, int64_t* step_rotary, int64_t rows, int64_t hidden,
                               unsigned* status, void* stream) {
  if (!active || !tokens || !hidden_state || !codec_embedding || !tables || !frames || !trailing || !trailing_len ||
      !pad || !positions || !rotary || !pred_inputs || !codes || !draws || !talker_uniform || !steps || !text ||
      !step_positions || !step_rotary)
    return fail(Q3T_EINVAL, "tick_gather: null pointer");
  if (rows < 1 || rows > 65535 || hidden < 8 || hidden % 8 || vocab < 1 || table_rows < 2 || trailing_rows < 1 ||
      codes_stride < 1)
    return fail(Q3T_EINVAL, "tick_gather: invalid sizes");
  if (!aligned16(hidden_state) || !aligned16(codec_embedding) || !aligned16(trailing) || !aligned16(pad) ||
      !aligned16(pred_inputs) || !aligned16(text))
    return fail(Q3T_EINVAL, "tick_gather: 16-byte alignment");
  int threads = int(hidden / 8);
  threads = threads > 256 ? 256 : ((threads + 31) / 32) * 32;
  if (threads < 32) threads = 32;
  return launch(tick_gather_kernel, dim3(unsigned(rows)), dim3(threads), 0, stream, true, "tick_gather", active,
                tokens, static_cast<const __nv_bfloat16*>(hidden_state),
                static_cast<const __nv_bfloat16*>(codec_embedding), vocab, tables, table_rows, frames,
                static_cast<const __nv_bfloat16*>(trailing), trailing_rows, trailing_len,
                static_cast<const __nv_bfloat16*>(pad), positions, rotary, static_cast<__nv_bfloat16*>(pred_inputs),
                codes, codes_stride, draws, talker_uniform, steps, static_cast<__nv_bfloat16*>(text), step_positions,
                step_rotary, int(hidden), status);
}

extern "C" int q3t_tick_commit(const int64_t* active, const int64_t* codes, int64_t codes_stride, int64_t codebooks,
                               const void* step_hidden, void* hidden_state, int64_t* ring, int64_t ring_depth,
                               int64_t* frames, int64_t* positions, int64_t* rotary, int64_t rows, int64_t hidden,
                               void* stream) {
  if (!active || !codes || !step_hidden || !hidden_state || !ring || !frames || !positions || !rotary)
    return fail(Q3T_EINVAL, "tick_commit: null pointer");
  if (rows < 1 || rows > 65535 || hidden < 8 || hidden % 8 || codebooks < 1 || codebooks > 256 || ring_depth < 1 ||
      codes_stride < codebooks)
    return fail(Q3T_EINVAL, "tick_commit: invalid sizes");
  if (!aligned16(step_hidden) || !aligned16(hidden_state)) return fail(Q3T_EINVAL, "tick_commit: 16-byte alignment");
  int threads = int(hidden / 8);
  threads = threads > 256 ? 256 : ((threads + 31) / 32) * 32;
  if (threads < 32) threads = 32;
  return launch(tick_commit_kernel, dim3(unsigned(rows)), dim3(threads), 0, stream, true, "tick_commit", active,
                codes, codes_stride, int(codebooks), static_cast<const __nv_bfloat16*>(step_hidden),
                static_cast<__nv_bfloat16*>(hidden_state), ring, ring_depth, frames, positions, rotary, int(hidden));
}

extern "C" int q3t_code_ring_write(const int64_t* codes, int64_t codes_stride, const int64_t* frame_indices,
                                   int64_t* ring, int64_t ring_depth, int64_t codebooks, int64_t count,
                                   void* stream) {
  if (!codes || !frame_indices || !ring) return fail(Q3T_EINVAL, "code_ring_write: null pointer");
  if (count < 1 || count > 65535 || ring_depth < 1 || codebooks < 1 || codes_stride < codebooks)
    return fail(Q3T_EINVAL, "code_ring_write: invalid sizes");
  return launch(ring_write_kernel, dim3(unsigned(count)), dim3(32), 0, stream, true, "code_ring_write", codes,
                codes_stride, frame_indices, ring, ring_depth, int(codebooks));
}

extern "C" int q3t_code_ring_read(const int64_t* ring, int64_t slots, int64_t ring_depth, int64_t codebooks,
                                  const int64_t* indices, const int64_t* starts, int64_t batch, int64_t length,
                                  int64_t* out, unsigned* status, void* stream) {
  if (!ring || !indices || !starts || !out) return fail(Q3T_EINVAL, "code_ring_read: null pointer");
  if (batch < 1 || batch > 65535 || slots < 1 || codebooks < 1 || length < 1 || length > ring_depth)
    return fail(Q3T_EINVAL, "code_ring_read: invalid sizes");
  return launch(ring_read_kernel, dim3(unsigned(batch)), dim3(128), 0, stream, true, "code_ring_read", ring, slots,
                ring_depth, int(codebooks), indices, starts, length, out, status);
}
