/*
 * q3t.h - C ABI of the B200 (sm_100a) kernels for the Qwen3-TTS
 * talker -> code-predictor -> codec decode path.
 *
 * Conventions
 *   - Every entry point is `extern "C"`, takes plain device pointers, element
 *     counts and element strides, and enqueues work on `stream` (a
 *     cudaStream_t passed as void*). Nothing synchronises with the host, so
 *     every entry point may be recorded into a CUDA graph.
 *   - Return value: Q3T_OK (0) or a negative error code. Arguments are
 *     validated before any launch; on error nothing is written and
 *     q3t_last_error() describes the failure (thread-local string).
 *   - The library never allocates or frees caller memory. Kernels that need
 *     scratch take a caller-owned `workspace` (size from the matching
 *     *_workspace_bytes query, zero-filled once before first use; the kernels
 *     leave it ready for the next call).
 *   - `status` (nullable) is a caller-owned device word. Kernels OR error bits
 *     into it instead of trapping: bit 0 TMA wait timeout, bit 1 MMA wait
 *     timeout, bit 2 flag wait timeout, bit 3 out-of-range index skipped.
 *
 * Each declaration names the reference interface it replaces
 * (InferMatrixLab/qwen3-tts-rsi-engine, paths inside that project).
 */
#ifndef Q3T_H
#define Q3T_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  Q3T_OK = 0,
  Q3T_EINVAL = -1,      /* invalid shape, stride, alignment or dtype */
  Q3T_EUNSUPPORTED = -2,/* valid but outside the shapes this build supports */
  Q3T_ECUDA = -3,       /* CUDA launch or driver error */
  Q3T_ESPACE = -4       /* workspace too small */
};

enum { Q3T_BF16 = 0, Q3T_F32 = 1 };

/* Epilogues of q3t_linear. */
enum {
  Q3T_EPI_STORE = 0,        /* out = acc (+ bias), rounded to out dtype */
  Q3T_EPI_RESIDUAL = 1,     /* out = bf16(residual + bf16(acc)) */
  Q3T_EPI_SWIGLU_PAIRED = 2,/* rows of each 128-row weight tile are [64 gate; 64 up];
                               out[:, f] = bf16(bf16(silu(gate_f)) * up_f) */
  Q3T_EPI_RESIDUAL_SCALED = 3,/* out = bf16(residual + bf16(scale[n] * bf16(acc + bias))) */
  Q3T_EPI_GELU = 4,         /* out = bf16(gelu_erf(bf16(acc + bias))) */
  Q3T_EPI_SILU = 5,         /* out = bf16(silu(bf16(acc + bias))) - text_projection fc1 + act */
  Q3T_EPI_SNAKE = 6         /* out = snake_bf16(bf16(acc + bias), alpha[n], inverse_beta[n]): the SnakeBeta
                               of the codec's next conv (q3t_conv_linear only) */
};

/* RMSNorm rounding modes. */
enum {
  Q3T_NORM_REFERENCE = 0, /* bf16(w * bf16(x * rsqrt(mean(x^2) + eps))) - HF Qwen3 RMSNorm */
  Q3T_NORM_NATIVE = 1     /* bf16(w * x * rsqrt(mean(x^2) + eps)) - one rounding */
};

int q3t_abi_version(void);
const char* q3t_last_error(void);
/* Number of kernels this library has launched from this process (all devices). */
uint64_t q3t_launch_count(void);

/* ------------------------------------------------------------------ KV arena */

/* Replaces qwen3_tts_engine/kv_triton_ascend.py:39 write() and the scatter in
 * qwen3_tts_engine/continuous.py:152-166 SlotCache.update().
 * keys/values: [batch, heads, 1, width] with element strides
 * {batch, head, dim} (strided views of a packed QKV projection are allowed).
 * target_keys/target_values: contiguous [batch, heads, capacity, width].
 * positions: int64 [batch]. target[b, h, positions[b], :] = source[b, h, 0, :].
 * Out-of-range positions are skipped and raise status bit 3. */
int q3t_kv_write(const void* keys, const int64_t* key_strides, const void* values,
                 const int64_t* value_strides, void* target_keys, void* target_values,
                 const int64_t* positions, int64_t batch, int64_t heads, int64_t width,
                 int64_t capacity, int dtype, unsigned* status, void* stream);

/* Replaces qwen3_tts_engine/packed_kv.py:6 copy_packed_prefix(target, source, slot, row, length).
 * target: 5-D [planes, slots, heads, capacity, width], source: 5-D
 * [planes, rows, heads, length, width], each with element strides.
 * target[:, slot, :, :length] = source[:, row, :, :length]. elem_size 2, 4 or 8. */
int q3t_copy_packed_prefix(void* target, const int64_t* target_shape, const int64_t* target_strides,
                           const void* source, const int64_t* source_shape,
                           const int64_t* source_strides, int elem_size, int64_t slot, int64_t row,
                           int64_t length, void* stream);

/* Replaces qwen3_tts_engine/continuous.py:124 SlotArena.move(),
 * qwen3_tts_engine/codec_slots.py:328 CodecSlots.move() and
 * qwen3_tts_engine/codec_code_buffer.py:29 CodecCodeBuffer.move().
 * For every plane p: copy slot_elems contiguous elements from slot `source`
 * to slot `destination` (strides in elements). No-op when source == destination. */
int q3t_slot_move(void* base, int64_t planes, int64_t plane_stride, int64_t slot_stride,
                  int64_t slot_elems, int elem_size, int64_t source, int64_t destination,
                  void* stream);

/* Replaces the capacity-doubling copy of qwen3_tts_engine/continuous.py:353-363
 * ensure_capacity(): rows x row_bytes from src (pitch src_pitch bytes) to dst (pitch dst_pitch). */
int q3t_copy_rows(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                  int64_t row_bytes, int64_t rows, void* stream);

/* Replaces qwen3_tts_engine/codec_slots.py:313 CodecSlots.reset_range() /
 * reset(): zero `count` slots starting at `start` in each plane. */
int q3t_slot_zero(void* base, int64_t planes, int64_t plane_stride, int64_t slot_stride,
                  int64_t slot_elems, int elem_size, int64_t start, int64_t count, void* stream);

/* Per-tick counter update of continuous.py:628-629 (state.frames += 1,
 * state.position += 1) on device-resident counters: values[i] += delta. */
int q3t_advance(int64_t* values, int64_t count, int64_t delta, void* stream);

/* ------------------------------------------------------------------ norms, rotary, activations */

/* Replaces qwen3_tts_engine/operators.py:16 AscendRMSNorm.forward (both modes).
 * x: [rows, width] (row stride x_stride), weight: [width], out: [rows, width] contiguous. */
int q3t_rms_norm(const void* x, int64_t x_stride, const void* weight, void* out, int64_t rows,
                 int64_t width, float eps, int mode, void* stream);

/* Replaces torch_npu.npu_add_rms_norm at qwen3_tts_engine/fused_decoder.py:34.
 * residual_out = bf16(a + h); normalized = rmsnorm(sum) * w. mode Q3T_NORM_NATIVE
 * normalises the unrounded fp32 sum (npu semantics); Q3T_NORM_REFERENCE
 * normalises the rounded residual with HF rounding. residual_out may alias h. */
int q3t_add_rms_norm(const void* a, const void* h, const void* weight, void* normalized,
                     void* residual_out, int64_t rows, int64_t width, float eps, int mode,
                     void* stream);

/* Replaces qwen3_tts_engine/rotary_triton_ascend.py:29 rotary(hidden, cos, sin):
 * BSND bf16 [batch, length, heads, width], cos/sin [batch, length, width],
 * bf16 rounding after every product and sum. */
int q3t_rotary(const void* x, const void* cos, const void* sin, void* out, int64_t batch,
               int64_t length, int64_t heads, int64_t width, void* stream);

/* Replaces torch_npu.npu_swiglu / act_fn(gate) * up at qwen3_tts_engine/packed_mlp.py:20-26:
 * packed [rows, 2*width] (gate | up) -> out [rows, width]. */
int q3t_swiglu(const void* packed, void* out, int64_t rows, int64_t width, void* stream);

/* Replaces qwen3_tts_engine/snake_triton_ascend.py:28 snake(hidden, alpha, inverse_beta):
 * NCT [batch, channels, length], alpha/inverse_beta [channels] (fp32 or input dtype).
 * dtype Q3T_BF16 rounds after every operation as the reference kernel does. */
int q3t_snake(const void* x, const void* alpha, const void* inverse_beta, void* out,
              int64_t batch, int64_t channels, int64_t length, int dtype, int coef_dtype,
              void* stream);

/* ------------------------------------------------------------------ dense projections */

/* Replaces torch.nn.functional.linear at qwen3_tts_engine/packed_attention.py:42,85,
 * qwen3_tts_engine/packed_mlp.py:20,27 and the codec head at continuous.py:613.
 * out[r, n] = epilogue(sum_k x[r, k] * weight[n, k] (+ bias[n])). tcgen05 GEMM,
 * weights as the 128-row UMMA operand, rows as N, split-K over a thread-block
 * cluster reduced through distributed shared memory (workspace unused; may be NULL).
 * Also the codec's convolutions (im2col rows from q3t_conv_gather), its
 * ConvNeXt pointwise layers (GELU / scaled-residual epilogues) and the layer-scaled
 * residuals of its transformer.
 * x, weight, bias, residual: bf16; out: bf16 or fp32 (Q3T_EPI_STORE only).
 * Alignment: base pointers 16 B, row strides multiples of 8 elements. */
size_t q3t_linear_workspace_bytes(int64_t rows, int64_t in_features, int64_t out_features);
int q3t_linear(const void* x, int64_t x_stride, int64_t rows, int64_t in_features,
               const void* weight, int64_t out_features, const void* bias, void* out,
               int64_t out_stride, int out_dtype, int epilogue, const void* residual,
               int64_t residual_stride, const void* scale, const void* weight_tiles,
               void* workspace, size_t workspace_bytes, unsigned* status, void* stream);

/* q3t_linear with the preceding RMSNorm folded in (qwen3_tts_engine/operators.py:16-23
 * followed by the projection at packed_attention.py:42 / packed_mlp.py:20):
 *   out[r, n] = epilogue(rsqrt(mean_k x[r, k]^2 + eps) * sum_k x[r, k] * weight[n, k] (+ bias[n]))
 * with the norm weight pre-multiplied into the projection by the caller
 * (weight[n, k] = W[n, k] * norm_weight[k], rounded to bf16). x is the raw
 * residual stream; the row sums of squares are taken from the activation tiles
 * the GEMM streams anyway, so no normalised copy of x is written. eps > 0. */
int q3t_linear_rownorm(const void* x, int64_t x_stride, int64_t rows, int64_t in_features,
                       const void* weight, int64_t out_features, const void* bias, void* out,
                       int64_t out_stride, int out_dtype, int epilogue, const void* residual,
                       int64_t residual_stride, const void* scale, float eps, const void* weight_tiles,
                       unsigned* status, void* stream);

/* Flags of q3t_linear_ex. */
#define Q3T_LINEAR_KEEP_WEIGHTS 1 /* load the weight tiles evict-last (the chain re-reads them soon) */
#define Q3T_LINEAR_NARROW 2       /* keep the split-K kernel at prefill-sized row counts (see below) */

/* q3t_linear (eps == 0) or q3t_linear_rownorm (eps > 0) with two cache controls:
 * - prefetch: [prefetch, prefetch + prefetch_bytes) (the next kernel's weights) is split
 *   over the CTAs and pulled into L2 before the dependency wait (a hint only: no
 *   ordering, no completion); 16-byte aligned, prefetch_bytes % 16 == 0; NULL or 0 = none;
 * - flags: Q3T_LINEAR_KEEP_WEIGHTS loads this GEMM's weight tiles with L2 evict-last
 *   priority instead of evict-first (the code predictor keeps part of its layers in L2
 *   across its 15 codebook steps, continuous.py:49-68).
 * Row counts in the thousands (a packed prefill; PrefillGraph's projections,
 * prefill_graph.py:31-50) with pre-tiled weights, a bf16 output, eps == 0, no prefetch and
 * no flags run a persistent kernel of 128-feature x 256-row tiles instead of the split-K
 * kernel; Q3T_LINEAR_NARROW keeps the split-K kernel (results agree to bf16 rounding). */
int q3t_linear_ex(const void* x, int64_t x_stride, int64_t rows, int64_t in_features,
                  const void* weight, int64_t out_features, const void* bias, void* out,
                  int64_t out_stride, int out_dtype, int epilogue, const void* residual,
                  int64_t residual_stride, const void* scale, float eps, const void* weight_tiles,
                  const void* prefetch, size_t prefetch_bytes, int flags, unsigned* status, void* stream);

/* A chain of dependent projections in one persistent launch: the projections a decode
 * layer runs between two attentions (PackedAttention's o_proj, packed_attention.py:85,
 * then PackedMLP's gate/up and down, packed_mlp.py:19-27, then the next layer's packed
 * QKV, packed_attention.py:42, with the RMSNorms of operators.py:16-23 folded in as in
 * q3t_linear_rownorm), or the last layer's projections followed by a codebook head.
 * Stage s computes out_s = epilogue(x_s @ W_s^T) exactly as q3t_linear(_rownorm) would
 * (W_s given as q3t_pack_weight_tiles tiles), but no stage waits for a kernel boundary:
 * every SM streams its even share of all the stages' weight tiles without a break, and
 * only the activation tiles of stage s wait until stage `depends` has stored all its
 * outputs (depends = -1: stage s reads only what earlier kernels wrote). Split-K partials
 * are reduced in a fixed order (deterministic). */
#define Q3T_CHAIN_MAX_STAGES 8
typedef struct {
  const void* x;              /* bf16 [rows, in_features], row stride x_stride */
  int64_t x_stride;
  const void* weight_tiles;   /* q3t_pack_weight_tiles of the bf16 [out_features, in_features] weight */
  int64_t in_features, out_features;
  void* out;                  /* bf16, or fp32 with Q3T_EPI_STORE; row stride out_stride */
  int64_t out_stride;
  int out_dtype;              /* Q3T_BF16 or Q3T_F32 */
  int epilogue;               /* Q3T_EPI_STORE, Q3T_EPI_RESIDUAL or Q3T_EPI_SWIGLU_PAIRED */
  const void* residual;       /* bf16, Q3T_EPI_RESIDUAL (may alias out) */
  int64_t residual_stride;
  const void* bias;           /* bf16 [out_features] or NULL */
  float row_norm_eps;         /* > 0: folded RMSNorm of x (see q3t_linear_rownorm); 0: none */
  int depends;                /* earlier stage whose output x (or the residual) reads; -1: none */
} q3t_chain_stage;

/* Workspace of q3t_linear_chain for `rows` activation rows (1..64): a counter block and the
 * split-K partials. Zero it once before the first call; every call leaves the counters zero. */
size_t q3t_linear_chain_workspace_bytes(int64_t rows);

/* Runs `count` (1..Q3T_CHAIN_MAX_STAGES) stages on `rows` (1..64) activation rows. Every stage
 * needs at least as many weight tiles x k-blocks as the device has SMs. One workspace per
 * stream: two chains sharing a workspace must not overlap on the GPU. */
int q3t_linear_chain(const q3t_chain_stage* stages, int count, int64_t rows, void* workspace,
                     size_t workspace_bytes, unsigned* status, void* stream);

/* Weight re-layout done once at load, in place of the reference's packed QKV and gate/up
 * concatenations (packed_attention.py:17-22, packed_mlp.py:13-14).
 * Pre-swizzled weight layout for q3t_linear (pass it as weight_tiles, weight may
 * then be NULL): tile (n, k) of 128 rows x 64 columns is the contiguous 16 KB image
 * of the 128-byte-swizzled shared-memory tile, tiles ordered [n][k], zero padded.
 * Each pipeline stage then streams one contiguous 16 KB block from HBM. */
size_t q3t_weight_tiles_bytes(int64_t out_features, int64_t in_features);
int q3t_pack_weight_tiles(const void* weight, int64_t out_features, int64_t in_features, void* tiles,
                          void* stream);

/* ------------------------------------------------------------------ attention */

/* Replaces the q_norm/k_norm, rotary and cache update of
 * qwen3_tts_engine/packed_attention.py:42-74 (text-only rotary, decode and prefill rows).
 * qkv: [rows, (q_heads + 2*kv_heads)*head_dim] bf16 (row stride qkv_stride);
 * row r belongs to slot r / length (or slots[r / length] when the slot table is given)
 * and sequence offset r % length. Null norm weights skip the head norms (codec).
 * cos/sin tables: [table_len, head_dim] bf16; rotary_positions[r] indexes them.
 * cache_positions[r]: KV write position of row r in target [slots, kv_heads, capacity, head_dim].
 * query_out: [rows, q_heads, head_dim]. */
int q3t_qk_norm_rope_kv(const void* qkv, int64_t qkv_stride, const void* q_norm_weight,
                        const void* k_norm_weight, float eps, const void* cos_table,
                        const void* sin_table, int64_t table_len, const int64_t* rotary_positions,
                        const int64_t* cache_positions, void* query_out, void* target_keys,
                        void* target_values, int64_t rows, int64_t length, const int64_t* slots,
                        int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t capacity,
                        unsigned* status, void* stream);

/* Causal prefill attention over packed prompts: the prefill call of
 * npu_fused_infer_attention_score (qwen3_tts_engine/npu_attention.py:21, query length L with
 * the causal mask PrefillGraph builds, prefill_graph.py:31-50), on tcgen05 tensor cores.
 * query [rows, q_heads, head_dim] bf16 (post q-norm and RoPE); keys/values the arena layer
 * [arena_slots, kv_heads, capacity, head_dim] bf16 holding every row's K/V already;
 * positions[r] the position of packed row r. units: int32 [unit_count][4] =
 * {first_row, count, keys, slot}: rows first_row .. first_row + count - 1 (count <= 64)
 * are positions of arena slot `slot`, each attending keys 0 .. positions[r] of that slot
 * (keys = 1 + the largest such position); count 0 = an unused entry. out [rows, q_heads,
 * head_dim] bf16; rows that no unit covers are not written. head_dim 128 with 2 query heads
 * per KV head. A unit whose fields do not fit raises the status word's bad-index bit and is
 * skipped. No workspace. */
int q3t_prefill_attention(const void* query, const void* keys, const void* values,
                          const int64_t* positions, const int32_t* units, int64_t unit_count, void* out,
                          int64_t rows, int64_t q_heads, int64_t kv_heads, int64_t head_dim,
                          int64_t arena_slots, int64_t capacity, float scale, unsigned* status,
                          void* stream);

/* Replaces torch_npu.npu_fused_infer_attention_score at qwen3_tts_engine/npu_attention.py:21
 * (and SDPA over SlotCache, continuous.py:188-198; the predictor's causal
 * 2-token first step, continuous.py:37-40; the codec's sliding window,
 * codec_slots.py:73-77). query rows [rows, q_heads, head_dim] bf16; row r
 * reads slot r / rows_per_slot of keys/values [slots, kv_heads, capacity, head_dim]
 * (bf16, contiguous) and sees keys max(0, p - window + 1) .. p with
 * p = positions[r] (window 0 = unbounded). With a slot table, row r reads
 * slot slots[r / rows_per_slot]. ring > 0 makes the arena a ring of `ring`
 * rows (capacity == ring): position p lives in row p % ring, positions are
 * unbounded and 1 <= window <= ring (the codec's KV tail, codec_slots.py:27-39).
 * Otherwise context bounds the grid (positions < context <= capacity).
 * arena_slots: the slot extent of keys/values. out [rows, q_heads, head_dim] bf16.
 * Linear arenas run on tensor-core fragments (mma.sync) with TMA-swizzled K/V tiles.
 * Split-KV with an in-kernel combine. */
size_t q3t_decode_attention_workspace_bytes(int64_t rows, int64_t q_heads, int64_t head_dim,
                                            int64_t context);
int q3t_decode_attention(const void* query, const void* keys, const void* values,
                         const int64_t* positions, void* out, int64_t rows, int64_t rows_per_slot,
                         const int64_t* slots, int64_t ring, int64_t q_heads, int64_t kv_heads,
                         int64_t head_dim, int64_t arena_slots, int64_t capacity, int64_t context,
                         int64_t window, float scale, void* workspace, size_t workspace_bytes,
                         unsigned* status, void* stream);

/* Chunk plan of the decode attention for this batch (once per decode step, before the
 * layers): with the query positions of the step's rows, writes into the attention
 * workspace the keys per split-KV chunk that let one wave of resident CTAs cover all
 * (row, kv head) pairs (a power of two times the default chunk). Later
 * q3t_decode_attention / _qkv calls on the same workspace (one query row per slot, no
 * window) use it; without a plan, or with a stale one, results are identical and only
 * the split differs. positions: int64 [rows]. Part of the replacement of the talker's
 * fused attention call (npu_attention.py:11-26), whose NPU operator splits the keys
 * internally; here the split is planned once per step instead of once per layer. */
int q3t_attention_plan(const int64_t* positions, int64_t rows, int64_t q_heads, int64_t kv_heads,
                       int64_t head_dim, int64_t context, void* workspace, size_t workspace_bytes,
                       void* stream);

/* Talker decode step attention with the per-head q/k RMSNorm, RoPE and the
 * K/V write of PackedAttention.forward (packed_attention.py:42-74) fused in:
 * reads the raw QKV projection rows qkv [rows, (q_heads + 2 kv_heads) * head_dim]
 * (row stride qkv_stride), normalises (q_norm/k_norm, nullable) and rotates them
 * at rotary_positions with the cos/sin tables, writes the new key/value of row b
 * at positions[b] of arena slot b, and attends over keys 0..positions[b]
 * (one query row per slot, no window). Same workspace as q3t_decode_attention. */
int q3t_decode_attention_qkv(const void* qkv, int64_t qkv_stride, const void* q_norm_weight,
                             const void* k_norm_weight, float eps, const void* cos_table,
                             const void* sin_table, int64_t table_len, const int64_t* rotary_positions,
                             void* keys, void* values, const int64_t* positions, void* out, int64_t rows,
                             int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t arena_slots,
                             int64_t capacity, int64_t context, float scale, void* workspace,
                             size_t workspace_bytes, unsigned* status, void* stream);

/* q3t_decode_attention_qkv with an L2 prefetch hint (the same replacement of
 * PackedAttention.forward's norm / RoPE / cache update / attention,
 * packed_attention.py:42-74): while the keys stream, the kernel's CTAs pull up
 * to two byte ranges (prefetchN, prefetchN_bytes; null / 0 = none; 16-byte
 * aligned, sizes multiples of 16) into L2 - in a decode step the weights of the
 * projections that follow the attention, so that those latency-bound GEMMs read
 * them from L2. The hint changes no result. */
int q3t_decode_attention_qkv_ex(const void* qkv, int64_t qkv_stride, const void* q_norm_weight,
                                const void* k_norm_weight, float eps, const void* cos_table,
                                const void* sin_table, int64_t table_len, const int64_t* rotary_positions,
                                void* keys, void* values, const int64_t* positions, void* out, int64_t rows,
                                int64_t q_heads, int64_t kv_heads, int64_t head_dim, int64_t arena_slots,
                                int64_t capacity, int64_t context, float scale, void* workspace,
                                size_t workspace_bytes, const void* prefetch0, size_t prefetch0_bytes,
                                const void* prefetch1, size_t prefetch1_bytes, unsigned* status,
                                void* stream);

/* No counterpart in the reference: an allocation-free form of
 * q3t_decode_attention for callers that cannot allocate device memory (a
 * runtime with a fixed pre-reserved pool, a foreign-language host without a
 * CUDA allocator). It takes q3t_decode_attention's arguments without the
 * workspace and without a slot table or ring: keys/values are linear arenas
 * [arena_slots, kv_heads, capacity, head_dim] and query row b reads slot
 * b / rows_per_slot, so arena_slots * rows_per_slot >= rows is required
 * (Q3T_EINVAL otherwise). Results agree with q3t_decode_attention within the
 * bf16 attention tolerance (it always runs the CUDA-core attention kernel,
 * while the workspace entry point may pick the tensor-core one). The split-KV
 * scratch is a 4 MiB file-scope device array that every GPU loading the
 * library keeps until exit. Limits: rows * kv_heads <= 16384 and the chunk
 * partials must fit the rest of the 4 MiB; larger calls return Q3T_ESPACE
 * before launching. The first call in each CUDA context resolves the array's
 * device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture. Calls share the array and keep the last call's contents
 * (each clears its own tickets first); calls that overlap on the GPU race and
 * must be ordered by the caller. No cudaMalloc/cudaFree anywhere. */
int q3t_decode_attention_noalloc(const void* query, const void* keys, const void* values,
                                 const int64_t* positions, void* out, int64_t rows,
                                 int64_t rows_per_slot, int64_t q_heads, int64_t kv_heads,
                                 int64_t head_dim, int64_t arena_slots, int64_t capacity,
                                 int64_t context, int64_t window, float scale, unsigned* status,
                                 void* stream);

/* ------------------------------------------------------------------ sampling */

/* Replaces qwen3_tts_engine/cdf_triton_ascend.py:20 select(cdf, uniforms):
 * token[r] = #{ j : cdf[r, j] / cdf[r, width-1] <= u[r] } with IEEE division. */
int q3t_cdf_select(const float* cdf, const float* uniforms, int64_t* tokens, int64_t rows,
                   int64_t width, void* stream);

/* Replaces qwen3_tts_engine/sampling.py:5 categorical(), the semantic
 * preprocessing of qwen3_tts_engine/continuous.py:365-370 and the seen update of
 * qwen3_tts_engine/sampling_graph.py:14-16, in one kernel per row:
 *   scores = float(logits)                         (bf16 or fp32 logits)
 *   if seen:    scores = seen ? (s < 0 ? s*penalty : s/penalty) : s
 *   if allowed: scores[~allowed] = -inf
 *   if steps:   scores[eos] = -inf where steps[r] < min_steps
 *   scores /= temperature; keep scores >= k-th largest (ties kept);
 *   softmax; optional top-p (smallest set with mass >= top_p; 1.0 disables);
 *   cdf = cumsum; token = #{ cdf / cdf[-1] <= u }.
 * u: uniforms[r * uniform_stride] when uniforms != NULL, else Philox4x32-10 with
 *    key = seed and counter = {c lo, c hi, 0, 0}, c = philox_offsets[r] + philox_add
 *    (row r when philox_offsets is NULL), first word mapped to [0, 1) as (x >> 8) * 2^-24.
 * seen_out (nullable, may alias seen): seen row copied, then seen_out[r, token] = 1. */
int q3t_sample(const void* logits, int logits_dtype, int64_t logits_stride, const uint8_t* seen,
               int64_t seen_stride, const uint8_t* allowed, const int64_t* steps, int64_t eos,
               int64_t min_steps, float penalty, float temperature, int64_t top_k, float top_p,
               const float* uniforms, int64_t uniform_stride, uint64_t seed,
               const int64_t* philox_offsets, int64_t philox_add, int64_t* tokens, int64_t token_stride,
               uint8_t* seen_out, int64_t seen_out_stride, int64_t rows, int64_t width,
               void* stream);

/* Device-side uniforms for sampling without a host table (the reference draws its
 * per-request tables on the host, sampling.py:17-19).
 * Philox4x32-10 uniforms in [0, 1): out[i] = u(key=seed, counter={offset + i/4 lo, hi, 0, 0})[i%4]. */
int q3t_philox_uniforms(uint64_t seed, uint64_t offset, float* out, int64_t count, void* stream);

/* ------------------------------------------------------------------ embeddings */

/* Replaces the frame embedding of qwen3_tts_engine/continuous.py:584-601
 * (talker codec embedding of codes[:, 0] plus the 15 predictor embeddings of
 * codes[:, 1..15], summed in fp32 and rounded once, then + text):
 * codes int64 [batch, 1 + groups] (row stride codes_stride);
 * first_table [first_vocab, hidden]; group_tables [groups, group_vocab, hidden];
 * text [batch, hidden] (row stride text_stride, nullable); out [batch, hidden] bf16. */
int q3t_frame_embed(const int64_t* codes, int64_t codes_stride, const void* first_table,
                    int64_t first_vocab, const void* group_tables, int64_t groups,
                    int64_t group_vocab, const void* text, int64_t text_stride, void* out,
                    int64_t batch, int64_t hidden, unsigned* status, void* stream);

/* Replaces the token embedding lookups of continuous.py:584 (talker.get_input_embeddings())
 * and custom_voice_prompt.py:38-63 (text embedding).
 * Row gather out[r] = table[ids[r]] (embedding lookup, bf16 rows of `hidden`). */
int q3t_embedding(const int64_t* ids, int64_t ids_stride, const void* table, int64_t vocab,
                  void* out, int64_t out_stride, int64_t rows, int64_t hidden, unsigned* status,
                  void* stream);

/* ------------------------------------------------------------------ codec state */

/* Replaces qwen3_tts_engine/codec_row_scatter.py:48 scatter_rows(target, indices, source):
 * target contiguous [slots, ...]; source [n, ...] with element strides (ndim 1..4);
 * target[indices[i]] = source[i]. Out-of-range indices are skipped (status bit 3). */
int q3t_scatter_rows(void* target, int64_t target_rows, const int64_t* indices,
                     const void* source, int ndim, const int64_t* source_shape,
                     const int64_t* source_strides, int elem_size, unsigned* status,
                     void* stream);

/* ------------------------------------------------------------------ incremental codec */

/* Replaces CachedQuantizer.decode (qwen3_tts_engine/cached_quantizer.py:17-30) up to
 * the output projections: out[(b,t)] = [sum_{q<semantic} table_q[code] | sum_{q>=semantic}
 * table_q[code]] (fp32 sums in codebook order, rounded once) as [batch*frames, 2*dim] bf16;
 * tables: pre-normalised codebooks [codebooks, bins, dim] bf16. The caller applies
 * [W_first | W_rest] with q3t_linear. codes: int64 with element strides (batch, codebook, frame). */
int q3t_rvq_gather(const int64_t* codes, int64_t b_stride, int64_t cb_stride, int64_t t_stride,
                   const void* tables, int64_t codebooks, int64_t semantic, int64_t bins,
                   int64_t dim, int64_t batch, int64_t frames, void* out, unsigned* status,
                   void* stream);

/* Replaces the causal-conv history concat of IncrementalCodec.run_module
 * (qwen3_tts_engine/incremental_codec.py:53-65) and the SnakeBeta that precedes a conv
 * (snake_triton_ascend.py, incremental_codec.py:42-49): im2col rows
 * col[(b,t), j*C + c] = snake(src(b, t - shift_j, c)) with shift_j = (taps-1-j)*dilation
 * (reverse = 0) or j*dilation (reverse = 1, transposed convs: [x[t] | x[t-1]]);
 * negative times read history [slots, history_len, C] of slot slots[b] (or b).
 * x: time-major [batch, frames, C] (row stride x_stride); alpha/inverse_beta nullable. */
int q3t_conv_gather(const void* x, int64_t x_stride, int64_t batch, int64_t frames,
                    int64_t channels, const void* history, int64_t history_len,
                    const int64_t* slots, int64_t taps, int64_t dilation, int reverse,
                    const float* alpha, const float* inverse_beta, void* col, void* stream);

/* Padded input of an implicit causal conv (the history concat of
 * incremental_codec.py:53-65 and the preceding SnakeBeta, without im2col):
 * xs[b, p, c] = snake([history[slots[b]] | x[b]][p, c]) for p < history_len + frames,
 * as bf16 [batch, history_len + frames, channels]; alpha/inverse_beta nullable (identity). */
int q3t_conv_pad(const void* x, int64_t x_stride, int64_t batch, int64_t frames, int64_t channels,
                 const void* history, int64_t history_len, const int64_t* slots, const float* alpha,
                 const float* inverse_beta, void* xs, void* stream);

/* Replaces the codec's causal and transposed conv modules as IncrementalCodec.run_module
 * applies them (incremental_codec.py:53-65).
 * Causal conv (kernel `taps`, `dilation`) as an implicit tcgen05 GEMM over q3t_conv_pad's
 * buffer xs [batch, pad + frames, channels]: k-block (tap j, 64 channels) streams frames
 * t + j*dilation (or t + (taps-1-j)*dilation with reverse: transposed convs' [x[t] | x[t-1]])
 * of its stream straight from xs through a 3-D TMA map, so no im2col copy is written.
 *   out[b*frames + t, n] = epilogue(sum_{j,c} W[n, j*Cp + c] * xs[b, t + shift_j, c] (+ bias[n]))
 * weight_tiles: q3t_pack_weight_tiles of W [out_features, taps*Cp], channels zero-padded per
 * tap to Cp = 64 * ceil(channels / 64). Epilogues STORE, RESIDUAL(_SCALED), GELU, SILU and
 * SNAKE (alpha / inverse_beta fp32 [out_features]); bf16 output. pad >= (taps-1)*dilation. */
int q3t_conv_linear(const void* xs, int64_t batch, int64_t frames, int64_t pad, int64_t channels,
                    int64_t taps, int64_t dilation, int reverse, const void* weight_tiles,
                    int64_t out_features, const void* bias, void* out, int64_t out_stride, int epilogue,
                    const void* residual, int64_t residual_stride, const void* scale,
                    const float* snake_alpha, const float* snake_inv, unsigned* status, void* stream);

/* history = last history_len frames of [history | x] per slot (incremental_codec.py:62). */
int q3t_conv_history(const void* x, int64_t x_stride, int64_t batch, int64_t frames,
                     int64_t channels, void* history, int64_t history_len, const int64_t* slots,
                     void* stream);

/* ConvNeXt depthwise causal conv (kernel 7, history 6) + LayerNorm over channels
 * (incremental_codec.py:80-84): out [batch*frames, C] bf16. Weights fp32. */
int q3t_dwconv_layernorm(const void* x, int64_t batch, int64_t frames, int64_t channels,
                         const void* history, int64_t history_len, const int64_t* slots,
                         const float* weight, const float* bias, const float* ln_weight,
                         const float* ln_bias, float eps, void* out, void* stream);

/* Frame positions of a codec chunk (codec_slots.py:70-72, 98): for rows (b, t),
 * rotary = frames[slot_b] + t, cache = (frames[slot_b] + t) % ring (ring 0: no modulo);
 * advance != 0 then adds `frames` to frames[slot_b]. */
int q3t_codec_positions(int64_t* frames_by_slot, const int64_t* slots, int64_t batch,
                        int64_t frames, int64_t ring, int64_t* rotary_positions,
                        int64_t* cache_positions, int advance, void* stream);

/* PCM conversion of qwen3_tts_engine/continuous.py:531-533 on the device:
 * wave = clip(x, -1, 1) (fp32, nullable), pcm = int16(wave * 32767) (nullable).
 * A nonfinite input sample raises status bit 16 (the reference raises
 * "Native codec emitted nonfinite audio" at continuous.py:530-531). */
int q3t_pcm16(const void* x, int64_t count, float* wave, int16_t* pcm, unsigned* status, void* stream);

/* ---------------------------------------------------------------- engine slots
 * Device-resident request state of ContinuousModel (RequestState,
 * qwen3_tts_engine/continuous.py:232-247): slot i holds the i-th active
 * request; arrays are [slots, ...]. Rows >= *active (a device int64) are graph
 * padding and receive the reference's padding values (continuous.py:580-583,
 * 599-604).
 *
 * q3t_tick_gather replaces the per-tick torch.cat/stack of continuous.py:575-606:
 *   pred_inputs[b] = (hidden_state[b], codec_embedding[tokens[b]])  [rows, 2, hidden] bf16
 *   codes[b * codes_stride] = tokens[b]
 *   draws[b, :16] = tables[b, frames[b], :]; talker_uniform[b] = tables[b, frames[b] + 1, 0]
 *   steps[b] = frames[b] + 1
 *   text[b] = frames[b] < trailing_len[b] ? trailing[b, frames[b]] : pad[b]
 *   step_positions[b] = positions[b]; step_rotary[b] = rotary[b]
 * tables: [slots, table_rows, 16] fp32 (random_table, sampling.py:17-19). */
int q3t_tick_gather(const int64_t* active, const int64_t* tokens, const void* hidden_state,
                    const void* codec_embedding, int64_t vocab, const float* tables, int64_t table_rows,
                    const int64_t* frames, const void* trailing, int64_t trailing_rows,
                    const int64_t* trailing_len, const void* pad, const int64_t* positions,
                    const int64_t* rotary, void* pred_inputs, int64_t* codes, int64_t codes_stride,
                    float* draws, float* talker_uniform, int64_t* steps, void* text,
                    int64_t* step_positions, int64_t* step_rotary, int64_t rows, int64_t hidden,
                    unsigned* status, void* stream);

/* Write-back of continuous.py:618-635 for rows b < *active:
 *   ring[b, frames[b] % ring_depth, :] = codes[b, :codebooks]  (CodecCodeBuffer.write,
 *   codec_code_buffer.py:12-17); hidden_state[b] = step_hidden[b];
 *   frames[b] += 1; positions[b] += 1; rotary[b] += 1. */
int q3t_tick_commit(const int64_t* active, const int64_t* codes, int64_t codes_stride, int64_t codebooks,
                    const void* step_hidden, void* hidden_state, int64_t* ring, int64_t ring_depth,
                    int64_t* frames, int64_t* positions, int64_t* rotary, int64_t rows, int64_t hidden,
                    void* stream);

/* CodecCodeBuffer.write (codec_code_buffer.py:12-17): ring[i, frame_indices[i] % depth] = codes[i]
 * for i < count; ring [slots, depth, codebooks] int64. */
int q3t_code_ring_write(const int64_t* codes, int64_t codes_stride, const int64_t* frame_indices,
                        int64_t* ring, int64_t ring_depth, int64_t codebooks, int64_t count, void* stream);

/* CodecCodeBuffer.read (codec_code_buffer.py:19-27):
 * out[i, c, t] = ring[indices[i], (starts[i] + t) % depth, c], out [batch, codebooks, length]. */
int q3t_code_ring_read(const int64_t* ring, int64_t slots, int64_t ring_depth, int64_t codebooks,
                       const int64_t* indices, const int64_t* starts, int64_t batch, int64_t length,
                       int64_t* out, unsigned* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* Q3T_H */
