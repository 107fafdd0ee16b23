// Shared device helpers for the sm_100a kernels: bf16 rounding, mbarriers,
// TMA / bulk copies, tcgen05 (UMMA + TMEM) wrappers and bounded waits.
//
// Every wait on an mbarrier or a flag is bounded by wall time read from
// %globaltimer. On expiry the waiting thread ORs an error bit into the
// caller-supplied status word and returns false; callers then skip the
// remaining work, release TMEM and exit, so a broken pipeline ends the
// kernel with an error status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "q3t.h"

#define Q3T_DEV __device__ __forceinline__

namespace q3t {

// ---------------------------------------------------------------- numerics
Q3T_DEV float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// bf16 SnakeBeta x + inv * sin(a * x)^2 with rounding after every op (snake_triton_ascend.py:20-24),
// as the codec's convolutions apply it (im2col gather, padded conv input, GEMM epilogue). The sine
// is the __sinf intrinsic: its error (about 1e-6 absolute at these phases) is far below the bf16
// rounding that follows, so a result can move by at most one bf16 unit, at a rounding boundary; the
// codec is held to SNR >= 40 dB against the fp32 oracle, and q3t_snake keeps the precise sinf.
Q3T_DEV float snake_bf16(float x, float a, float inv) {
  const float phase = bf16r(x * a);
  const float sine = bf16r(__sinf(phase));
  const float square = bf16r(sine * sine);
  const float scaled = bf16r(inv * square);
  return bf16r(x + scaled);
}
Q3T_DEV float ld_bf16(const __nv_bfloat16* p) { return __bfloat162float(*p); }

// Unpack 8 bf16 (one 16-byte vector) to fp32.
Q3T_DEV void unpack8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
Q3T_DEV uint4 pack8(const float (&f)[8]) {
  uint4 v;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return v;
}

Q3T_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
Q3T_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---------------------------------------------------------------- time / status
// Error bits written to the status word by bounded waits.
enum : unsigned {
  kStatusTmaTimeout = 1u << 0,
  kStatusMmaTimeout = 1u << 1,
  kStatusFlagTimeout = 1u << 2,
  kStatusBadIndex = 1u << 3,
  kStatusNonFinite = 1u << 4,
};
// Two seconds: every kernel here finishes in well under a millisecond.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

Q3T_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
Q3T_DEV void raise_status(unsigned* status, unsigned bits) {
  if (status != nullptr) atomicOr(status, bits);
}

// ---------------------------------------------------------------- shared memory
Q3T_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
Q3T_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
Q3T_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
Q3T_DEV void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
Q3T_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
Q3T_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
Q3T_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded parity wait. Returns false (and raises `bits`) after kWaitLimitNs.
Q3T_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* status, unsigned bits) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > kWaitLimitNs) {
      raise_status(status, bits);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA / bulk copies
// No multicast anywhere: every CTA loads its own tiles.
Q3T_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
Q3T_DEV uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
Q3T_DEV uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2-D tiled tensor load; x (innermost, elements) * element size must be a multiple of 16 bytes.
Q3T_DEV void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// 3-D tiled tensor load; the same alignment rule for x.
Q3T_DEV void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Tiled tensor stores from shared memory (bulk-group completion); the coordinates are
// non-negative and x * element size is a multiple of 16 bytes. Out-of-range parts are clipped.
Q3T_DEV void tma_store_2d(const CUtensorMap* map, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
Q3T_DEV void tma_store_3d(const CUtensorMap* map, const void* smem_src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z), "r"(smem_u32(smem_src))
               : "memory");
}
Q3T_DEV void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until every committed bulk store has finished READING its shared-memory source.
Q3T_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// L2 prefetch hint for a global range (16-byte aligned address, bytes % 16 == 0); no completion.
Q3T_DEV void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}
// Share `id` of `parts` equal shares of a byte range (16-byte units), pulled into L2 in
// requests of at most 32 KB; no completion, no effect on results.
Q3T_DEV void prefetch_l2_share(const uint8_t* base, uint64_t bytes, uint64_t id, uint64_t parts) {
  const uint64_t units = bytes / 16, per = (units + parts - 1) / parts;
  const uint64_t u0 = id * per, u1 = u0 + per < units ? u0 + per : units;
  for (uint64_t u = u0; u < u1; u += 2048) {
    const uint64_t n = u1 - u < 2048 ? u1 - u : 2048;
    prefetch_l2(base + u * 16, uint32_t(n * 16));
  }
}
// Untiled bulk copy global -> shared with an L2 cache policy (createpolicy); same alignment.
Q3T_DEV void bulk_load_hint(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// Untiled bulk copy global -> shared; both addresses 16-byte aligned, bytes % 16 == 0.
Q3T_DEV void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// Wait for the preceding kernel in the stream to complete (no-op without the
// PDL attribute), then allow the next kernel to begin launching: its CTAs may
// become resident while this grid runs and do their dependency-free prologue
// (barrier setup, weight prefetch) before their own wait. Triggering only
// after the wait keeps at most two grids of the chain resident at a time, and
// since the trigger fires once every CTA of this grid has executed it, the
// early CTAs never take launch slots from this grid.
Q3T_DEV void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
Q3T_DEV void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_result)),
               "r"(ncols)
               : "memory");
}
Q3T_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
Q3T_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
Q3T_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
Q3T_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulator, one elected thread.
Q3T_DEV void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when all previously issued tcgen05.mma of this thread complete.
Q3T_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// Load 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
Q3T_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Load N (8, 16 or 32) consecutive fp32 columns of this warp's 32 TMEM lanes with one
// instruction and one wait.
template <int N>
Q3T_DEV void tmem_ld(uint32_t taddr, float (&v)[N]) {
  static_assert(N == 8 || N == 16 || N == 32, "tmem_ld: 8, 16 or 32 columns");
  if constexpr (N == 16) {
    tmem_ld16(taddr, v);
  } else if constexpr (N == 8) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
  } else {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
  }
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 64 bf16 (128 B), 8-row core groups 1024 B apart.
// Fields (sm_100 UMMA descriptor): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version=1 [46,48), layout=SWIZZLE_128B(2) [61,64).
Q3T_DEV uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}
// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4)                                  // D format: f32
         | (1u << 7)                                // A format: bf16
         | (1u << 10)                               // B format: bf16
         | (static_cast<uint32_t>(n >> 3) << 17)    // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);   // M >> 4
}

}  // namespace q3t
