// Host-side helpers shared by the entry points: error strings, launch
// accounting and a launcher that sets the programmatic-dependent-launch
// attribute so a kernel may start while its predecessor drains.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "q3t.h"

namespace q3t {

// Records a printf-style message for q3t_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);
// Converts the last CUDA error (if any) into Q3T_ECUDA.
int check_cuda(const char* what);
// Counts kernel launches issued by this library.
void note_launch();
// Number of SMs of the current device (cached per device).
int sm_count();

// 2-D bf16 tensor map over a row-major matrix: dims {cols, rows}, row stride in
// elements, box {box_cols, box_rows}, 128-byte swizzle (box_cols * 2 <= 128).
int make_map_bf16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t stride_elems,
                  int box_cols, int box_rows);
// 3-D bf16 tensor map over a dense [d2][d1][d0] array: box {box0, box1, box2}, 128-byte swizzle.
int make_map_bf16_3d(CUtensorMap* map, const void* base, int64_t d0, int64_t d1, int64_t d2, int box0, int box1,
                     int box2);

// A per-device one-time set-up (a kernel attribute, a cached query): `run(init)`
// calls init() for the current device until it first succeeds, under a mutex, so
// host threads that make their first calls concurrently neither race on the flag
// nor skip the set-up.
class PerDevice {
 public:
  template <typename Init>
  int run(Init&& init, const char* what) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
      return fail(Q3T_ECUDA, "%s: no current CUDA device", what);
    if (done_[dev].load(std::memory_order_acquire)) return Q3T_OK;
    std::lock_guard<std::mutex> lock(mutex_);
    if (done_[dev].load(std::memory_order_relaxed)) return Q3T_OK;
    const int rc = init(dev);
    if (rc == Q3T_OK) done_[dev].store(true, std::memory_order_release);
    return rc;
  }

 private:
  static constexpr int kMaxDevices = 64;
  std::mutex mutex_;
  std::atomic<bool> done_[kMaxDevices] = {};
};

// Raises `kernel`'s dynamic shared-memory limit to `bytes` once per device.
template <typename Kernel>
int smem_limit(PerDevice& once, Kernel* kernel, int bytes, const char* what) {
  return once.run(
      [&](int) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
          return check_cuda(what);
        return int(Q3T_OK);
      },
      what);
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Launch `kernel` with optional programmatic stream serialization (PDL).
template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream, bool pdl,
           const char* name, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = as_stream(stream);
  cudaLaunchAttribute attr[1];
  if (pdl) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (err != cudaSuccess) return fail(Q3T_ECUDA, "%s launch failed: %s", name, cudaGetErrorString(err));
  note_launch();
  return Q3T_OK;
}

}  // namespace q3t
