// Library-wide entry points: ABI version, error strings, launch accounting.
#include <atomic>
#include <mutex>
#include <stdio.h>

#include "host.cuh"

namespace q3t {

namespace {
thread_local char g_error[512] = "";
std::atomic<uint64_t> g_launches{0};
std::atomic<int> g_sms[64];
}  // namespace

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_cuda(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return fail(Q3T_ECUDA, "%s: %s", what, cudaGetErrorString(err));
  return Q3T_OK;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  int n = g_sms[dev].load(std::memory_order_relaxed);
  if (n == 0) {  // the same value from every thread: a racing first query is harmless
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

namespace {
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiled tiled_encoder() {
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
}  // namespace

int make_map_bf16(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int64_t stride_elems, int box_cols,
                  int box_rows) {
  EncodeTiled enc = tiled_encoder();
  if (enc == nullptr) return fail(Q3T_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cuuint64_t(cols), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(stride_elems) * 2};
  cuuint32_t box[2] = {cuuint32_t(box_cols), cuuint32_t(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q3T_EINVAL, "tensor map encode failed (%d)", int(r));
  return Q3T_OK;
}

int make_map_bf16_3d(CUtensorMap* map, const void* base, int64_t d0, int64_t d1, int64_t d2, int box0, int box1,
                     int box2) {
  EncodeTiled enc = tiled_encoder();
  if (enc == nullptr) return fail(Q3T_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {cuuint64_t(d0), cuuint64_t(d1), cuuint64_t(d2)};
  cuuint64_t strides[2] = {cuuint64_t(d0) * 2, cuuint64_t(d0) * cuuint64_t(d1) * 2};
  cuuint32_t box[3] = {cuuint32_t(box0), cuuint32_t(box1), cuuint32_t(box2)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(Q3T_EINVAL, "tensor map encode failed (%d)", int(r));
  return Q3T_OK;
}

}  // namespace q3t

extern "C" int q3t_abi_version(void) { return 1; }
extern "C" const char* q3t_last_error(void) { return q3t::g_error; }
extern "C" uint64_t q3t_launch_count(void) { return q3t::g_launches.load(); }
