// Library-wide entry points: ABI version, error strings, launch accounting.
#include <atomic>
#include <stdio.h>

#include "host.cuh"

namespace q3t {

namespace {
thread_local char g_error[512] = "";
std::atomic<uint64_t> g_launches{0};
int g_sms[64] = {0};
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
  if (g_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

}  // namespace q3t

extern "C" int q3t_abi_version(void) { return 1; }
extern "C" const char* q3t_last_error(void) { return q3t::g_error; }
extern "C" uint64_t q3t_launch_count(void) { return q3t::g_launches.load(); }
