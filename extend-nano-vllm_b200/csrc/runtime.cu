// Library-wide state: the thread-local error message, the device status word
// and per-device attribute caches.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include "common.cuh"

namespace b200moe {

__device__ int g_status = 0;

namespace {
thread_local char t_error[512] = "";
int g_sm_count[64] = {0};
}  // namespace

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_error, sizeof(t_error), fmt, ap);
  va_end(ap);
}

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  return dev;
}

int sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= 64) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

bool pdl_enabled(unsigned family) {
  static const unsigned mask = [] {
    const char *v = getenv("B200MOE_PDL");
    if (v == nullptr || *v == '\0') return ~0u;
    return static_cast<unsigned>(strtoul(v, nullptr, 0));
  }();
  return (mask & family) != 0;
}

}  // namespace b200moe

extern "C" {

const char *b200moe_last_error(void) { return b200moe::t_error; }

int b200moe_abi_version(void) { return 1; }

int b200moe_device_status(int *status, int clear) {
  B200_ARG(status != nullptr, "status must not be NULL");
  B200_CUDA(cudaMemcpyFromSymbol(status, b200moe::g_status, sizeof(int)));
  if (clear) {
    const int zero = 0;
    B200_CUDA(cudaMemcpyToSymbol(b200moe::g_status, &zero, sizeof(int)));
  }
  return B200MOE_OK;
}

}  // extern "C"
