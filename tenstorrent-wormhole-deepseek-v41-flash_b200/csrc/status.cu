// Error reporting for the C ABI: a thread-local message behind dsmoe_last_error().
#include <stdarg.h>
#include <stdio.h>

#include "common.cuh"

namespace dsmoe {

static thread_local char g_err[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int cuda_status(const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", where, cudaGetErrorString(e));
    return DSMOE_ERR_CUDA;
  }
  return DSMOE_OK;
}

}  // namespace dsmoe

extern "C" const char* dsmoe_last_error(void) { return dsmoe::g_err; }
extern "C" int dsmoe_version(void) { return 1; }
