// Error reporting for the C ABI: a per-thread message plus an integer status.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

static thread_local char g_last_error[512] = "";

int q35_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int q35_check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return q35_fail(Q35_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return Q35_OK;
}

extern "C" const char* q35_last_error(void) { return g_last_error; }
extern "C" int q35_abi_version(void) { return 1; }
