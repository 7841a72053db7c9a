// Status reporting shared by every C-ABI entry point.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "q4b.h"

namespace q4b {

static thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("Q4B_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(Q4B_ELAUNCH, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return Q4B_OK;
}

}  // namespace q4b

extern "C" const char* q4b_last_error(void) { return q4b::g_last_error.c_str(); }

extern "C" int q4b_abi_version(void) { return 1; }
