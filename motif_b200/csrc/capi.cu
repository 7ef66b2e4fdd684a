// Status / error plumbing shared by every C-ABI entry point.
#include <cstdarg>
#include <cstdio>

#include "common.cuh"

namespace mb {

static thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(MB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  g_last_error[0] = '\0';
  return MB_OK;
}

}  // namespace mb

extern "C" const char* motif_b200_last_error(void) { return mb::g_last_error; }
extern "C" int motif_b200_abi_version(void) { return 1; }
