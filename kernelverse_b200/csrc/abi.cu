// Error reporting and version entry points of libkvb.so.
#include <cstdarg>
#include <cstdio>

#include "kvb_common.cuh"

namespace kvb {

static thread_local char g_last_error[512] = "no error";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return KVB_OK;
}

}  // namespace kvb

extern "C" const char* kvb_last_error(void) { return kvb::g_last_error; }
extern "C" int kvb_abi_version(void) { return 1; }
