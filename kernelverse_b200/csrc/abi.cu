// Error reporting and version entry points of libkvb.so.
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <vector>

#include "kvb_common.cuh"
#include "kvb_async.cuh"

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

static std::mutex& readers_mutex() {
  static std::mutex m;
  return m;
}
static std::vector<StatusReader>& readers() {
  static std::vector<StatusReader> v;
  return v;
}
void register_status_reader(StatusReader fn) {
  std::lock_guard<std::mutex> g(readers_mutex());
  readers().push_back(fn);
}

namespace {
// Self-test of div_rn (Markstein division): out[i] = a[i] / b[i] through a Divisor.
__global__ void selftest_div_kernel(const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = div_rn(a[i], make_divisor(b[i]));
}
}  // namespace

}  // namespace kvb

extern "C" unsigned int kvb_device_status(int reset) {
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    kvb::set_error(KVB_E_LAUNCH, "device_status: %s", cudaGetErrorString(e));
    return 0x80000000u;
  }
  unsigned int v = 0;
  std::lock_guard<std::mutex> g(kvb::readers_mutex());
  for (auto fn : kvb::readers()) v |= fn(reset != 0);
  return v;
}

extern "C" int kvb_selftest_div_rn(const float* a, const float* b, float* out, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!a || !b || !out))) return kvb::set_error(KVB_E_ARG, "selftest_div_rn: bad arguments");
  if (n == 0) return KVB_OK;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  kvb::selftest_div_kernel<<<blocks, 256, 0, kvb::as_stream(stream)>>>(a, b, out, n);
  return kvb::check_launch("selftest_div_kernel");
}

extern "C" const char* kvb_last_error(void) { return kvb::g_last_error; }
extern "C" int kvb_abi_version(void) { return 1; }
