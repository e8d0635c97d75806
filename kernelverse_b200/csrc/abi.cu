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
static std::vector<WaitLimitSetter>& limit_setters() {
  static std::vector<WaitLimitSetter> v;
  return v;
}
void register_status_reader(StatusReader fn, WaitLimitSetter set_limit) {
  std::lock_guard<std::mutex> g(readers_mutex());
  readers().push_back(fn);
  limit_setters().push_back(set_limit);
}

namespace {
// Self-test of the bounded wait: one bulk copy of 16 bytes completes on barrier `landed`, then
// the kernel waits on barrier `never`, on which nothing ever arrives.  That wait gives up after
// the current limit (setting status bit 0), the kernel drains its copy (bounded wait on
// `landed`) and reports what it saw: out[0] = the copied word, out[1] = 1 if the wait on
// `never` gave up, out[2] = 1 if the drain completed.  One thread does it all.
__global__ void selftest_wait_kernel(const int4* src, int* out) {
  __shared__ __align__(16) int4 stage;
  __shared__ __align__(8) uint64_t landed, never;
  if (threadIdx.x != 0) return;
  mbar_init(&landed, 1);
  mbar_init(&never, 1);
  fence_mbar_init();
  mbar_arrive_expect_tx(&landed, 16);
  bulk_g2s(&stage, src, 16, &landed, policy_evict_first());
  const bool gave_up = !mbar_wait_bounded(&never, 0);
  const bool drained = mbar_wait_bounded(&landed, 0);
  out[0] = drained ? stage.x : 0;
  out[1] = gave_up ? 1 : 0;
  out[2] = drained ? 1 : 0;
}

// Self-test of div_rn (Markstein division): out[i] = a[i] / b[i] through a Divisor.  Elements
// with i % 4 in {2, 3} whose dividend is in the fast domain go through the packed path
// (div2_rn_fast, the dividend and its negation in one register), the others through div_rn.
__global__ void selftest_div_kernel(const float* a, const float* b, float* out, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const Divisor d = make_divisor(b[i]);
    if ((i & 2) && fabsf(a[i]) >= d.thresh) {
      const float2 q = f2_unpack(div2_rn_fast(f2_pack(a[i], -a[i]), d));
      out[i] = (q.y == -q.x) ? q.x : __int_as_float(0x7fc00000);   // lanes must agree (NaN otherwise)
    } else {
      out[i] = div_rn(a[i], d);
    }
  }
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

extern "C" int kvb_check_device(int reset) {
  const unsigned int v = kvb_device_status(reset);
  if (v & 0x80000000u) return KVB_E_LAUNCH;          // message already set by kvb_device_status
  if (v & kvb::kStatusWaitTimeout)
    return kvb::set_error(KVB_E_TIMEOUT, "a bounded device-side wait gave up (status %#x): outputs of that launch "
                          "are invalid", v);
  if (v & 6u)
    return kvb::set_error(KVB_E_INDEX, "an out-of-range slot, block-table entry or indptr range was skipped "
                          "(status %#x)", v);
  return KVB_OK;
}

extern "C" int kvb_set_wait_limit_ns(uint64_t limit_ns) {
  if (limit_ns == 0) limit_ns = kvb::kWaitLimitNs;
  std::lock_guard<std::mutex> g(kvb::readers_mutex());
  for (auto fn : kvb::limit_setters())
    if (fn(limit_ns)) return kvb::set_error(KVB_E_LAUNCH, "set_wait_limit_ns: cudaMemcpyToSymbol failed");
  return KVB_OK;
}

extern "C" int kvb_selftest_wait_timeout(const void* src16, int* out, void* stream) {
  if (!src16 || !out || (reinterpret_cast<uintptr_t>(src16) & 15))
    return kvb::set_error(KVB_E_ARG, "selftest_wait_timeout: src16 must be a 16-byte-aligned device pointer, out non-null");
  kvb::selftest_wait_kernel<<<1, 32, 0, kvb::as_stream(stream)>>>(static_cast<const int4*>(src16), out);
  return kvb::check_launch("selftest_wait_kernel");
}

extern "C" int kvb_selftest_div_rn(const float* a, const float* b, float* out, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!a || !b || !out))) return kvb::set_error(KVB_E_ARG, "selftest_div_rn: bad arguments");
  if (n == 0) return KVB_OK;
  const int blocks = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  kvb::selftest_div_kernel<<<blocks, 256, 0, kvb::as_stream(stream)>>>(a, b, out, n);
  return kvb::check_launch("selftest_div_kernel");
}

extern "C" const char* kvb_last_error(void) { return kvb::g_last_error; }
extern "C" int kvb_abi_version(void) { return 2; }
