// mbarrier / bulk-copy (cp.async.bulk) primitives and bounded waits for sm_100a kernels.
//
// Every wait on an mbarrier is bounded by wall time (%globaltimer): a wait that
// gives up records a code in the translation unit's device status word and
// returns false, so a kernel can drain and exit instead of hanging the GPU.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace kvb {

// Device status word of the including translation unit (0 = ok).  Read and reset
// from the host with kvb_device_status().
static __device__ unsigned int g_tu_status = 0;

constexpr unsigned int kStatusWaitTimeout = 1u;     // an mbarrier wait ran out of time
constexpr uint64_t kWaitLimitNs = 2000000000ull;    // 2 s: the default bound of every wait

// The bound itself, per translation unit; kvb_set_wait_limit_ns() changes it in all of them
// (a test lowers it to make a wait run out quickly).  Read only once a wait has not
// completed at its first try.
static __device__ uint64_t g_wait_limit_ns = kWaitLimitNs;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (bulk copies / TMA).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of `bar` to complete; gives up after g_wait_limit_ns.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = *(volatile uint64_t*)&g_wait_limit_ns;
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 255u && globaltimer_ns() - t0 > limit) {
      atomicOr(&g_tu_status, kStatusWaitTimeout);
      return false;
    }
  }
}

// 1-D bulk copy global -> shared, completion signalled on `bar` (complete_tx).  dst, src and
// bytes must be multiples of 16.  `policy` is an L2 cache-policy descriptor (createpolicy).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

}  // namespace kvb

// Host side: every translation unit that includes this header registers a reader of its
// status word, so kvb_device_status() can report and reset all of them.
namespace kvb {
using StatusReader = unsigned int (*)(bool reset);
using WaitLimitSetter = int (*)(uint64_t ns);
void register_status_reader(StatusReader fn, WaitLimitSetter set_limit);
namespace {
unsigned int read_tu_status(bool reset) {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_tu_status, sizeof(v)) != cudaSuccess) return 0xffffffffu;
  if (reset && v) {
    const unsigned int zero = 0;
    cudaMemcpyToSymbol(g_tu_status, &zero, sizeof(zero));
  }
  return v;
}
int set_tu_wait_limit(uint64_t ns) {
  return cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof(ns)) == cudaSuccess ? 0 : 1;
}
struct StatusRegistrar {
  StatusRegistrar() { register_status_reader(&read_tu_status, &set_tu_wait_limit); }
};
static StatusRegistrar g_status_registrar;
}  // namespace
}  // namespace kvb
