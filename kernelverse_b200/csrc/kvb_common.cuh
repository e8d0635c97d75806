// Shared device/host helpers for the kvb sm_100a kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <utility>

#include "../../include/kvb.h"

namespace kvb {

// ------------------------------------------------------------------ host-side error reporting
// Sets the thread-local message returned by kvb_last_error() and returns `code`.
#if defined(__GNUC__)
__attribute__((format(printf, 2, 3)))
#endif
int set_error(int code, const char* fmt, ...);
// Checks the launch that was just issued (no synchronisation).
int check_launch(const char* what);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }
inline int dtype_size(int dt) {
  switch (dt) {
    case KVB_F32: case KVB_I32: return 4;
    case KVB_F16: case KVB_BF16: return 2;
    case KVB_I8: case KVB_U8: case KVB_E4M3: return 1;
    case KVB_I64: return 8;
    default: return 0;
  }
}
inline bool is_float_dtype(int dt) { return dt == KVB_F32 || dt == KVB_F16 || dt == KVB_BF16; }
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

constexpr float kInt8Max = 127.0f;
constexpr float kE4m3Max = 448.0f;
// operators/quantization/dynamic_scaled_int8_quant/helpers.py:8 -- 1 / (448 * 512) as float32
constexpr float kMinScalingFactor = 1.0f / (448.0f * 512.0f);

// ------------------------------------------------------------------ element conversion
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// Eight consecutive elements of T, moved with 128-bit (16-bit T) or 2x128-bit (float) accesses.
template <typename T> struct Vec8 {
  static constexpr int kBytes = 8 * sizeof(T);
  static constexpr int kWords = kBytes / 16;   // uint4 words: 1 for 16-bit types, 2 for float
  uint4 w[kWords];
  __device__ __forceinline__ void load(const T* p) {
    const uint4* s = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = __ldg(s + i);
  }
  __device__ __forceinline__ void load_stream(const T* p) {   // read-once data: evict-first
    const uint4* s = reinterpret_cast<const uint4*>(p);
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = __ldcs(s + i);
  }
  __device__ __forceinline__ void store(T* p) const {
    uint4* d = reinterpret_cast<uint4*>(p);
#pragma unroll
    for (int i = 0; i < kWords; ++i) d[i] = w[i];
  }
  __device__ __forceinline__ float get(int i) const {
    const T* e = reinterpret_cast<const T*>(w);
    return Elem<T>::to_f(e[i]);
  }
  __device__ __forceinline__ void set(int i, float v) {
    T* e = reinterpret_cast<T*>(w);
    e[i] = Elem<T>::from_f(v);
  }
  // All eight elements as float32 / from float32 (round-to-nearest-even), using packed
  // conversions for the 16-bit types.
  __device__ __forceinline__ void unpack(float f[8]) const;
  __device__ __forceinline__ void pack(const float f[8]);
};

template <> __device__ __forceinline__ void Vec8<__nv_bfloat16>::unpack(float f[8]) const {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}
template <> __device__ __forceinline__ void Vec8<__nv_bfloat16>::pack(const float f[8]) {
  uint32_t* u = reinterpret_cast<uint32_t*>(w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    u[i] = *reinterpret_cast<uint32_t*>(&h);
  }
}
template <> __device__ __forceinline__ void Vec8<__half>::unpack(float f[8]) const {
  const __half2* h = reinterpret_cast<const __half2*>(w);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
template <> __device__ __forceinline__ void Vec8<__half>::pack(const float f[8]) {
  __half2* h = reinterpret_cast<__half2*>(w);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
}
template <> __device__ __forceinline__ void Vec8<float>::unpack(float f[8]) const {
  const float* e = reinterpret_cast<const float*>(w);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = e[i];
}
template <> __device__ __forceinline__ void Vec8<float>::pack(const float f[8]) {
  float* e = reinterpret_cast<float*>(w);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = f[i];
}

// ------------------------------------------------------------------ reductions
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// Max over `width` consecutive lanes (width a power of two <= 32).
__device__ __forceinline__ float group_max(float v, int width) {
  for (int o = width >> 1; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide reduction; `scratch` holds >= 32 floats.  All threads get the result.
template <bool kMax>
__device__ __forceinline__ float block_reduce(float v, float* scratch) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  v = kMax ? warp_max(v) : warp_sum(v);
  __syncthreads();               // scratch may still be read by a previous reduction
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  float r = lane < nwarps ? scratch[lane] : (kMax ? 0.0f : 0.0f);
  r = kMax ? warp_max(r) : warp_sum(r);
  return r;
}

// Warp max of non-negative floats with the sm_100a redux instruction (one instruction).
__device__ __forceinline__ float warp_max_redux(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
}

// Block reduction with a single barrier.  `buf` (>= 32 floats) must differ from the
// buffer of the previous reduction of the block: that reduction's barrier then already
// guarantees its buffer has been read, so consecutive reductions alternate two buffers.
template <bool kMax>
__device__ __forceinline__ float block_reduce_1bar(float v, float* buf) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  v = kMax ? warp_max_redux(v) : warp_sum(v);
  if (lane == 0) buf[warp] = v;
  __syncthreads();
  float r = lane < nwarps ? buf[lane] : 0.0f;
  return kMax ? warp_max_redux(r) : warp_sum(r);
}

// ------------------------------------------------------------------ programmatic dependent launch
// A kernel launched with launch_pdl may start (and run its set-up) while the previous kernel in
// the stream finishes; pdl_wait() returns once that kernel has completed and its memory is
// visible, so everything global is read or written after it.  pdl_trigger() lets the next such
// kernel be scheduled once every CTA of this grid has issued it (or exited); that kernel may then
// run its own set-up, but it too reads and writes nothing global before its pdl_wait(), which
// is what makes an early trigger safe.  Both return at once without a dependent launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Bulk prefetch of [src, src + bytes) into L2 (src and bytes multiples of 16).  It returns no
// data to the SM and L2 is where every SM's writes meet, so issuing it before pdl_wait() is
// safe: a line the previous grid writes afterwards is updated in L2, and the loads that read it
// are issued after the wait.
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// ------------------------------------------------------------------ quantisation primitives
// Correctly rounded a / b from a precomputed y = RN(1/b), by Markstein's method
// (P. Markstein, "IA-64 and Elementary Functions", 2000, Thm. 8.10): with y the
// correctly rounded reciprocal and q0 = RN(a*y) within an ulp of a/b, the remainder
// r = a - b*q0 is exact in one FMA and q1 = RN(q0 + r*y) is the round-to-nearest
// quotient.  The theorem assumes that nothing underflows or overflows in the
// intermediate steps.  Domain of the fast path: 2^-120 <= b <= 2^120 and
// max(2^-96, b * 2^-100) <= |a| <= 2^100 * b -- the quantisers always have
// |a| <= 448 * b because b is the group's amax / 448 (or / 127) or larger.
// Below the lower bound (zero included, which keeps the quotient's sign) the
// IEEE division is used; when b is out of range every element of the group is.
// A divisor is set up once per quantisation group and reused for every element.
// tests/test_gpu_numerics.py checks div_rn against CUDA's __fdiv_rn bit for bit.
struct Divisor {
  float b, y, thresh;
};
__device__ __forceinline__ Divisor make_divisor(float b) {
  Divisor d;
  d.b = b;
  d.y = __frcp_rn(b);
  d.thresh = (b >= 0x1p-120f && b <= 0x1p120f) ? fmaxf(0x1p-96f, b * 0x1p-100f) : __int_as_float(0x7f800000);
  return d;
}
// Fast path only: the caller has checked |a| >= d.thresh.
__device__ __forceinline__ float div_rn_fast(float a, const Divisor& d) {
  const float q0 = __fmul_rn(a, d.y);
  const float r = __fmaf_rn(-d.b, q0, a);
  return __fmaf_rn(r, d.y, q0);
}
__device__ __forceinline__ float div_rn(float a, const Divisor& d) {
  if (fabsf(a) < d.thresh) return __fdiv_rn(a, d.b);
  return div_rn_fast(a, d);
}

// ------------------------------------------------------------------ packed float32 (sm_100a)
// Two float32 lanes in one 64-bit register for the packed FMUL2 / FFMA2 / FADD2 instructions
// (PTX mul/fma/add .rn.f32x2): each lane is rounded exactly as the scalar .rn instruction.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// div_rn_fast on two dividends at once: the same three correctly rounded steps per lane.
__device__ __forceinline__ uint64_t div2_rn_fast(uint64_t a, const Divisor& d) {
  const uint64_t y = f2_pack(d.y, d.y), nb = f2_pack(-d.b, -d.b);
  uint64_t q0, r, q1;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(q0) : "l"(a), "l"(y));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(nb), "l"(q0), "l"(a));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(q1) : "l"(r), "l"(y), "l"(q0));
  return q1;
}

// int8 code: round-half-even of the IEEE float32 quotient x / scale, clamped to +-127.
// kChecked = false: the caller has verified |x| >= d.thresh for the values passed.
template <bool kChecked = true>
__device__ __forceinline__ int8_t quant_int8(float x, const Divisor& d) {
  float q = rintf(kChecked ? div_rn(x, d) : div_rn_fast(x, d));
  q = fminf(fmaxf(q, -kInt8Max), kInt8Max);
  return static_cast<int8_t>(__float2int_rn(q));
}

// True when the divisor lies in the Markstein domain (2^-120 <= b <= 2^120).  If in addition b
// is a group's amax / qmax (qmax = 127 or 448, possibly rounded to a 16-bit type) or larger,
// the unchecked quantisers below are exact for every value of the group: values with
// |x| >= d.thresh get the correctly rounded quotient, and smaller ones have |x / b| < 2^-100,
// whose int8 or e4m3 code is (signed) zero however the last bit of the quotient falls.
__device__ __forceinline__ bool fast_divisor(const Divisor& d) { return d.thresh < __int_as_float(0x7f800000); }

// int8 codes of four values under fast_divisor(d), |x| <= 127 * b * (1 + 2^-8):
//  * |quotient| <= 127.25, so round-half-even then clamp to +-127 is round-half-even alone;
//  * rounding is the addition of 1.5 * 2^23 (one round-to-nearest-even add puts the integer
//    in the low mantissa bits; its low byte is the two's-complement code), which replaces a
//    quarter-rate float-to-int conversion, and byte permutes pack four codes into a word
//    (a0 in the low byte).
__device__ __forceinline__ uint32_t quant4_fast(float a0, float a1, float a2, float a3, const Divisor& d) {
  constexpr float kRound = 12582912.0f;   // 1.5 * 2^23
  const uint32_t b0 = __float_as_uint(__fadd_rn(div_rn_fast(a0, d), kRound));
  const uint32_t b1 = __float_as_uint(__fadd_rn(div_rn_fast(a1, d), kRound));
  const uint32_t b2 = __float_as_uint(__fadd_rn(div_rn_fast(a2, d), kRound));
  const uint32_t b3 = __float_as_uint(__fadd_rn(div_rn_fast(a3, d), kRound));
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// quant4_fast with packed arithmetic: the four codes of (a0, a1) and (a2, a3), each pair given
// as one packed register; identical results.
__device__ __forceinline__ uint32_t quant4_fast_x2(uint64_t a01, uint64_t a23, const Divisor& d) {
  const uint64_t k = f2_pack(12582912.0f, 12582912.0f);   // 1.5 * 2^23 in both lanes
  uint64_t r01, r23;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r01) : "l"(div2_rn_fast(a01, d)), "l"(k));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r23) : "l"(div2_rn_fast(a23, d)), "l"(k));
  const uint32_t b0 = (uint32_t)r01, b1 = (uint32_t)(r01 >> 32), b2 = (uint32_t)r23, b3 = (uint32_t)(r23 >> 32);
  return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// quant_e4m3x2<false> on a packed pair (low lane in the low byte), the quotients computed with
// packed arithmetic; identical results.
__device__ __forceinline__ uint16_t quant_e4m3x2_fast_x2(uint64_t ab, const Divisor& d) {
  const float2 q = f2_unpack(div2_rn_fast(ab, d));
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(q, __NV_SATFINITE, __NV_E4M3));
}

// e4m3fn codes of clamp(x / scale, +-448) for two values (a in the low byte).  The
// hardware conversion (cvt.rn.satfinite.e4m3x2.f32) rounds to nearest even and
// saturates to +-448, which is exactly clamp-then-cast.
template <bool kChecked = true>
__device__ __forceinline__ uint16_t quant_e4m3x2(float a, float b, const Divisor& d) {
  const float qa = kChecked ? div_rn(a, d) : div_rn_fast(a, d);
  const float qb = kChecked ? div_rn(b, d) : div_rn_fast(b, d);
  return static_cast<uint16_t>(__nv_cvt_float2_to_fp8x2(make_float2(qa, qb), __NV_SATFINITE, __NV_E4M3));
}

}  // namespace kvb
