// Dynamic int8 quantisation kernels: per-tensor and per-(token, group).
//
// Memory-bound: every kernel reads x once from HBM (the per-tensor form reads it
// twice, the second pass normally from L2) and writes 1 byte per element plus
// one float32 scale per group.  Loads are 128-bit, group amax reductions use
// warp shuffles (groups of <= 256 elements live inside one warp) or one block
// reduction per group (larger groups, e.g. whole tokens), and the quotient is
// an IEEE division so the codes are bit-identical to the reference's
// round(x / scale).
#include "kvb_common.cuh"

namespace kvb {
namespace {

// Packs eight int8 codes of one Vec8 into a 64-bit word (little-endian order); the general
// path for any divisor (IEEE division below the Markstein threshold, clamp to +-127).
template <typename T>
__device__ __forceinline__ uint2 quant8_checked(const Vec8<T>& v, const Divisor& d) {
  float f[8];
  v.unpack(f);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) lo |= (uint32_t)(uint8_t)quant_int8<true>(f[i], d) << (8 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) hi |= (uint32_t)(uint8_t)quant_int8<true>(f[4 + i], d) << (8 * i);
  return make_uint2(lo, hi);
}

template <typename T>
__device__ __forceinline__ uint2 quant8_fast(const Vec8<T>& v, const Divisor& d) {
  float f[8];
  v.unpack(f);
  return make_uint2(quant4_fast(f[0], f[1], f[2], f[3], d), quant4_fast(f[4], f[5], f[6], f[7], d));
}

template <typename T>
__device__ __forceinline__ float vec_amax(const Vec8<T>& v) {
  float f[8], m = 0.0f;
  v.unpack(f);
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
  return m;
}
// ---------------------------------------------------------------- per-tensor
// Two kernels chained as programmatic dependents, with no state to zero between calls: pass 1
// writes one partial amax per CTA, pass 2 reduces the partials and quantises, reading x again
// (from L2 when x fits there, which it normally does right after pass 1).
constexpr int kTensorThreads = 256;
constexpr int kTensorMaxBlocks = 2048;    // partial maxima the workspace holds
// Vec8s a thread keeps in flight: 8 of 16 bytes for 16-bit inputs, 4 of 32 for float.
template <typename T> constexpr int tensor_unroll() { return sizeof(T) == 4 ? 4 : 8; }

// Pass 1: partial[blockIdx.x] = amax(|x|) over the CTA's share of x.
template <typename T>
__global__ void __launch_bounds__(kTensorThreads, 4) tensor_amax_kernel(const T* __restrict__ x, int64_t numel,
                                                                     int64_t nvec, float* __restrict__ partial) {
  __shared__ float scratch[32];
  constexpr int U = tensor_unroll<T>();
  const int64_t stride = (int64_t)gridDim.x * kTensorThreads;
  pdl_trigger();
  if (threadIdx.x < U) {   // the CTA's first round of x into L2 while the previous kernel finishes
    const int64_t v = (int64_t)blockIdx.x * kTensorThreads + threadIdx.x * stride;
    if (v < nvec) prefetch_l2_bulk(x + v * 8, (uint32_t)(std::min<int64_t>(kTensorThreads, nvec - v) * Vec8<T>::kBytes));
  }
  pdl_wait();
  float m = 0.0f;
  for (int64_t v = (int64_t)blockIdx.x * kTensorThreads + threadIdx.x; v < nvec; v += U * stride) {
    Vec8<T> a[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v + u * stride < nvec) a[u].load(x + (v + u * stride) * 8);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v + u * stride < nvec) m = fmaxf(m, vec_amax(a[u]));
  }
  for (int64_t i = nvec * 8 + (int64_t)blockIdx.x * kTensorThreads + threadIdx.x; i < numel; i += stride)
    m = fmaxf(m, fabsf(Elem<T>::to_f(x[i])));
  m = block_reduce<true>(m, scratch);
  if (threadIdx.x == 0) partial[blockIdx.x] = m;
}

// scale = max(float(T(amax / 127)), MIN_SCALING_FACTOR): amax / 127 is evaluated in float32
// and rounded to the input dtype, as the reference's input-dtype arithmetic does
// (dynamic_scaled_int8_quant.py:22).
template <typename T>
__device__ __forceinline__ float tensor_scale(float amax) {
  return fmaxf(Elem<T>::to_f(Elem<T>::from_f(__fdiv_rn(amax, kInt8Max))), kMinScalingFactor);
}

// Pass 2: amax = max over the npartial partials of pass 1; q = round(clamp(x / scale)).
template <typename T>
__global__ void __launch_bounds__(kTensorThreads, 4) tensor_quant_kernel(const T* __restrict__ x, int64_t numel,
                                                                      int64_t nvec, const float* partial, int npartial,
                                                                      int8_t* __restrict__ q,
                                                                      float* __restrict__ scale_out,
                                                                      int32_t* __restrict__ azp_out) {
  __shared__ float scratch[32];
  pdl_trigger();
  pdl_wait();
  float m = 0.0f;
  for (int i = threadIdx.x; i < npartial; i += kTensorThreads) m = fmaxf(m, __ldcg(partial + i));
  const float scale = tensor_scale<T>(block_reduce<true>(m, scratch));
  const Divisor d = make_divisor(scale);
  const bool fast = fast_divisor(d);
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    *scale_out = scale;
    if (azp_out) *azp_out = 0;
  }
  constexpr int U = tensor_unroll<T>();
  const int64_t stride = (int64_t)gridDim.x * kTensorThreads;
  uint2* q8 = reinterpret_cast<uint2*>(q);
  for (int64_t v = (int64_t)blockIdx.x * kTensorThreads + threadIdx.x; v < nvec; v += U * stride) {
    Vec8<T> a[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v + u * stride < nvec) a[u].load(x + (v + u * stride) * 8);
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v + u * stride < nvec) q8[v + u * stride] = fast ? quant8_fast(a[u], d) : quant8_checked(a[u], d);
  }
  for (int64_t i = nvec * 8 + (int64_t)blockIdx.x * kTensorThreads + threadIdx.x; i < numel; i += stride)
    q[i] = quant_int8(Elem<T>::to_f(x[i]), d);
}

// ---------------------------------------------------------------- static scale
// q = clamp(round_half_even(x / max(scale, MIN_SCALE) + azp), +-127) in float32
// (static_scaled_int8_quant.py:28-32 in its float32 correctness mode).  The scale is not an
// amax here, so x is first clamped to +-(|azp| + 256) * s: beyond that the result is +-127
// either way, and inside it the quotient is in the FMA-division domain (values below the
// division threshold still give quotients under 2^-100, which round away against azp).
__device__ __forceinline__ uint32_t static_code4(const float (&f)[8], int base, const Divisor& d, float lim, float z) {
  constexpr float kRound = 12582912.0f;   // 1.5 * 2^23: rounds half to even into the low byte
  uint32_t b[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float xc = fminf(fmaxf(f[base + i], -lim), lim);
    const float v = fminf(fmaxf(__fadd_rn(div_rn_fast(xc, d), z), -kInt8Max), kInt8Max);
    b[i] = __float_as_uint(__fadd_rn(v, kRound));
  }
  return __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
}
__device__ __forceinline__ int8_t static_code_checked(float x, float s, float z) {
  const float v = fminf(fmaxf(__fadd_rn(__fdiv_rn(x, s), z), -kInt8Max), kInt8Max);
  return (int8_t)__float2int_rn(v);
}

template <typename T>
__global__ void __launch_bounds__(256) static_quant_kernel(const T* __restrict__ x, int64_t numel, int64_t nvec,
                                                           const float* __restrict__ scale,
                                                           const int32_t* __restrict__ azp, int8_t* __restrict__ q) {
  const float s = fmaxf(*scale, kMinScalingFactor);
  const float z = azp ? (float)*azp : 0.0f;
  const Divisor d = make_divisor(s);
  const bool fast = fast_divisor(d) && fabsf(z) <= 0x1p90f;
  const float lim = (fabsf(z) + 256.0f) * s;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += stride) {
    Vec8<T> a;
    a.load_stream(x + v * 8);
    float f[8];
    a.unpack(f);
    uint2 out;
    if (fast) {
      out = make_uint2(static_code4(f, 0, d, lim, z), static_code4(f, 4, d, lim, z));
    } else {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lo |= (uint32_t)(uint8_t)static_code_checked(f[i], s, z) << (8 * i);
        hi |= (uint32_t)(uint8_t)static_code_checked(f[4 + i], s, z) << (8 * i);
      }
      out = make_uint2(lo, hi);
    }
    reinterpret_cast<uint2*>(q)[v] = out;
  }
  for (int64_t i = nvec * 8 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < numel; i += stride)
    q[i] = static_code_checked(Elem<T>::to_f(x[i]), s, z);
}

// ---------------------------------------------------------------- per-group, small groups
// 8-element vectors, one per lane of a warp sub-chunk; a group of G = 8*L elements spans L
// consecutive lanes (L a power of two <= 32), so its amax is an L-lane shuffle reduction.
// Each warp takes U sub-chunks of 32 vectors per step (whole groups, since lanes divides 32) and
// issues all their loads before reducing any, so U loads per thread are in flight.
template <typename T, int U>
__global__ void __launch_bounds__(256) group_quant_subwarp_kernel(const T* __restrict__ x, int64_t nvec, int lanes,
                                                                  float eps, int8_t* __restrict__ q,
                                                                  float* __restrict__ scales) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  // The loop bound is warp-uniform so every lane joins each shuffle.
  for (int64_t w = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w * 32 * U < nvec; w += nwarps) {
    const int64_t v0 = w * 32 * U + lane;
    Vec8<T> a[U];
    float m[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v0 + u * 32 < nvec) a[u].load_stream(x + (v0 + u * 32) * 8);
#pragma unroll
    for (int u = 0; u < U; ++u) m[u] = v0 + u * 32 < nvec ? vec_amax(a[u]) : 0.0f;
#pragma unroll
    for (int u = 0; u < U; ++u) m[u] = group_max(m[u], lanes);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t v = v0 + u * 32;
      if (v < nvec) {
        const float scale = fmaxf(__fdiv_rn(m[u], kInt8Max), eps);
        const Divisor d = make_divisor(scale);
        reinterpret_cast<uint2*>(q)[v] = fast_divisor(d) ? quant8_fast(a[u], d) : quant8_checked(a[u], d);
        if ((v & (lanes - 1)) == 0) scales[v / lanes] = scale;
      }
    }
  }
}

// ---------------------------------------------------------------- per-group, large groups
// One CTA per group (e.g. one token row); the group stays in registers between the
// amax reduction and the quantisation, so x is read from HBM exactly once.  kMinBlocks
// bounds the registers so that a whole BASELINE-sized batch (2048 rows of 128 threads)
// is resident in one wave.
template <typename T, int VPT, int kMaxThreads, int kMinBlocks>
__global__ void __launch_bounds__(kMaxThreads, kMinBlocks)
    group_quant_rowblock_kernel(const T* __restrict__ x, int group_vecs, float eps, int8_t* __restrict__ q,
                                float* __restrict__ scales) {
  __shared__ float scratch[32];
  pdl_trigger();
  pdl_wait();            // launched as a programmatic dependent (launch_pdl)
  const int64_t g = blockIdx.x;
  const T* xg = x + g * group_vecs * 8;
  Vec8<T> a[VPT];
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = threadIdx.x + j * blockDim.x;
    if (v < group_vecs) a[j].load_stream(xg + (int64_t)v * 8);
  }
#pragma unroll
  for (int j = 0; j < VPT; ++j)
    if (threadIdx.x + j * blockDim.x < group_vecs) m = fmaxf(m, vec_amax(a[j]));
  m = block_reduce_1bar<true>(m, scratch);   // the block's only reduction
  const float scale = fmaxf(__fdiv_rn(m, kInt8Max), eps);
  const Divisor d = make_divisor(scale);
  uint2* qg = reinterpret_cast<uint2*>(q + g * group_vecs * 8);
  if (fast_divisor(d)) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = threadIdx.x + j * blockDim.x;
      if (v < group_vecs) qg[v] = quant8_fast(a[j], d);
    }
  } else {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = threadIdx.x + j * blockDim.x;
      if (v < group_vecs) qg[v] = quant8_checked(a[j], d);
    }
  }
  if (threadIdx.x == 0) scales[g] = scale;
}

// ---------------------------------------------------------------- per-group, long groups, teams
// CTAs of 512 threads form 16 / WG teams of WG warps; each team quantises one group (a token
// row for per-token quantisation), so a CTA covers several groups and the launch needs 4-16x
// fewer CTAs than one CTA per group (a dependent launch of 2048 CTAs costs ~1.7 us more than
// one of a few hundred on a B200).  Every thread loads its VPT vectors of the group with
// 128-bit streaming loads before any arithmetic.  At BASELINE sizes the kernel is bound by
// issue as much as by DRAM, so the instruction count shapes it: the elements are converted to
// float32 once (shared by the amax and the codes), the amax is one team reduction (a named
// barrier), amax / 127 uses the FMA-corrected division with the divisor 127, and the codes use
// packed float32 arithmetic (two lanes per instruction): about four instructions per element
// plus a fixed cost per warp, which four warps of four vectors a thread keep small.
constexpr int kTeamThreads = 512;

__device__ __forceinline__ uint2 quant8_fast_x2(const float (&f)[8], const Divisor& d) {
  return make_uint2(quant4_fast_x2(f2_pack(f[0], f[1]), f2_pack(f[2], f[3]), d),
                    quant4_fast_x2(f2_pack(f[4], f[5]), f2_pack(f[6], f[7]), d));
}

// The general path from float32 values: correctly rounded quotient for any divisor, clamped.
__device__ __forceinline__ uint2 quant8_checked_f(const float (&f)[8], const Divisor& d) {
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) lo |= (uint32_t)(uint8_t)quant_int8<true>(f[i], d) << (8 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) hi |= (uint32_t)(uint8_t)quant_int8<true>(f[4 + i], d) << (8 * i);
  return make_uint2(lo, hi);
}

__device__ __forceinline__ void named_bar_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <typename T, int VPT, int WG, int kMinBlocks>
__global__ void __launch_bounds__(kTeamThreads, kMinBlocks)
    group_quant_teams_kernel(const T* __restrict__ x, int64_t ngroups, int gvec, float eps, int8_t* __restrict__ q,
                             float* __restrict__ scales) {
  constexpr int kTeams = kTeamThreads / 32 / WG;
  constexpr int kThreads = WG * 32;           // threads of a team
  __shared__ float red[kTeams][WG];
  const int tid = threadIdx.x, lane = tid & 31;
  const int team = tid / kThreads, ttid = tid % kThreads;
  const int64_t g = (int64_t)blockIdx.x * kTeams + team;
  const bool live = g < ngroups;              // team-uniform
  pdl_trigger();
  pdl_wait();            // launched as a programmatic dependent (launch_pdl)
  Vec8<T> a[VPT];
  const T* xg = x + g * gvec * 8;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = ttid + j * kThreads;
    if (live && v < gvec) a[j].load_stream(xg + (int64_t)v * 8);
  }
  float f[VPT][8];
  float m = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    a[j].unpack(f[j]);
    if (live && ttid + j * kThreads < gvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(f[j][e]));
    }
  }
  m = warp_max_redux(m);
  if (WG > 1) {
    if (lane == 0) red[team][ttid >> 5] = m;
    named_bar_sync(1 + team, kThreads);      // one reduction per team and launch: one buffer suffices
    m = warp_max_redux(lane < WG ? red[team][lane] : 0.0f);
  }
  if (!live) return;
  const float scale = fmaxf(div_rn(m, make_divisor(kInt8Max)), eps);   // == IEEE m / 127
  const Divisor d = make_divisor(scale);
  uint2* qg = reinterpret_cast<uint2*>(q + g * gvec * 8);
  if (fast_divisor(d)) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = ttid + j * kThreads;
      if (v < gvec) qg[v] = quant8_fast_x2(f[j], d);
    }
  } else {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = ttid + j * kThreads;
      if (v < gvec) qg[v] = quant8_checked(a[j], d);
    }
  }
  if (ttid == 0) scales[g] = scale;
}

// ---------------------------------------------------------------- per-group, 16-bit, rolling
// The team kernel's work as a persistent loop with a one-group prefetch: CTAs of 512 threads
// (two resident per SM, grid = 2 x SMs) form 16 / WG teams; a team walks the groups
// g, g + (all teams), ... and issues the loads of its next group as soon as the current group's
// data has arrived (right after its amax), so while the team reduces, divides and stores one
// group the next one is in flight.  Keeping one group in flight per team rather than all of
// them lets early groups land early: with every group requested at once the DRAM interleaves
// them and all land near the end, after which the arithmetic is a serial tail.  For 16-bit
// inputs with two vectors a thread (the data of two groups fits the 64 registers a thread has).
// kFull: every group is exactly VPT x (team threads) vectors (power-of-two rows such as the
// BASELINE first config), so no per-vector bounds predicate is needed.
template <typename T, int VPT, int WG, bool kFull>
__global__ void __launch_bounds__(kTeamThreads, 2)
    group_quant_rolling_kernel(const T* __restrict__ x, int64_t ngroups, int gvec_arg, float eps,
                               int8_t* __restrict__ q, float* __restrict__ scales) {
  constexpr int kTeams = kTeamThreads / 32 / WG;
  constexpr int kThreads = WG * 32;
  const int gvec = kFull ? VPT * kThreads : gvec_arg;
  __shared__ float red[kTeams][2][WG];        // per team, alternating buffers of consecutive reductions
  const int tid = threadIdx.x, lane = tid & 31;
  const int team = tid / kThreads, ttid = tid % kThreads;
  const int64_t stride = (int64_t)gridDim.x * kTeams;
  int64_t g = (int64_t)blockIdx.x * kTeams + team;   // team-uniform from here on
  pdl_trigger();
  // This team's rows start on their way from DRAM into L2 while the previous grid finishes
  // (prefetch_l2_bulk may precede pdl_wait; [2048, 4096] back to back: 5.39 -> 5.25 us).
  if (ttid == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0)
    for (int64_t gg = g; gg < ngroups; gg += stride) prefetch_l2_bulk(x + gg * gvec * 8, (uint32_t)gvec * 16u);
  pdl_wait();            // launched as a programmatic dependent (launch_pdl)
  Vec8<T> cur[VPT], nxt[VPT];
  if (g < ngroups) {
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = ttid + j * kThreads;
      if (v < gvec) cur[j].load_stream(x + g * gvec * 8 + (int64_t)v * 8);
    }
  }
  for (int it = 0; g < ngroups; g += stride, ++it) {
    float f[VPT][8];
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      cur[j].unpack(f[j]);
      if (ttid + j * kThreads < gvec) {
#pragma unroll
        for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(f[j][e]));
      }
    }
    const int64_t gn = g + stride;       // prefetch: this group's data has arrived (used above)
    if (gn < ngroups) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = ttid + j * kThreads;
        if (v < gvec) nxt[j].load_stream(x + gn * gvec * 8 + (int64_t)v * 8);
      }
    }
    m = warp_max_redux(m);
    if (WG > 1) {
      float* buf = red[team][it & 1];
      if (lane == 0) buf[ttid >> 5] = m;
      named_bar_sync(1 + team, kThreads);
      m = warp_max_redux(lane < WG ? buf[lane] : 0.0f);
    }
    const float scale = fmaxf(div_rn(m, make_divisor(kInt8Max)), eps);   // == IEEE m / 127
    const Divisor d = make_divisor(scale);
    uint2* qg = reinterpret_cast<uint2*>(q + g * gvec * 8);
    if (fast_divisor(d)) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = ttid + j * kThreads;
        if (v < gvec) qg[v] = quant8_fast_x2(f[j], d);
      }
    } else {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = ttid + j * kThreads;
        if (v < gvec) qg[v] = quant8_checked_f(f[j], d);
      }
    }
    if (ttid == 0) scales[g] = scale;
#pragma unroll
    for (int j = 0; j < VPT; ++j) cur[j] = nxt[j];
  }
}

// ---------------------------------------------------------------- any shape / alignment
// One warp per group, two passes over global memory (correctness path for odd sizes).
template <typename T>
__global__ void __launch_bounds__(256) group_quant_scalar_kernel(const T* __restrict__ x, int64_t ngroups,
                                                                 int64_t group_size, float eps,
                                                                 int8_t* __restrict__ q, float* __restrict__ scales) {
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int lane = threadIdx.x & 31;
  for (int64_t g = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < ngroups; g += warps) {
    const T* xg = x + g * group_size;
    float m = 0.0f;
    for (int64_t i = lane; i < group_size; i += 32) m = fmaxf(m, fabsf(Elem<T>::to_f(xg[i])));
    m = warp_max(m);
    const float scale = fmaxf(__fdiv_rn(m, kInt8Max), eps);
    const Divisor d = make_divisor(scale);
    for (int64_t i = lane; i < group_size; i += 32) q[g * group_size + i] = quant_int8(Elem<T>::to_f(xg[i]), d);
    if (lane == 0) scales[g] = scale;
  }
}

int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// CTAs of both per-tensor passes: enough for one unrolled round a thread, at most 4 a SM (all
// resident at once) and kTensorMaxBlocks.
int tensor_blocks(int64_t work, int unroll) {
  const int64_t per_block = (int64_t)kTensorThreads * unroll;
  const int64_t cap = std::min<int64_t>(kTensorMaxBlocks, (int64_t)sm_count() * 4);
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + per_block - 1) / per_block, cap));
}

template <typename T>
int launch_tensor_quant(const void* xv, int64_t numel, int8_t* q, float* scale, int32_t* azp, float* partial,
                        cudaStream_t st) {
  const T* x = static_cast<const T*>(xv);
  const bool vec = aligned16(x) && aligned8(q);
  const int64_t nvec = vec ? numel / 8 : 0;
  const int blocks = tensor_blocks(nvec > 0 ? nvec : numel, nvec > 0 ? tensor_unroll<T>() : 1);
  cudaError_t e = launch_pdl(tensor_amax_kernel<T>, dim3(blocks), dim3(kTensorThreads), 0, st, x, numel, nvec, partial);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "tensor_amax_kernel: %s", cudaGetErrorString(e));
  e = launch_pdl(tensor_quant_kernel<T>, dim3(blocks), dim3(kTensorThreads), 0, st, x, numel, nvec,
                 static_cast<const float*>(partial), blocks, q, scale, azp);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "tensor_quant_kernel: %s", cudaGetErrorString(e));
  return check_launch("tensor_quant_kernel");
}

template <typename T, int VPT>
int launch_rowblock(const T* x, int64_t ngroups, int64_t gvec, float eps, int8_t* q, float* scales, cudaStream_t st) {
  int threads = (int)((gvec + VPT - 1) / VPT);
  threads = ((threads + 31) / 32) * 32;
  if (threads > 1024) return set_error(KVB_E_SHAPE, "group too large for the register-resident path");
  cudaError_t e;
  if (threads <= 128)
    e = launch_pdl(group_quant_rowblock_kernel<T, VPT, 128, 16>, dim3((unsigned)ngroups), dim3(threads), 0, st, x,
                   (int)gvec, eps, q, scales);
  else
    e = launch_pdl(group_quant_rowblock_kernel<T, VPT, 1024, 1>, dim3((unsigned)ngroups), dim3(threads), 0, st, x,
                   (int)gvec, eps, q, scales);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "group_quant_rowblock_kernel: %s", cudaGetErrorString(e));
  return check_launch("group_quant_rowblock_kernel");
}

// Team path (group_quant_teams_kernel) for groups of 64 to 512 * VPT vectors: WG = the warps
// that cover a group with at most VPT vectors a thread (a power of two, at most 16).
template <typename T, int VPT, int WG, int kMinBlocks>
int launch_teams(const T* x, int64_t ngroups, int64_t gvec, float eps, int8_t* q, float* scales, cudaStream_t st) {
  constexpr int kTeams = kTeamThreads / 32 / WG;
  const int64_t grid = (ngroups + kTeams - 1) / kTeams;
  if (grid > 0x7fffffff) return set_error(KVB_E_SHAPE, "per_token_group_quant_int8: too many groups");
  cudaError_t e = launch_pdl(group_quant_teams_kernel<T, VPT, WG, kMinBlocks>, dim3((unsigned)grid),
                             dim3(kTeamThreads), 0, st, x, ngroups, (int)gvec, eps, q, scales);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "group_quant_teams_kernel: %s", cudaGetErrorString(e));
  return check_launch("group_quant_teams_kernel");
}

template <typename T>
int launch_teams_any(const T* x, int64_t ngroups, int64_t gvec, float eps, int8_t* q, float* scales, cudaStream_t st) {
  constexpr int V = sizeof(T) == 4 ? 2 : 4;   // vectors a thread (float vectors are twice as wide)
  if (gvec <= 32 * V) return launch_teams<T, V, 1, 2>(x, ngroups, gvec, eps, q, scales, st);
  if (gvec <= 64 * V) return launch_teams<T, V, 2, 2>(x, ngroups, gvec, eps, q, scales, st);
  if (gvec <= 128 * V) return launch_teams<T, V, 4, 2>(x, ngroups, gvec, eps, q, scales, st);
  if (gvec <= 256 * V) return launch_teams<T, V, 8, 2>(x, ngroups, gvec, eps, q, scales, st);
  return launch_teams<T, V, 16, 2>(x, ngroups, gvec, eps, q, scales, st);
}

// Rolling path (group_quant_rolling_kernel) for 16-bit inputs with 64 to 1024 vectors a group:
// two vectors a thread, WG = gvec / 64 rounded up to a power of two.
template <typename T, int WG>
int launch_rolling(const T* x, int64_t ngroups, int64_t gvec, float eps, int8_t* q, float* scales, cudaStream_t st) {
  constexpr int kTeams = kTeamThreads / 32 / WG;
  // Two CTAs per SM at most, then as few CTAs as give every team the same number of rounds
  // (2048 groups: 256 CTAs of 4 rounds each rather than 296 with a last round 46 % full).
  int64_t grid = std::min<int64_t>((ngroups + kTeams - 1) / kTeams, 2 * (int64_t)sm_count());
  const int64_t rounds = (ngroups + grid * kTeams - 1) / (grid * kTeams);
  grid = (ngroups + kTeams * rounds - 1) / (kTeams * rounds);
  const bool full = gvec == 2 * WG * 32;
  cudaError_t e = full ? launch_pdl(group_quant_rolling_kernel<T, 2, WG, true>, dim3((unsigned)grid),
                                    dim3(kTeamThreads), 0, st, x, ngroups, (int)gvec, eps, q, scales)
                       : launch_pdl(group_quant_rolling_kernel<T, 2, WG, false>, dim3((unsigned)grid),
                                    dim3(kTeamThreads), 0, st, x, ngroups, (int)gvec, eps, q, scales);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "group_quant_rolling_kernel: %s", cudaGetErrorString(e));
  return check_launch("group_quant_rolling_kernel");
}

template <typename T>
int launch_rolling_any(const T* x, int64_t ngroups, int64_t gvec, float eps, int8_t* q, float* scales,
                       cudaStream_t st) {
  if (gvec <= 64) return launch_rolling<T, 1>(x, ngroups, gvec, eps, q, scales, st);
  if (gvec <= 128) return launch_rolling<T, 2>(x, ngroups, gvec, eps, q, scales, st);
  if (gvec <= 256) return launch_rolling<T, 4>(x, ngroups, gvec, eps, q, scales, st);
  if (gvec <= 512) return launch_rolling<T, 8>(x, ngroups, gvec, eps, q, scales, st);
  return launch_rolling<T, 16>(x, ngroups, gvec, eps, q, scales, st);
}

template <typename T>
int launch_group_quant(const void* xv, int64_t tokens, int64_t hidden, int64_t G, float eps, int8_t* q,
                       float* scales, cudaStream_t st) {
  const T* x = static_cast<const T*>(xv);
  const int64_t ngroups = tokens * (hidden / G);
  if (ngroups == 0) return KVB_OK;
  const bool vec = (G % 8 == 0) && aligned16(x) && aligned8(q);
  if (vec) {
    const int64_t lanes = G / 8;
    if (lanes <= 32 && (lanes & (lanes - 1)) == 0) {
      const int64_t nvec = tokens * hidden / 8;
      constexpr int U = sizeof(T) == 4 ? 2 : 4;   // 64 bytes of x a thread in flight
      int blocks = (int)std::min<int64_t>((nvec + 256 * U - 1) / (256 * U), (int64_t)sm_count() * 8);
      group_quant_subwarp_kernel<T, U><<<blocks, 256, 0, st>>>(x, nvec, (int)lanes, eps, q, scales);
      return check_launch("group_quant_subwarp_kernel");
    }
    if (sizeof(T) == 2 && lanes >= 64 && lanes <= 1024)
      return launch_rolling_any<T>(x, ngroups, lanes, eps, q, scales, st);
    if (lanes >= 64 && lanes <= 512 * (sizeof(T) == 4 ? 2 : 4))
      return launch_teams_any<T>(x, ngroups, lanes, eps, q, scales, st);
    if (ngroups <= 0x7fffffff) {
      if (lanes <= 4 * 1024) return launch_rowblock<T, 4>(x, ngroups, lanes, eps, q, scales, st);
      if (lanes <= 8 * 1024) return launch_rowblock<T, 8>(x, ngroups, lanes, eps, q, scales, st);
    }
  }
  const int64_t warps_needed = ngroups;
  int blocks = (int)std::min<int64_t>((warps_needed + 7) / 8, (int64_t)sm_count() * 16);
  group_quant_scalar_kernel<T><<<blocks, 256, 0, st>>>(x, ngroups, G, eps, q, scales);
  return check_launch("group_quant_scalar_kernel");
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" size_t kvb_dynamic_scaled_int8_quant_workspace_size(void) { return kTensorMaxBlocks * sizeof(float); }

extern "C" int kvb_dynamic_scaled_int8_quant(const void* x, int x_dtype, int64_t numel, int8_t* q, float* scale,
                                             int32_t* azp, void* workspace, size_t workspace_bytes, void* stream) {
  if (numel < 0) return set_error(KVB_E_ARG, "dynamic_scaled_int8_quant: numel < 0");
  if (!x || !q || !scale) return set_error(KVB_E_ARG, "dynamic_scaled_int8_quant: null pointer");
  if (!workspace || workspace_bytes < kvb_dynamic_scaled_int8_quant_workspace_size())
    return set_error(KVB_E_WORKSPACE, "dynamic_scaled_int8_quant: workspace of >= %zu bytes required",
                     kvb_dynamic_scaled_int8_quant_workspace_size());
  if (((uintptr_t)workspace & 3u) != 0) return set_error(KVB_E_ALIGN, "dynamic_scaled_int8_quant: workspace not 4-byte aligned");
  float* amax = static_cast<float*>(workspace);
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case KVB_F32: return launch_tensor_quant<float>(x, numel, q, scale, azp, amax, st);
    case KVB_F16: return launch_tensor_quant<__half>(x, numel, q, scale, azp, amax, st);
    case KVB_BF16: return launch_tensor_quant<__nv_bfloat16>(x, numel, q, scale, azp, amax, st);
    default: return set_error(KVB_E_DTYPE, "dynamic_scaled_int8_quant: x dtype %d unsupported", x_dtype);
  }
}

template <typename T>
int launch_static_quant(const void* xv, int64_t numel, const float* scale, const int32_t* azp, int8_t* q,
                        cudaStream_t st) {
  const T* x = static_cast<const T*>(xv);
  const bool vec = aligned16(x) && aligned8(q);
  const int64_t nvec = vec ? numel / 8 : 0;
  const int64_t work = nvec > 0 ? nvec : numel;
  int blocks = (int)std::min<int64_t>((work + 255) / 256, (int64_t)sm_count() * 8);
  if (blocks < 1) blocks = 1;
  static_quant_kernel<T><<<blocks, 256, 0, st>>>(x, numel, nvec, scale, azp, q);
  return check_launch("static_quant_kernel");
}

extern "C" int kvb_static_scaled_int8_quant(const void* x, int x_dtype, int64_t numel, const float* scale,
                                            const int32_t* azp, int8_t* q, void* stream) {
  if (numel < 0) return set_error(KVB_E_ARG, "static_scaled_int8_quant: numel < 0");
  if (numel == 0) return KVB_OK;
  if (!x || !q || !scale) return set_error(KVB_E_ARG, "static_scaled_int8_quant: null pointer");
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case KVB_F32: return launch_static_quant<float>(x, numel, scale, azp, q, st);
    case KVB_F16: return launch_static_quant<__half>(x, numel, scale, azp, q, st);
    case KVB_BF16: return launch_static_quant<__nv_bfloat16>(x, numel, scale, azp, q, st);
    default: return set_error(KVB_E_DTYPE, "static_scaled_int8_quant: x dtype %d unsupported", x_dtype);
  }
}

extern "C" int kvb_per_token_group_quant_int8(const void* x, int x_dtype, int64_t tokens, int64_t hidden,
                                              int64_t group_size, float eps, int8_t* q, float* scales, void* stream) {
  if (tokens < 0 || hidden < 0) return set_error(KVB_E_ARG, "per_token_group_quant_int8: negative size");
  if (group_size <= 0 || (hidden % group_size) != 0)
    return set_error(KVB_E_SHAPE, "per_token_group_quant_int8: hidden (%lld) must be a multiple of group_size (%lld)",
                     (long long)hidden, (long long)group_size);
  if (!(eps > 0.0f)) return set_error(KVB_E_ARG, "per_token_group_quant_int8: eps must be positive");
  if (tokens * hidden == 0) return KVB_OK;
  if (!x || !q || !scales) return set_error(KVB_E_ARG, "per_token_group_quant_int8: null pointer");
  cudaStream_t st = as_stream(stream);
  switch (x_dtype) {
    case KVB_F32: return launch_group_quant<float>(x, tokens, hidden, group_size, eps, q, scales, st);
    case KVB_F16: return launch_group_quant<__half>(x, tokens, hidden, group_size, eps, q, scales, st);
    case KVB_BF16: return launch_group_quant<__nv_bfloat16>(x, tokens, hidden, group_size, eps, q, scales, st);
    default: return set_error(KVB_E_DTYPE, "per_token_group_quant_int8: x dtype %d unsupported", x_dtype);
  }
}
