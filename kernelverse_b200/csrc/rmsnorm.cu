// Residual add + RMSNorm, optionally fused with dynamic per-row int8 / e4m3 quantisation.
//
// Main path (rows of up to 24 KB per input): a persistent kernel, 2-3 CTAs per
// SM, each looping over rows.  One thread streams the next rows' x and residual
// into a double-buffered shared-memory ring with 1-D bulk copies
// (cp.async.bulk, completion on an mbarrier, L2 evict-first), so HBM reads of
// row k+1 and k+2 overlap the reductions and stores of row k.  The float32 sum
// s = x + r stays in registers through both block reductions (sum of squares,
// then amax of the normalised row) and every output is written once: the
// kernel moves exactly the algorithmic bytes.  The weight slice a thread needs
// is loaded into registers once per CTA.
//
// Fallbacks: a one-CTA-per-row register kernel for longer rows and a scalar
// kernel for unaligned or odd sizes.
//
// Arithmetic order follows operators/normalization/add_rmsnorm/add_rmsnorm.py:30-35
// in its float32 "correctness" mode: s = x + r; var = sum(s^2) / H;
// rinv = 1 / sqrt(var + eps); y = (s * rinv) * w.  Every quotient is IEEE (no
// fast-math), so only the float32 summation order of sum(s^2) differs from the
// reference.
#include "kvb_common.cuh"
#include "kvb_async.cuh"

namespace kvb {
namespace {

enum Mode { kOutY = 0, kQuantE4m3 = 1, kQuantInt8 = 2 };

template <typename T, int VPT, int MODE>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ res, const T* __restrict__ w,
                                   int64_t nvec, float hidden_f, float eps, T* __restrict__ out,
                                   uint8_t* __restrict__ codes, float* __restrict__ scales) {
  __shared__ float scratch[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * nvec * 8;
  const T* rr = res + row * nvec * 8;
  float s[VPT][8];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t v = threadIdx.x + (int64_t)j * blockDim.x;
    if (v < nvec) {
      Vec8<T> a, b;
      a.load_stream(xr + v * 8);
      b.load_stream(rr + v * 8);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        s[j][k] = a.get(k) + b.get(k);
        ss = fmaf(s[j][k], s[j][k], ss);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 8; ++k) s[j][k] = 0.0f;
    }
  }
  ss = block_reduce<false>(ss, scratch);
  const float rinv = 1.0f / sqrtf(__fdiv_rn(ss, hidden_f) + eps);

  if (MODE == kOutY) {
    T* orow = out + row * nvec * 8;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int64_t v = threadIdx.x + (int64_t)j * blockDim.x;
      if (v < nvec) {
        Vec8<T> wv, o;
        wv.load(w + v * 8);
#pragma unroll
        for (int k = 0; k < 8; ++k) o.set(k, __fmul_rn(__fmul_rn(s[j][k], rinv), wv.get(k)));
        o.store(orow + v * 8);
      }
    }
    return;
  }

  // Fused quantisation: write the updated residual, turn s into y in place, reduce amax.
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t v = threadIdx.x + (int64_t)j * blockDim.x;
    if (v < nvec) {
      Vec8<T> wv;
      wv.load(w + v * 8);
      if (out) {
        Vec8<T> o;
#pragma unroll
        for (int k = 0; k < 8; ++k) o.set(k, s[j][k]);
        o.store(out + row * nvec * 8 + v * 8);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        s[j][k] = __fmul_rn(__fmul_rn(s[j][k], rinv), wv.get(k));
        amax = fmaxf(amax, fabsf(s[j][k]));
      }
    }
  }
  amax = block_reduce<true>(amax, scratch);
  const float qmax = MODE == kQuantE4m3 ? kE4m3Max : kInt8Max;
  const float scale = fmaxf(__fdiv_rn(amax, qmax), kMinScalingFactor);
  const Divisor dv = make_divisor(scale);
  uint2* crow = reinterpret_cast<uint2*>(codes + row * nvec * 8);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int64_t v = threadIdx.x + (int64_t)j * blockDim.x;
    if (v < nvec) {
      uint32_t lo, hi;
      if (MODE == kQuantE4m3) {
        lo = quant_e4m3x2(s[j][0], s[j][1], dv) | ((uint32_t)quant_e4m3x2(s[j][2], s[j][3], dv) << 16);
        hi = quant_e4m3x2(s[j][4], s[j][5], dv) | ((uint32_t)quant_e4m3x2(s[j][6], s[j][7], dv) << 16);
      } else {
        lo = hi = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          lo |= (uint32_t)(uint8_t)quant_int8(s[j][k], dv) << (8 * k);
          hi |= (uint32_t)(uint8_t)quant_int8(s[j][4 + k], dv) << (8 * k);
        }
      }
      __stcs(crow + v, make_uint2(lo, hi));
    }
  }
  if (threadIdx.x == 0) scales[row] = scale;
}

// Any hidden size / alignment: three passes over the row through L1/L2 (correctness path).
template <typename T, int MODE>
__global__ void __launch_bounds__(256) add_rmsnorm_scalar_kernel(const T* __restrict__ x, const T* __restrict__ res,
                                                                 const T* __restrict__ w, int64_t hidden, float eps,
                                                                 T* __restrict__ out, uint8_t* __restrict__ codes,
                                                                 float* __restrict__ scales) {
  __shared__ float scratch[32];
  const int64_t base = (int64_t)blockIdx.x * hidden;
  float ss = 0.0f;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float s = Elem<T>::to_f(x[base + i]) + Elem<T>::to_f(res[base + i]);
    ss = fmaf(s, s, ss);
  }
  ss = block_reduce<false>(ss, scratch);
  const float rinv = 1.0f / sqrtf(__fdiv_rn(ss, (float)hidden) + eps);
  float amax = 0.0f;
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float s = Elem<T>::to_f(x[base + i]) + Elem<T>::to_f(res[base + i]);
    const float y = __fmul_rn(__fmul_rn(s, rinv), Elem<T>::to_f(w[i]));
    if (MODE == kOutY) {
      out[base + i] = Elem<T>::from_f(y);
    } else {
      amax = fmaxf(amax, fabsf(y));
    }
  }
  if (MODE == kOutY) return;
  amax = block_reduce<true>(amax, scratch);
  const float qmax = MODE == kQuantE4m3 ? kE4m3Max : kInt8Max;
  const float scale = fmaxf(__fdiv_rn(amax, qmax), kMinScalingFactor);
  const Divisor dv = make_divisor(scale);
  __syncthreads();   // every thread has re-read x/res before the residual may be overwritten in place
  for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x) {
    const float s = Elem<T>::to_f(x[base + i]) + Elem<T>::to_f(res[base + i]);
    const float y = __fmul_rn(__fmul_rn(s, rinv), Elem<T>::to_f(w[i]));
    if (MODE == kQuantE4m3) {
      codes[base + i] = (uint8_t)(quant_e4m3x2(y, 0.0f, dv) & 0xff);
    } else {
      codes[base + i] = (uint8_t)quant_int8(y, dv);
    }
  }
  if (out) {
    __syncthreads();
    for (int64_t i = threadIdx.x; i < hidden; i += blockDim.x)
      out[base + i] = Elem<T>::from_f(Elem<T>::to_f(x[base + i]) + Elem<T>::to_f(res[base + i]));
  }
  if (threadIdx.x == 0) scales[blockIdx.x] = scale;
}


// ---------------------------------------------------------------------------------------------
// Persistent, bulk-copy-pipelined kernel.  Dynamic shared memory holds kStages stages of
// [x row | residual row]; full[s] completes when both bulk copies of stage s have landed.
constexpr int kStages = 2;
#ifndef KVB_RMSNORM_PREFETCH_ROWS
#define KVB_RMSNORM_PREFETCH_ROWS 2   // rows a CTA prefetches into L2 before its programmatic-dependent wait
#endif

template <typename T>
__device__ __forceinline__ void issue_row(const T* x, const T* res, int64_t row, int nvec, uint8_t* stage,
                                          uint32_t row_bytes, uint64_t* bar, uint64_t pol) {
  mbar_arrive_expect_tx(bar, 2 * row_bytes);
  bulk_g2s(stage, x + row * (int64_t)nvec * 8, row_bytes, bar, pol);
  bulk_g2s(stage + row_bytes, res + row * (int64_t)nvec * 8, row_bytes, bar, pol);
}

// Codes of one thread's VPT vectors of a row (y already in s), packed 8 per 64-bit store.
// Unchecked divisors take the packed-float32 quotients (two lanes per instruction).
template <int VPT, int MODE, bool kChecked>
__device__ __forceinline__ void store_codes(const float (&s)[VPT][8], const Divisor& dv, uint2* crow, int tid,
                                            int stride, int nvec) {
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = tid + j * stride;
    if (v < nvec) {
      uint32_t lo, hi;
      if (MODE == kQuantE4m3 && !kChecked) {
        lo = quant_e4m3x2_fast_x2(f2_pack(s[j][0], s[j][1]), dv) |
             ((uint32_t)quant_e4m3x2_fast_x2(f2_pack(s[j][2], s[j][3]), dv) << 16);
        hi = quant_e4m3x2_fast_x2(f2_pack(s[j][4], s[j][5]), dv) |
             ((uint32_t)quant_e4m3x2_fast_x2(f2_pack(s[j][6], s[j][7]), dv) << 16);
      } else if (MODE == kQuantE4m3) {
        lo = quant_e4m3x2<kChecked>(s[j][0], s[j][1], dv) | ((uint32_t)quant_e4m3x2<kChecked>(s[j][2], s[j][3], dv) << 16);
        hi = quant_e4m3x2<kChecked>(s[j][4], s[j][5], dv) | ((uint32_t)quant_e4m3x2<kChecked>(s[j][6], s[j][7], dv) << 16);
      } else if (!kChecked) {
        lo = quant4_fast_x2(f2_pack(s[j][0], s[j][1]), f2_pack(s[j][2], s[j][3]), dv);
        hi = quant4_fast_x2(f2_pack(s[j][4], s[j][5]), f2_pack(s[j][6], s[j][7]), dv);
      } else {
        lo = hi = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          lo |= (uint32_t)(uint8_t)quant_int8<true>(s[j][e], dv) << (8 * e);
          hi |= (uint32_t)(uint8_t)quant_int8<true>(s[j][4 + e], dv) << (8 * e);
        }
      }
      __stcs(crow + v, make_uint2(lo, hi));
    }
  }
}

template <typename T, int VPT, int MODE>
__global__ void __launch_bounds__(512) add_rmsnorm_pipe_kernel(const T* __restrict__ x, const T* __restrict__ res,
                                                               const T* __restrict__ w, int64_t rows, int nvec,
                                                               float hidden_f, float eps, T* __restrict__ out,
                                                               uint8_t* __restrict__ codes, float* __restrict__ scales) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kStages];
  __shared__ float red_sum[32], red_max[32];   // alternating buffers of the two reductions
  const uint32_t row_bytes = (uint32_t)nvec * 8u * (uint32_t)sizeof(T);
  const int64_t G = gridDim.x;
  const int tid = threadIdx.x;
  const int nthr = blockDim.x;

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  if (tid == 0 && KVB_RMSNORM_PREFETCH_ROWS > 0) {
    // This CTA's first rows start on their way from DRAM into L2 while the previous grid
    // finishes (prefetch_l2_bulk may precede pdl_wait).  [8192, 8192] back to back: 80.4 ->
    // 78.7 us with two rows; four or eight rows measured 79.3-79.9.
    for (int s = 0; s < KVB_RMSNORM_PREFETCH_ROWS; ++s) {
      const int64_t row = blockIdx.x + s * G;
      if (row >= rows) break;
      prefetch_l2_bulk(x + row * nvec * 8, row_bytes);
      prefetch_l2_bulk(res + row * nvec * 8, row_bytes);
    }
  }
  pdl_wait();            // launched as a programmatic dependent (launch_pdl): global data from here on
  const uint64_t pol = policy_evict_first();
  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      const int64_t row = blockIdx.x + s * G;
      if (row < rows) issue_row(x, res, row, nvec, smem + s * 2 * row_bytes, row_bytes, &full[s], pol);
    }
  }
  float wf[VPT][8];   // this thread's weight slice as float32, loaded once per CTA
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = tid + j * nthr;
    Vec8<T> t;
    if (v < nvec) {
      t.load(w + (int64_t)v * 8);
      t.unpack(wf[j]);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) wf[j][e] = 0.0f;
    }
  }

  int k = 0;
  bool failed = false;
  for (int64_t row = blockIdx.x; row < rows; row += G, ++k) {
    const int st = k % kStages;
    const uint32_t par = (uint32_t)(k / kStages) & 1u;
    const bool ok = mbar_wait_bounded(&full[st], par);
    if (__syncthreads_or(!ok)) {
      failed = true;
      break;
    }
    const uint4* sx = reinterpret_cast<const uint4*>(smem + st * 2 * row_bytes);
    const uint4* sr = reinterpret_cast<const uint4*>(smem + st * 2 * row_bytes + row_bytes);
    float s[VPT][8];
    uint64_t ss2 = f2_pack(0.0f, 0.0f);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = tid + j * nthr;
      if (v < nvec) {
        Vec8<T> a, b;
#pragma unroll
        for (int i = 0; i < Vec8<T>::kWords; ++i) {
          a.w[i] = sx[v * Vec8<T>::kWords + i];
          b.w[i] = sr[v * Vec8<T>::kWords + i];
        }
        float fb[8];
        a.unpack(s[j]);
        b.unpack(fb);
        // s = x + r and the sum of squares on packed pairs (two partial sums)
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const uint64_t p = f2_add(f2_pack(s[j][e], s[j][e + 1]), f2_pack(fb[e], fb[e + 1]));
          ss2 = f2_fma(p, p, ss2);
          const float2 u = f2_unpack(p);
          s[j][e] = u.x;
          s[j][e + 1] = u.y;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) s[j][e] = 0.0f;
      }
    }
    const float2 ssp = f2_unpack(ss2);
    const float ss = block_reduce_1bar<false>(ssp.x + ssp.y, red_sum);   // after this every thread has read stage st
    if (tid == 0) {
      const int64_t next = row + kStages * G;
      if (next < rows) issue_row(x, res, next, nvec, smem + st * 2 * row_bytes, row_bytes, &full[st], pol);
    }
    const float rinv = 1.0f / sqrtf(__fdiv_rn(ss, hidden_f) + eps);
    T* orow = out ? out + row * (int64_t)nvec * 8 : nullptr;

    if (MODE == kOutY) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = tid + j * nthr;
        if (v < nvec) {
          float yf[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) yf[e] = __fmul_rn(__fmul_rn(s[j][e], rinv), wf[j][e]);
          Vec8<T> o;
          o.pack(yf);
          o.store(orow + (int64_t)v * 8);
        }
      }
      continue;
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = tid + j * nthr;
      if (v < nvec) {
        if (orow) {
          Vec8<T> o;
          o.pack(s[j]);
          o.store(orow + (int64_t)v * 8);
        }
        const uint64_t r2 = f2_pack(rinv, rinv);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {   // y = (s * rinv) * w on packed pairs
          const float2 y = f2_unpack(f2_mul(f2_mul(f2_pack(s[j][e], s[j][e + 1]), r2), f2_pack(wf[j][e], wf[j][e + 1])));
          s[j][e] = y.x;
          s[j][e + 1] = y.y;
          amax = fmaxf(amax, fmaxf(fabsf(y.x), fabsf(y.y)));
        }
      }
    }
    amax = block_reduce_1bar<true>(amax, red_max);
    const float qmax = MODE == kQuantE4m3 ? kE4m3Max : kInt8Max;
    const float scale = fmaxf(__fdiv_rn(amax, qmax), kMinScalingFactor);
    const Divisor dv = make_divisor(scale);
    uint2* crow = reinterpret_cast<uint2*>(codes + row * (int64_t)nvec * 8);
    // The scale is the row's amax / qmax (or the floor above it), so one check of the
    // divisor's range covers every value of the row (fast_divisor).
    if (fast_divisor(dv))
      store_codes<VPT, MODE, false>(s, dv, crow, tid, nthr, nvec);
    else
      store_codes<VPT, MODE, true>(s, dv, crow, tid, nthr, nvec);
    if (tid == 0) scales[row] = scale;
  }
  if (failed && tid == 0) {
    // Drain: wait (bounded) for the copies this CTA still has in flight before exiting.
    for (int i = 0; i < kStages; ++i) {
      const int kk = k + i;
      if (blockIdx.x + (int64_t)kk * G < rows) mbar_wait_bounded(&full[kk % kStages], (uint32_t)(kk / kStages) & 1u);
    }
  }
}

struct PipeConfig {
  int grid;
  size_t smem;
};

// Grid = (resident CTAs per SM) x (SM count), computed once per instantiation and device.
template <typename T, int VPT, int MODE>
int launch_pipe(const T* x, const T* r, const T* w, int64_t rows, int64_t nvec, float eps, T* out, uint8_t* codes,
                float* scales, cudaStream_t st) {
  const int threads = (int)std::min<int64_t>(512, ((nvec + VPT - 1) / VPT + 31) / 32 * 32);
  const size_t smem = (size_t)kStages * 2 * nvec * 8 * sizeof(T);
  static int cached_dev = -1, cached_blocks = 0, cached_threads = 0;
  static size_t cached_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  auto kern = add_rmsnorm_pipe_kernel<T, VPT, MODE>;
  if (dev != cached_dev || smem != cached_smem || threads != cached_threads) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "add_rmsnorm: smem attribute: %s", cudaGetErrorString(e));
    int nb = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, threads, smem);
    if (e != cudaSuccess || nb < 1) return set_error(KVB_E_LAUNCH, "add_rmsnorm: occupancy query failed");
    cached_dev = dev;
    cached_smem = smem;
    cached_threads = threads;
    cached_blocks = nb;
  }
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t grid = std::min<int64_t>(rows, (int64_t)cached_blocks * sms);
  cudaError_t e = launch_pdl(kern, dim3((unsigned)grid), dim3(threads), smem, st, x, r, w, rows, (int)nvec,
                             (float)(nvec * 8), eps, out, codes, scales);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "add_rmsnorm_pipe_kernel: %s", cudaGetErrorString(e));
  return check_launch("add_rmsnorm_pipe_kernel");
}

template <typename T, int MODE, int VPT>
int launch_vec(const T* x, const T* r, const T* w, int64_t rows, int64_t nvec, float eps, T* out, uint8_t* codes,
               float* scales, cudaStream_t st) {
  int threads = (int)((nvec + VPT - 1) / VPT);
  threads = ((threads + 31) / 32) * 32;
  add_rmsnorm_kernel<T, VPT, MODE><<<(unsigned)rows, threads, 0, st>>>(x, r, w, nvec, (float)(nvec * 8), eps, out,
                                                                         codes, scales);
  return check_launch("add_rmsnorm_kernel");
}

template <typename T, int MODE>
int launch(const void* xv, const void* rv, const void* wv, int64_t rows, int64_t hidden, float eps, void* outv,
           void* codesv, float* scales, cudaStream_t st) {
  const T* x = static_cast<const T*>(xv);
  const T* r = static_cast<const T*>(rv);
  const T* w = static_cast<const T*>(wv);
  T* out = static_cast<T*>(outv);
  uint8_t* codes = static_cast<uint8_t*>(codesv);
  if (rows == 0 || hidden == 0) return KVB_OK;
  if (rows > 0x7fffffffLL) return set_error(KVB_E_SHAPE, "add_rmsnorm: too many rows");
  // The fused form may write the updated residual over `residual` in place: the vector
  // kernel reads its row fully into registers before writing, so aliasing is safe there.
  const bool vec = hidden % 8 == 0 && aligned16(x) && aligned16(r) && aligned16(w) && (!out || aligned16(out)) &&
                   (!codes || aligned8(codes)) && hidden / 8 <= 16 * 256;
  // Persistent pipelined path: rows of 1..24 KB per input, at least 256 vectors of work.
  const int64_t row_bytes = hidden * (int64_t)sizeof(T);
  if (vec && hidden / 8 >= 256 && row_bytes <= 24 * 1024) {
    const int64_t nvec = hidden / 8;
    if (nvec <= 512) return launch_pipe<T, 1, MODE>(x, r, w, rows, nvec, eps, out, codes, scales, st);
    // Up to 1024 vectors: 4 per thread (256 threads) rather than 2 (512): the per-row work every
    // thread repeats (two reductions, the rsqrt, the scale and its reciprocal) is amortised
    // over twice the elements -- 83.9 -> 82.5 us at [8192, 8192].
    if (nvec <= 1024) return launch_pipe<T, 4, MODE>(x, r, w, rows, nvec, eps, out, codes, scales, st);
    return launch_pipe<T, 3, MODE>(x, r, w, rows, nvec, eps, out, codes, scales, st);
  }
  if (vec) {
    const int64_t nvec = hidden / 8;
    if (nvec <= 256) return launch_vec<T, MODE, 1>(x, r, w, rows, nvec, eps, out, codes, scales, st);
    if (nvec <= 512) return launch_vec<T, MODE, 2>(x, r, w, rows, nvec, eps, out, codes, scales, st);
    if (nvec <= 1024) return launch_vec<T, MODE, 4>(x, r, w, rows, nvec, eps, out, codes, scales, st);
    if (nvec <= 2048) return launch_vec<T, MODE, 8>(x, r, w, rows, nvec, eps, out, codes, scales, st);
    return launch_vec<T, MODE, 16>(x, r, w, rows, nvec, eps, out, codes, scales, st);
  }
  add_rmsnorm_scalar_kernel<T, MODE><<<(unsigned)rows, 256, 0, st>>>(x, r, w, hidden, eps, out, codes, scales);
  return check_launch("add_rmsnorm_scalar_kernel");
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_add_rmsnorm(const void* x, const void* residual, const void* weight, int dtype, int64_t rows,
                               int64_t hidden, float eps, void* out, void* stream) {
  if (rows < 0 || hidden < 0) return set_error(KVB_E_ARG, "add_rmsnorm: negative size");
  if (rows * hidden == 0) return KVB_OK;
  if (!x || !residual || !weight || !out) return set_error(KVB_E_ARG, "add_rmsnorm: null pointer");
  if (!(eps > 0.0f)) return set_error(KVB_E_ARG, "add_rmsnorm: eps must be positive");
  cudaStream_t st = as_stream(stream);
  switch (dtype) {
    case KVB_F32: return launch<float, kOutY>(x, residual, weight, rows, hidden, eps, out, nullptr, nullptr, st);
    case KVB_F16: return launch<__half, kOutY>(x, residual, weight, rows, hidden, eps, out, nullptr, nullptr, st);
    case KVB_BF16: return launch<__nv_bfloat16, kOutY>(x, residual, weight, rows, hidden, eps, out, nullptr, nullptr, st);
    default: return set_error(KVB_E_DTYPE, "add_rmsnorm: dtype %d unsupported", dtype);
  }
}

extern "C" int kvb_add_rmsnorm_quant(const void* x, const void* residual, const void* weight, int dtype, int64_t rows,
                                     int64_t hidden, float eps, void* residual_out, void* codes, int code_dtype,
                                     float* scales, void* stream) {
  if (rows < 0 || hidden < 0) return set_error(KVB_E_ARG, "add_rmsnorm_quant: negative size");
  if (rows * hidden == 0) return KVB_OK;
  if (!x || !residual || !weight || !codes || !scales) return set_error(KVB_E_ARG, "add_rmsnorm_quant: null pointer");
  if (!(eps > 0.0f)) return set_error(KVB_E_ARG, "add_rmsnorm_quant: eps must be positive");
  if (residual_out == x) return set_error(KVB_E_ARG, "add_rmsnorm_quant: residual_out may alias residual, not x");
  cudaStream_t st = as_stream(stream);
#define KVB_RMS_CASE(T)                                                                                        \
  if (code_dtype == KVB_E4M3)                                                                                  \
    return launch<T, kQuantE4m3>(x, residual, weight, rows, hidden, eps, residual_out, codes, scales, st);    \
  if (code_dtype == KVB_I8)                                                                                    \
    return launch<T, kQuantInt8>(x, residual, weight, rows, hidden, eps, residual_out, codes, scales, st);    \
  return set_error(KVB_E_DTYPE, "add_rmsnorm_quant: code dtype %d unsupported", code_dtype);
  switch (dtype) {
    case KVB_F32: { KVB_RMS_CASE(float) }
    case KVB_F16: { KVB_RMS_CASE(__half) }
    case KVB_BF16: { KVB_RMS_CASE(__nv_bfloat16) }
    default: return set_error(KVB_E_DTYPE, "add_rmsnorm_quant: dtype %d unsupported", dtype);
  }
#undef KVB_RMS_CASE
}
