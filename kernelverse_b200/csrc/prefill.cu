// Packed, variable-length causal prefill attention
// (operators/attention/batched_prefill_attention/batched_prefill_attention.py:30-73).
//
// Request b owns query rows [qo[b], qo[b+1]) and keys [kv[b], kv[b+1]); with q_len <= kv_len its
// query row i sits at absolute position kv_len - q_len + i and attends keys 0..that position of
// KV head h / (Hq / Hkv):  out = softmax(scale * q k^T) v, with float32 softmax state.
//
// Flash-attention tiling: one CTA per (64 query rows of one request, one query head); four warps
// of 16 rows.  K/V tiles of BK keys are double-buffered in shared memory by cp.async (rows past
// the request zero-filled); S = Q K^T and O += P V run on mma.sync tensor-core tiles with float32
// accumulation, and the online softmax works in the log2 domain (running max and sum per row,
// the output rescaled when the max grows).  16-bit inputs use m16n8k16 with P rounded to the
// input type for the PV product.  float32 inputs use m16n8k8 TF32 with every operand split into a
// TF32 head and a TF32 remainder and three products per tile (head.head + head.rest + rest.head),
// which keeps the products to about float32 accuracy.  The heads of one query tile are adjacent
// in the grid, so the CTAs of a KV group run together and share each K/V tile through L2; each
// request's query tiles are issued from its last (longest causal span) to its first.
#include "kvb_common.cuh"
#include "kvb_async.cuh"

namespace kvb {
namespace {

constexpr int kPfRows = 64;          // query rows per CTA
constexpr int kPfThreads = 128;      // four warps of 16 rows
constexpr unsigned int kStatusBadIndptr = 4u;   // an indptr range outside the packed tensors

struct PrefillArgs {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* qo;     // [batch + 1]
  const int32_t* kvp;    // [batch + 1]
  void* out;
  int64_t total_q, total_kv;
  int batch, hq, hkv, group, D;
  float scale_log2;      // softmax_scale * log2(e)
};

template <typename T> struct PfTraits;
template <> struct PfTraits<__nv_bfloat16> { static constexpr bool k16 = true; static constexpr bool kBf = true; static constexpr int kBK = 64; };
template <> struct PfTraits<__half> { static constexpr bool k16 = true; static constexpr bool kBf = false; static constexpr int kBK = 64; };
template <> struct PfTraits<float> { static constexpr bool k16 = false; static constexpr int kBK = 32; };

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

template <bool kBf>
__device__ __forceinline__ void mma_k16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (kBf)
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  else
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// x = head + rest with head = x rounded to TF32 and rest (exact in float32) rounded to TF32.
__device__ __forceinline__ void split_tf32(float x, uint32_t& head, uint32_t& rest) {
  uint32_t h, r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x - __uint_as_float(h)));
  head = h;
  rest = r;
}
// 3xTF32 product into d: the two small cross terms first, then the heads.
__device__ __forceinline__ void mma_3xtf32(float (&d)[4], const float (&a)[4], float b0, float b1) {
  uint32_t ah[4], ar[4], bh0, br0, bh1, br1;
#pragma unroll
  for (int i = 0; i < 4; ++i) split_tf32(a[i], ah[i], ar[i]);
  split_tf32(b0, bh0, br0);
  split_tf32(b1, bh1, br1);
  mma_tf32(d, ar, bh0, bh1);
  mma_tf32(d, ah, br0, br1);
  mma_tf32(d, ah, bh0, bh1);
}

__device__ __forceinline__ float ex2f(float x) {   // 2^x (MUFU.EX2; ex2(-inf) = +0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <typename T>
__device__ __forceinline__ uint32_t pack16(float lo, float hi) {
  if constexpr (PfTraits<T>::kBf) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// rows x D elements of T (token stride `stride` elements) into shared rows of kRowB bytes; rows
// at or past `valid` are zero-filled without reading global memory.
template <typename T, int kRowB>
__device__ __forceinline__ void load_rows(uint32_t sdst, const T* src, int rows, int valid, int64_t stride, int chunks) {
  for (int i = threadIdx.x; i < rows * chunks; i += kPfThreads) {
    const int r = i / chunks, c = i - r * chunks;
    const bool ok = r < valid;
    cp_async16(sdst + (uint32_t)(r * kRowB + c * 16), src + (ok ? (int64_t)r * stride : 0) + c * (16 / (int)sizeof(T)), ok);
  }
}

template <typename T, int DP>
__global__ void __launch_bounds__(kPfThreads, 2) prefill_kernel(const __grid_constant__ PrefillArgs a) {
  using TR = PfTraits<T>;
  constexpr int BK = TR::kBK;
  constexpr int ES = (int)sizeof(T);
  constexpr int kRowB = DP * ES + 16;     // padded row: conflict-free ldmatrix / fragment loads
  constexpr int NT = BK / 8;              // key n-tiles of S
  constexpr int ND = DP / 8;              // d n-tiles of O
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* const qs = smem;
  uint8_t* const ks = qs + kPfRows * kRowB;          // [2][BK] rows
  uint8_t* const vs = ks + 2 * BK * kRowB;           // [2][BK] rows
  const int h = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int D = a.D;

  // Padding columns [D, DP) of every shared row are zero for the whole kernel (the copies never
  // write them), so they add nothing to Q K^T.
  if (D < DP) {
    const int pad_words = (DP - D) * ES / 4;
    for (int i = threadIdx.x; i < (kPfRows + 4 * BK) * pad_words; i += kPfThreads) {
      const int r = i / pad_words, c = i - r * pad_words;
      reinterpret_cast<uint32_t*>(smem + r * kRowB + D * ES)[c] = 0u;
    }
  }
  pdl_trigger();
  pdl_wait();            // launched as a programmatic dependent: global data from here on

  // (request, query tile) of this CTA: request b's tiles, last first.
  int b = -1, tile = 0;
  {
    int rem = (int)blockIdx.y;
    for (int r = 0; r < a.batch; ++r) {
      const int ql = a.qo[r + 1] - a.qo[r];
      const int nt = ql > 0 ? (ql + kPfRows - 1) / kPfRows : 0;
      if (rem < nt) {
        b = r;
        tile = nt - 1 - rem;
        break;
      }
      rem -= nt;
    }
  }
  if (b < 0) return;
  const int q0 = a.qo[b], ql = a.qo[b + 1] - q0;
  const int k0 = a.kvp[b], kl = a.kvp[b + 1] - k0;
  if (q0 < 0 || (int64_t)q0 + ql > a.total_q || k0 < 0 || kl < 0 || (int64_t)k0 + kl > a.total_kv) {
    if (threadIdx.x == 0) atomicOr(&g_tu_status, kStatusBadIndptr);
    return;
  }
  const int i0 = tile * kPfRows;
  const int rows = min(kPfRows, ql - i0);
  const int off = kl - ql;                             // position of query row i = off + i
  const int last = min(off + i0 + rows - 1, kl - 1);   // last key any row of the tile attends
  const int ntiles = last >= 0 ? last / BK + 1 : 0;
  const int kvh = h / a.group;
  const int64_t qstride = (int64_t)a.hq * D, kstride = (int64_t)a.hkv * D;
  const T* qg = reinterpret_cast<const T*>(a.q) + ((int64_t)q0 + i0) * qstride + (int64_t)h * D;
  const T* kg = reinterpret_cast<const T*>(a.k) + (int64_t)k0 * kstride + (int64_t)kvh * D;
  const T* vg = reinterpret_cast<const T*>(a.v) + (int64_t)k0 * kstride + (int64_t)kvh * D;
  const int chunks = D * ES / 16;

  const uint32_t qs_a = smem_u32(qs), ks_a = smem_u32(ks), vs_a = smem_u32(vs);
  load_rows<T, kRowB>(qs_a, qg, kPfRows, rows, qstride, chunks);
  cp_async_commit();
  if (ntiles > 0) {
    load_rows<T, kRowB>(ks_a, kg, BK, min(BK, kl), kstride, chunks);
    load_rows<T, kRowB>(vs_a, vg, BK, min(BK, kl), kstride, chunks);
  }
  cp_async_commit();

  const int r0 = warp * 16;                          // this warp's first row in the tile
  const int pos0 = off + i0 + r0 + g, pos1 = pos0 + 8;   // positions of the thread's two rows
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  float o[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  uint32_t qf[TR::k16 ? DP / 16 : 1][4];             // Q fragments (16-bit path), loaded once

  for (int j = 0; j < ntiles; ++j) {
    if (j + 1 < ntiles) {
      const int nb = (j + 1) & 1, kb = (j + 1) * BK;
      load_rows<T, kRowB>(ks_a + nb * BK * kRowB, kg + (int64_t)kb * kstride, BK, min(BK, kl - kb), kstride, chunks);
      load_rows<T, kRowB>(vs_a + nb * BK * kRowB, vg + (int64_t)kb * kstride, BK, min(BK, kl - kb), kstride, chunks);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int buf = j & 1;
    const uint8_t* kb_s = ks + buf * BK * kRowB;
    const uint8_t* vb_s = vs + buf * BK * kRowB;
    const uint32_t kb_a = ks_a + buf * BK * kRowB, vb_a = vs_a + buf * BK * kRowB;

    // ---- S = Q K^T for this warp's 16 rows and BK keys
    float s[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.0f;
    if constexpr (TR::k16) {
      const int mat = lane >> 3, rr = lane & 7;
      if (j == 0) {
#pragma unroll
        for (int kk = 0; kk < DP / 16; ++kk)
          ldsm_x4(qf[kk], qs_a + (uint32_t)((r0 + (mat & 1) * 8 + rr) * kRowB + (kk * 16 + (mat >> 1) * 8) * 2));
      }
#pragma unroll
      for (int kk = 0; kk < DP / 16; ++kk) {
#pragma unroll
        for (int n = 0; n < NT; n += 2) {
          uint32_t bq[4];
          ldsm_x4(bq, kb_a + (uint32_t)((n * 8 + (mat >> 1) * 8 + rr) * kRowB + (kk * 16 + (mat & 1) * 8) * 2));
          mma_k16<TR::kBf>(s[n], qf[kk], bq[0], bq[1]);
          mma_k16<TR::kBf>(s[n + 1], qf[kk], bq[2], bq[3]);
        }
      }
    } else {
      const float* q_r0 = reinterpret_cast<const float*>(qs + (r0 + g) * kRowB) + t;
      const float* q_r1 = reinterpret_cast<const float*>(qs + (r0 + g + 8) * kRowB) + t;
#pragma unroll
      for (int kk = 0; kk < DP / 8; ++kk) {
        const float af[4] = {q_r0[kk * 8], q_r1[kk * 8], q_r0[kk * 8 + 4], q_r1[kk * 8 + 4]};
#pragma unroll
        for (int n = 0; n < NT; ++n) {
          const float* kr = reinterpret_cast<const float*>(kb_s + (n * 8 + g) * kRowB) + kk * 8 + t;
          mma_3xtf32(s[n], af, kr[0], kr[4]);
        }
      }
    }

    // ---- scale, causal mask (only where the tile reaches past this warp's first row), online softmax
    const int kbase = j * BK;
    const bool mask = kbase + BK - 1 > off + i0 + r0;
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = kbase + n * 8 + 2 * t + e;
        float v0 = s[n][e] * a.scale_log2, v1 = s[n][2 + e] * a.scale_log2;
        if (mask) {
          if (key > pos0) v0 = -INFINITY;
          if (key > pos1) v1 = -INFINITY;
        }
        s[n][e] = v0;
        s[n][2 + e] = v1;
        mx0 = fmaxf(mx0, v0);
        mx1 = fmaxf(mx1, v1);
      }
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float al0 = ex2f(m0 - mx0), al1 = ex2f(m1 - mx1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.0f, rs1 = 0.0f;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      s[n][0] = ex2f(s[n][0] - mx0);
      s[n][1] = ex2f(s[n][1] - mx0);
      s[n][2] = ex2f(s[n][2] - mx1);
      s[n][3] = ex2f(s[n][3] - mx1);
      rs0 += s[n][0] + s[n][1];
      rs1 += s[n][2] + s[n][3];
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      o[n][0] *= al0;
      o[n][1] *= al0;
      o[n][2] *= al1;
      o[n][3] *= al1;
    }

    // ---- O += P V
    if constexpr (TR::k16) {
      const int mat = lane >> 3, rr = lane & 7;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint32_t pa[4] = {pack16<T>(s[2 * kk][0], s[2 * kk][1]), pack16<T>(s[2 * kk][2], s[2 * kk][3]),
                                pack16<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]),
                                pack16<T>(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
        for (int n = 0; n < ND; n += 2) {
          uint32_t bv[4];
          ldsm_x4_t(bv, vb_a + (uint32_t)((kk * 16 + (mat & 1) * 8 + rr) * kRowB + (n + (mat >> 1)) * 8 * 2));
          mma_k16<TR::kBf>(o[n], pa, bv[0], bv[1]);
          if (n + 1 < ND) mma_k16<TR::kBf>(o[n + 1], pa, bv[2], bv[3]);
        }
      }
    } else {
      // A column t <-> key 2t and column t + 4 <-> key 2t + 1 of each 8-key step, so the S
      // accumulator layout is the A fragment as it stands; V's rows are taken in the same order.
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const float pa[4] = {s[n][0], s[n][2], s[n][1], s[n][3]};
        const float* v0 = reinterpret_cast<const float*>(vb_s + (n * 8 + 2 * t) * kRowB) + g;
        const float* v1 = reinterpret_cast<const float*>(vb_s + (n * 8 + 2 * t + 1) * kRowB) + g;
#pragma unroll
        for (int nd = 0; nd < ND; ++nd) mma_3xtf32(o[nd], pa, v0[nd * 8], v1[nd * 8]);
      }
    }
    __syncthreads();     // every warp is done with this buffer before the next copy reuses it
  }
  cp_async_wait<0>();    // (no copy is left in flight when there were no key tiles)

  // ---- normalise and store the valid rows and columns
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = 1.0f / l0, inv1 = 1.0f / l1;
  const int row0 = i0 + r0 + g, row1 = row0 + 8;
  T* og = reinterpret_cast<T*>(a.out) + (int64_t)q0 * qstride + (int64_t)h * D;
#pragma unroll
  for (int n = 0; n < ND; ++n) {
    const int col = n * 8 + 2 * t;
    if (col >= D) continue;
    if (row0 < ql) {
      T* p = og + (int64_t)row0 * qstride + col;
      if constexpr (TR::k16) *reinterpret_cast<uint32_t*>(p) = pack16<T>(o[n][0] * inv0, o[n][1] * inv0);
      else *reinterpret_cast<float2*>(p) = make_float2(o[n][0] * inv0, o[n][1] * inv0);
    }
    if (row1 < ql) {
      T* p = og + (int64_t)row1 * qstride + col;
      if constexpr (TR::k16) *reinterpret_cast<uint32_t*>(p) = pack16<T>(o[n][2] * inv1, o[n][3] * inv1);
      else *reinterpret_cast<float2*>(p) = make_float2(o[n][2] * inv1, o[n][3] * inv1);
    }
  }
}

template <typename T, int DP>
int launch_prefill(const PrefillArgs& a, int tiles_ub, cudaStream_t st) {
  constexpr int BK = PfTraits<T>::kBK;
  constexpr size_t smem = (size_t)(kPfRows + 4 * BK) * (DP * sizeof(T) + 16);
  auto kern = prefill_kernel<T, DP>;
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "batched_prefill_attention: smem attribute: %s", cudaGetErrorString(e));
    set_dev = dev;
  }
  cudaError_t e = launch_pdl(kern, dim3((unsigned)a.hq, (unsigned)tiles_ub), dim3(kPfThreads), smem, st, a);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "prefill_kernel: %s", cudaGetErrorString(e));
  return check_launch("prefill_kernel");
}

template <typename T>
int dispatch_prefill(const PrefillArgs& a, int tiles_ub, cudaStream_t st) {
  const int dp = (a.D + 15) / 16 * 16;
  switch (dp) {
    case 16: return launch_prefill<T, 16>(a, tiles_ub, st);
    case 32: return launch_prefill<T, 32>(a, tiles_ub, st);
    case 48: return launch_prefill<T, 48>(a, tiles_ub, st);
    case 64: return launch_prefill<T, 64>(a, tiles_ub, st);
    case 80: return launch_prefill<T, 80>(a, tiles_ub, st);
    case 96: return launch_prefill<T, 96>(a, tiles_ub, st);
    case 112: return launch_prefill<T, 112>(a, tiles_ub, st);
    case 128: return launch_prefill<T, 128>(a, tiles_ub, st);
    default: return set_error(KVB_E_SHAPE, "batched_prefill_attention: head_dim %d > 128", a.D);
  }
}

}  // namespace

int prefill_tcgen05(const void* q, const void* k, const void* v, bool bf16, const int32_t* qo, const int32_t* kvp,
                    int batch, int64_t total_q, int64_t total_kv, int hq, int hkv, int D, float scale_log2, void* out,
                    int kernel, cudaStream_t st);

}  // namespace kvb

using namespace kvb;

extern "C" int kvb_batched_prefill_attention_variant(const void* q, const void* k, const void* v, int dtype,
                                                     const int32_t* qo_indptr, const int32_t* kv_indptr, int batch,
                                                     int64_t total_q, int64_t total_kv, int num_q_heads,
                                                     int num_kv_heads, int head_dim, float softmax_scale, void* out,
                                                     int variant, void* stream);

extern "C" int kvb_batched_prefill_attention(const void* q, const void* k, const void* v, int dtype,
                                             const int32_t* qo_indptr, const int32_t* kv_indptr, int batch,
                                             int64_t total_q, int64_t total_kv, int num_q_heads, int num_kv_heads,
                                             int head_dim, float softmax_scale, void* out, void* stream) {
  return kvb_batched_prefill_attention_variant(q, k, v, dtype, qo_indptr, kv_indptr, batch, total_q, total_kv,
                                               num_q_heads, num_kv_heads, head_dim, softmax_scale, out, 0, stream);
}

extern "C" int kvb_batched_prefill_attention_variant(const void* q, const void* k, const void* v, int dtype,
                                                     const int32_t* qo_indptr, const int32_t* kv_indptr, int batch,
                                                     int64_t total_q, int64_t total_kv, int num_q_heads,
                                                     int num_kv_heads, int head_dim, float softmax_scale, void* out,
                                                     int variant, void* stream) {
  if (variant < 0 || variant > 3) return set_error(KVB_E_ARG, "batched_prefill_attention: variant %d", variant);
  if (batch < 0 || total_q < 0 || total_kv < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
    return set_error(KVB_E_ARG, "batched_prefill_attention: bad sizes");
  if (num_q_heads % num_kv_heads) return set_error(KVB_E_SHAPE, "batched_prefill_attention: num_q_heads must be a multiple of num_kv_heads");
  if (head_dim % 8) return set_error(KVB_E_SHAPE, "batched_prefill_attention: head_dim must be a multiple of 8");
  if (head_dim > 128) return set_error(KVB_E_SHAPE, "batched_prefill_attention: head_dim %d > 128", head_dim);
  if (batch == 0 || total_q == 0) return KVB_OK;
  if (!q || !k || !v || !qo_indptr || !kv_indptr || !out) return set_error(KVB_E_ARG, "batched_prefill_attention: null pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned8(out))
    return set_error(KVB_E_ALIGN, "batched_prefill_attention: q/k/v 16-byte and out 8-byte alignment");
  // Query tiles over all requests: sum ceil(q_len / 64) <= total_q / 64 + batch.
  const int64_t tiles_ub = total_q / kPfRows + batch;
  if (tiles_ub > 65535 || num_q_heads > 65535 || total_q > INT32_MAX || total_kv > INT32_MAX)
    return set_error(KVB_E_SHAPE, "batched_prefill_attention: too many query tiles");
  PrefillArgs a{};
  a.q = q; a.k = k; a.v = v; a.qo = qo_indptr; a.kvp = kv_indptr; a.out = out;
  a.total_q = total_q; a.total_kv = total_kv;
  a.batch = batch; a.hq = num_q_heads; a.hkv = num_kv_heads; a.group = num_q_heads / num_kv_heads; a.D = head_dim;
  a.scale_log2 = softmax_scale * 1.4426950408889634f;
  cudaStream_t st = as_stream(stream);
  // 16-bit inputs with head_dim in {64, 80, 96, 112, 128} run on tcgen05 (its tensor maps take
  // boxes of 64 head elements x 128 tokens, and it stores 16-byte vectors); the rest on the
  // mma.sync kernel.
  const bool tc_ok = (dtype == KVB_BF16 || dtype == KVB_F16) && head_dim % 16 == 0 && head_dim >= 64 &&
                     total_q >= 128 && total_kv >= 128 && aligned16(out) && softmax_scale != 0.0f;
  if (variant >= 2 && !tc_ok) return set_error(KVB_E_SHAPE, "batched_prefill_attention: no tcgen05 kernel for this case");
  if (tc_ok && variant != 1)
    return prefill_tcgen05(q, k, v, dtype == KVB_BF16, qo_indptr, kv_indptr, batch, total_q, total_kv, num_q_heads,
                           num_kv_heads, head_dim, a.scale_log2, out, variant == 0 ? 0 : variant - 1, st);
  switch (dtype) {
    case KVB_BF16: return dispatch_prefill<__nv_bfloat16>(a, (int)tiles_ub, st);
    case KVB_F16: return dispatch_prefill<__half>(a, (int)tiles_ub, st);
    case KVB_F32: return dispatch_prefill<float>(a, (int)tiles_ub, st);
    default: return set_error(KVB_E_DTYPE, "batched_prefill_attention: dtype %d", dtype);
  }
}
