// Paged GQA decode attention (split-KV) over an e4m3, fp16 or bf16 KV cache, with an
// optional fused write of each sequence's newest token into an e4m3 cache.
//
// Cache layout: [num_blocks, block_size, Hkv, D] -- the memory order the reference's
// paged_attention_v1/v2 read (their reshape(-1, Hkv, D) of a gathered block) and
// paged_kv_cache_update writes.  A 16-token chunk of one sequence is therefore 16 rows of
// Hkv*D elements, contiguous inside a block (16 KB for e4m3, Hkv=8, D=128).
//
// One CTA = one (sequence, partition of `part` tokens).  A producer warp streams 16-token
// chunks of K and V (all heads) into a `kStages`-deep shared-memory ring with 1-D bulk
// copies (cp.async.bulk, mbarrier completion); consumer warps each own one KV head and up
// to 8 query heads of its GQA group:
//   S^T[16 tok x 8 heads] = K[16 x D] . Q^T[D x 8]     (mma.sync m16n8k16, f32 accumulate)
//   online softmax in the log2 domain (scale folded with log2(e) and the e4m3 K scale)
//   O^T[D x 8] += V^T[D x 16 tok] . P^T[16 tok x 8]     (mma.sync m16n8k16)
// e4m3 codes become f16 pairs in registers (cvt.rn.f16x2.e4m3x2).  Because a dot product
// and the sum over tokens do not depend on the order of their terms, the head dimension is
// permuted so every thread reads one contiguous run of a K row (D/4 elements) and of a V
// row (D/8 elements); Q and the output use the same permutations.  Partials (max, sum,
// unnormalised output per partition) go to a float32 workspace and a merge kernel
// combines them (paged_attention_v2.py:163-173); when asked, the v2 partition outputs
// (exp_sums, max_logits, tmp_out = weighted / (exp_sum + 1e-6)) are written as well.
#include <cmath>

#include "kvb_common.cuh"
#include "kvb_async.cuh"

namespace kvb {
namespace {

constexpr int kChunk = 16;
constexpr int kStagesMax = 4;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr unsigned int kStatusBadIndex = 2u;   // a block-table entry outside [0, num_blocks)

template <typename KT> struct CacheTraits;
template <> struct CacheTraits<uint8_t> { static constexpr int kBytes = 1; static constexpr bool kBf16 = false; };
template <> struct CacheTraits<__half> { static constexpr int kBytes = 2; static constexpr bool kBf16 = false; };
template <> struct CacheTraits<__nv_bfloat16> { static constexpr int kBytes = 2; static constexpr bool kBf16 = true; };

// Not volatile: the MMA has outputs, and the compiler may interleave it with the surrounding
// conversions and shared-memory loads.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, bool bf16) {
  if (bf16) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t lo16) {
  uint32_t r;
  const uint16_t v = (uint16_t)lo16;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi, bool bf16) {
  if (bf16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__device__ __forceinline__ float load_f(const T* p, int64_t i) { return Elem<T>::to_f(p[i]); }

// 2^x with the hardware approximation (MUFU.EX2, relative error ~2^-22; ex2(-inf) = +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// NW consecutive 32-bit words from shared memory with the widest aligned accesses.
template <int NW>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t (&w)[NW]) {
  if constexpr (NW % 4 == 0) {
#pragma unroll
    for (int u = 0; u < NW / 4; ++u) {
      const uint4 x = reinterpret_cast<const uint4*>(p)[u];
      w[4 * u] = x.x; w[4 * u + 1] = x.y; w[4 * u + 2] = x.z; w[4 * u + 3] = x.w;
    }
  } else if constexpr (NW == 2) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    w[0] = x.x; w[1] = x.y;
  } else {
    static_assert(NW == 1, "unsupported span");
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

struct DecodeArgs {
  const void* q;            // [B, Hq, D] (q_dtype)
  const void* k_cache;      // [num_blocks, bs, Hkv, D]
  const void* v_cache;
  const float* k_scale;     // [Hkv] (e4m3 caches) or null
  const float* v_scale;
  const void* seq_lens;     // [B] int32 or int64
  const int32_t* block_table;  // [B, bt_stride] or null (block b holds all of sequence b)
  int64_t bt_stride;
  int64_t num_blocks;
  const void* k_new;        // [B, Hkv, D] (new_dtype) or null: fused write of token seq_len-1
  const void* v_new;
  float* m_part;            // [B, Hq, P]   (log2-domain max)
  float* l_part;            // [B, Hq, P]
  float* o_part;            // [B, Hq, P, D] (unnormalised)
  void* exp_sums;           // optional v2 outputs [B, Hq, P] / [B, Hq, P, D] (out dtype)
  void* max_logits;
  void* tmp_out;
  float sm_scale;
  int batch, hq, hkv, group, bs, part, pmax, tiles_per_kv, stages;
  int q_dtype, new_dtype, sl64, v2_dtype;
  int qtok;                 // CTA rows per cached sequence: CTA row b reads sequence b / qtok
  int hc;                   // KV heads per CTA (hkv, or a divisor of it with the heads split over grid.z)
  int fold;                 // query rows per CTA row: CTA row b serves query rows b*fold .. b*fold+fold-1,
                            // each KV head's tile holding group * fold (query row, head) pairs
};

// Length of the cached sequence that query row b attends to.
__device__ __forceinline__ int64_t seq_len_of(const DecodeArgs& a, int b) {
  const int sq = b / a.qtok;
  return a.sl64 ? reinterpret_cast<const int64_t*>(a.seq_lens)[sq] : (int64_t)reinterpret_cast<const int32_t*>(a.seq_lens)[sq];
}

__device__ __forceinline__ float load_any(const void* p, int dt, int64_t i) {
  if (dt == KVB_BF16) return load_f(reinterpret_cast<const __nv_bfloat16*>(p), i);
  if (dt == KVB_F16) return load_f(reinterpret_cast<const __half*>(p), i);
  return reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_any(void* p, int dt, int64_t i, float v) {
  if (dt == KVB_BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dt == KVB_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

// Physical row (block * bs + offset) of token t of the sequence query row b attends to; -1 if
// the table entry is invalid.
__device__ __forceinline__ int64_t token_row(const DecodeArgs& a, int b, int64_t t) {
  const int64_t blk = t / a.bs;
  const int64_t sq = b / a.qtok;
  const int64_t phys = a.block_table ? (int64_t)a.block_table[sq * a.bt_stride + blk] : sq;
  if (phys < 0 || phys >= a.num_blocks) return -1;
  return phys * a.bs + (t - blk * a.bs);
}

template <typename KT, int D, int MAXT>
__global__ void __launch_bounds__(MAXT, MAXT <= 288 ? 2 : 1) paged_decode_kernel(const __grid_constant__ DecodeArgs a) {
  using TR = CacheTraits<KT>;
  constexpr int EB = TR::kBytes;
  constexpr bool BF = TR::kBf16;
  constexpr int KSPAN = D / 4 * EB;     // bytes of a K row one thread reads
  constexpr int VSPAN = D / 8 * EB;     // bytes of a V row one thread reads
  constexpr int KW = KSPAN / 4, VW = VSPAN / 4;   // ... in 32-bit words
  constexpr int SLABS = D / 16;         // mma k-slabs of QK = m-tiles of PV

  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint64_t full[kStagesMax], empty[kStagesMax];

  const int p = blockIdx.x, b = blockIdx.y;
  const int h0 = blockIdx.z * a.hc;                  // first KV head of this CTA
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ncons = a.hc * a.tiles_per_kv;           // consumer warps; warp ncons is the producer
  const int S = a.stages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], ncons);
    }
    fence_mbar_init();
  }
  __syncthreads();
  // Launched as a programmatic dependent: everything above overlaps the previous grid's tail and
  // nothing global is touched before pdl_wait().  The merge grid may be scheduled from then on.
  pdl_wait();
  pdl_trigger();
  const int64_t L = seq_len_of(a, b);
  const int64_t t_begin = (int64_t)p * a.part;
  const int64_t t_end = (L < t_begin + a.part ? L : t_begin + a.part);
  const int D_ = D;

  if (t_begin >= L) {
    // Partition past this sequence's end: v2 outputs hold exp_sum 0, max -inf, tmp_out 0.
    if (a.exp_sums) {   // this CTA's query heads only: [h0 * group, (h0 + hc) * group)
      const int qh0 = h0 * a.group, nqh = a.hc * a.group;
      for (int i = threadIdx.x; i < nqh; i += blockDim.x) {
        const int64_t o = ((int64_t)b * a.hq + qh0 + i) * a.pmax + p;
        store_any(a.exp_sums, a.v2_dtype, o, 0.0f);
        store_any(a.max_logits, a.v2_dtype, o, -INFINITY);
      }
      for (int i = threadIdx.x; i < nqh * D_; i += blockDim.x) {
        const int h = qh0 + i / D_, d = i % D_;
        store_any(a.tmp_out, a.v2_dtype, (((int64_t)b * a.hq + h) * a.pmax + p) * D_ + d, 0.0f);
      }
    }
    return;
  }
  const int nchunks = (int)((t_end - t_begin + kChunk - 1) / kChunk);
  const uint32_t row_bytes = (uint32_t)(a.hkv * D * EB);   // a token row in the cache (all KV heads)
  const uint32_t srow = (uint32_t)(a.hc * D * EB);         // its slice of this CTA's heads, as staged
  const uint32_t head_off = (uint32_t)(h0 * D * EB);
  const uint32_t chunk_bytes = kChunk * srow;
  auto kstage = [&](int s) { return smem + (size_t)s * 2 * chunk_bytes; };
  auto vstage = [&](int s) { return smem + (size_t)s * 2 * chunk_bytes + chunk_bytes; };

  // ------------------------------------------------------------------ producer warp
  if (warp == ncons) {
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t* kc = reinterpret_cast<const uint8_t*>(a.k_cache);
      const uint8_t* vc = reinterpret_cast<const uint8_t*>(a.v_cache);
      int s = 0;
      uint32_t ph = 0;                               // stage i % S and phase (i / S) & 1, without divisions
      for (int i = 0; i < nchunks; ++i, s = (s + 1 == S) ? 0 : s + 1, ph ^= (s == 0) ? 1u : 0u) {
        if (i >= S && !mbar_wait_bounded(&empty[s], ph ^ 1u)) break;
        const int64_t t0 = t_begin + (int64_t)i * kChunk;
        const int64_t t1 = t_end < t0 + kChunk ? t_end : t0 + kChunk;   // rows past the end are not copied
        mbar_arrive_expect_tx(&full[s], 2u * (uint32_t)(t1 - t0) * srow);
        if (srow != row_bytes) {
          // Heads split over CTAs: each token row's slice of this CTA's heads, one copy each; the
          // block is looked up once per run of rows inside it.
          for (int64_t t = t0; t < t1;) {
            const int64_t n = min(t1 - t, (int64_t)a.bs - t % a.bs);
            const int64_t row = token_row(a, b, t);
            if (row < 0) {
              atomicOr(&g_tu_status, kStatusBadIndex);
              asm volatile("mbarrier.complete_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&full[s])),
                           "r"(2 * (uint32_t)n * srow) : "memory");
            } else {
              for (int64_t j = 0; j < n; ++j) {
                const size_t doff = (size_t)(t + j - t0) * srow;
                bulk_g2s(kstage(s) + doff, kc + (row + j) * row_bytes + head_off, srow, &full[s], pol);
                bulk_g2s(vstage(s) + doff, vc + (row + j) * row_bytes + head_off, srow, &full[s], pol);
              }
            }
            t += n;
          }
          continue;
        }
        // All heads: the chunk is copied as runs of rows that stay inside one block (any block size).
        for (int64_t t = t0; t < t1;) {
          const int64_t n = min(t1 - t, (int64_t)a.bs - t % a.bs);
          const int64_t row = token_row(a, b, t);
          const uint32_t nb = (uint32_t)n * row_bytes;
          const size_t doff = (size_t)(t - t0) * row_bytes;
          if (row < 0) {   // invalid block index: record it and complete the transaction without a copy
            atomicOr(&g_tu_status, kStatusBadIndex);
            asm volatile("mbarrier.complete_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&full[s])),
                         "r"(2 * nb) : "memory");
          } else {
            bulk_g2s(kstage(s) + doff, kc + row * row_bytes, nb, &full[s], pol);
            bulk_g2s(vstage(s) + doff, vc + row * row_bytes, nb, &full[s], pol);
          }
          t += n;
        }
      }
      // Wait (bounded) until the consumers are done with every stage before the CTA exits.
      for (int i = max(0, nchunks - S); i < nchunks; ++i) mbar_wait_bounded(&empty[i % S], (uint32_t)(i / S) & 1u);
    }
    return;
  }
  if (warp > ncons) return;

  // ------------------------------------------------------------------ consumer warps
  const int g = lane >> 2, c = lane & 3;
  const int kvl = warp / a.tiles_per_kv, nt = warp % a.tiles_per_kv;   // KV head within this CTA's group
  const int kvh = h0 + kvl;
  const int qn = nt * 8 + g;                         // this lane's query within the tile group (B operand col)
  const bool qvalid = qn < a.group * a.fold;
  const int qtq = qn / a.group;                      // its query row within the CTA row (0 without folding)
  const int qhead = kvh * a.group + (qn - qtq * a.group);
  const int64_t qrow = (int64_t)b * a.fold + qtq;
  // Q as the B operand of QK, permuted: slab j, regs (b0, b1) = dims (D/4)c + 4j + {0,1 | 2,3}.
  uint32_t qf[SLABS][2];
#pragma unroll
  for (int j = 0; j < SLABS; ++j) {
    float q4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      q4[e] = qvalid ? load_any(a.q, a.q_dtype, (qrow * a.hq + qhead) * D + (D / 4) * c + 4 * j + e) : 0.0f;
    qf[j][0] = pack2(q4[0], q4[1], BF);
    qf[j][1] = pack2(q4[2], q4[3], BF);
  }
  const float ksc = a.k_scale ? a.k_scale[kvh] : 1.0f;
  const float vsc = a.v_scale ? a.v_scale[kvh] : 1.0f;
  const float qk_scale = a.sm_scale * kLog2e * ksc;

  float o[SLABS][4];
#pragma unroll
  for (int t = 0; t < SLABS; ++t) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;   // heads 2c, 2c+1 (log2 domain)
  const int64_t new_tok = a.k_new ? L - 1 : -1;

  bool failed = false;
  int s = 0;
  uint32_t ph = 0;                                   // stage i % S and phase (i / S) & 1
  for (int i = 0; i < nchunks; ++i, s = (s + 1 == S) ? 0 : s + 1, ph ^= (s == 0) ? 1u : 0u) {
    if (!mbar_wait_bounded(&full[s], ph)) {
      failed = true;
      break;
    }
    const int64_t t0 = t_begin + (int64_t)i * kChunk;
    uint8_t* ks = kstage(s);
    uint8_t* vs = vstage(s);
    if (new_tok >= t0 && new_tok < t0 + kChunk) {
      // Fused KV write: quantise this head's new K/V, patch the staged row and write the slot.
      if constexpr (EB == 1) {
        const int r = (int)(new_tok - t0);
        const int64_t row = token_row(a, b, new_tok);
        for (int d = lane * 2; d < D; d += 64) {
          const int64_t src = ((int64_t)b * a.hkv + kvh) * D + d;
          const uint16_t kc2 = quant_e4m3x2(load_any(a.k_new, a.new_dtype, src), load_any(a.k_new, a.new_dtype, src + 1),
                                            make_divisor(ksc));
          const uint16_t vc2 = quant_e4m3x2(load_any(a.v_new, a.new_dtype, src), load_any(a.v_new, a.new_dtype, src + 1),
                                            make_divisor(vsc));
          const size_t off = (size_t)r * srow + (size_t)kvl * D + d;
          *reinterpret_cast<uint16_t*>(ks + off) = kc2;
          *reinterpret_cast<uint16_t*>(vs + off) = vc2;
          if (nt == 0 && row >= 0) {
            *reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(const_cast<void*>(a.k_cache)) + row * row_bytes +
                                         (int64_t)kvh * D + d) = kc2;
            *reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(const_cast<void*>(a.v_cache)) + row * row_bytes +
                                         (int64_t)kvh * D + d) = vc2;
          }
        }
        __syncwarp();
      }
    }
    // ---- S^T = K . Q^T for tokens g and g+8
    const int nvalid = (int)(t_end - t0 < kChunk ? t_end - t0 : kChunk);
    uint32_t kw0[KW], kw1[KW];
    {
      const uint8_t* r0 = ks + (size_t)g * srow + (size_t)kvl * D * EB + c * KSPAN;
      const uint8_t* r1 = r0 + 8 * (size_t)srow;
      if constexpr (KW == 8) {
        // Two 16-byte halves per row: lanes of odd g load them in the opposite order, so the
        // eight lanes of a quarter-warp hit eight different bank groups; selects undo the swap.
        const int sw = (g & 1) * 16;
        const uint4 a0 = *reinterpret_cast<const uint4*>(r0 + sw), a1 = *reinterpret_cast<const uint4*>(r0 + 16 - sw);
        const uint4 b0 = *reinterpret_cast<const uint4*>(r1 + sw), b1 = *reinterpret_cast<const uint4*>(r1 + 16 - sw);
        const bool odd = g & 1;
        const uint4 lo0 = odd ? a1 : a0, hi0 = odd ? a0 : a1, lo1 = odd ? b1 : b0, hi1 = odd ? b0 : b1;
        kw0[0] = lo0.x; kw0[1] = lo0.y; kw0[2] = lo0.z; kw0[3] = lo0.w;
        kw0[4] = hi0.x; kw0[5] = hi0.y; kw0[6] = hi0.z; kw0[7] = hi0.w;
        kw1[0] = lo1.x; kw1[1] = lo1.y; kw1[2] = lo1.z; kw1[3] = lo1.w;
        kw1[4] = hi1.x; kw1[5] = hi1.y; kw1[6] = hi1.z; kw1[7] = hi1.w;
      } else {
        load_words<KW>(r0, kw0);
        load_words<KW>(r1, kw1);
      }
    }
    float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < SLABS; ++j) {
      uint32_t af[4];
      if constexpr (EB == 1) {
        af[0] = e4m3x2_to_f16x2(kw0[j] & 0xffffu);
        af[1] = e4m3x2_to_f16x2(kw1[j] & 0xffffu);
        af[2] = e4m3x2_to_f16x2(kw0[j] >> 16);
        af[3] = e4m3x2_to_f16x2(kw1[j] >> 16);
      } else {
        af[0] = kw0[2 * j];
        af[1] = kw1[2 * j];
        af[2] = kw0[2 * j + 1];
        af[3] = kw1[2 * j + 1];
      }
      mma16816(sacc, af, qf[j][0], qf[j][1], BF);
    }
    // ---- online softmax; sacc = {tok g: head 2c, 2c+1; tok g+8: head 2c, 2c+1}
    float sv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int tok = g + (e >= 2 ? 8 : 0);
      sv[e] = tok < nvalid ? sacc[e] * qk_scale : -INFINITY;
    }
    float mx0 = fmaxf(sv[0], sv[2]), mx1 = fmaxf(sv[1], sv[3]);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float mu0 = mn0 == -INFINITY ? 0.0f : mn0, mu1 = mn1 == -INFINITY ? 0.0f : mn1;
    const float al0 = ex2(m0 - mu0), al1 = ex2(m1 - mu1);
    const float p0 = ex2(sv[0] - mu0), p1 = ex2(sv[1] - mu1), p2 = ex2(sv[2] - mu0), p3 = ex2(sv[3] - mu1);
    l0 = l0 * al0 + (p0 + p2);
    l1 = l1 * al1 + (p1 + p3);
    m0 = mn0;
    m1 = mn1;
    if (__any_sync(0xffffffffu, al0 != 1.0f || al1 != 1.0f)) {   // skipped once the running maxima settle
#pragma unroll
      for (int t = 0; t < SLABS; ++t) {
        o[t][0] *= al0;
        o[t][2] *= al0;
        o[t][1] *= al1;
        o[t][3] *= al1;
      }
    }
    // ---- P^T as the B operand: lane (g, c) needs head g, tokens {2c, 2c+1 | 2c+8, 2c+9}
    uint32_t pb0, pb1;
    {
      const uint32_t pe = pack2(p0, p2, BF);     // head 2c:   tokens g, g+8
      const uint32_t po = pack2(p1, p3, BF);     // head 2c+1: tokens g, g+8
      const int srcA = 8 * c + (g >> 1), srcB = srcA + 4;
      const uint32_t aE = __shfl_sync(0xffffffffu, pe, srcA), aO = __shfl_sync(0xffffffffu, po, srcA);
      const uint32_t bE = __shfl_sync(0xffffffffu, pe, srcB), bO = __shfl_sync(0xffffffffu, po, srcB);
      const uint32_t A = (g & 1) ? aO : aE, B = (g & 1) ? bO : bE;
      pb0 = qvalid ? prmt(A, B, 0x5410) : 0u;
      pb1 = qvalid ? prmt(A, B, 0x7632) : 0u;
    }
    // ---- O^T += V^T . P^T; this lane reads V rows 2c, 2c+1, 2c+8, 2c+9 at dims [(D/8)g, +D/8)
    uint32_t vw[4][VW];
    {
      const int toks[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const uint8_t* src = vs + (size_t)toks[rr] * srow + (size_t)kvl * D * EB + g * VSPAN;
        load_words<VW>(src, vw[rr]);
        if (toks[rr] >= nvalid) {      // rows past the sequence end hold stale bytes: zero them
#pragma unroll
          for (int u = 0; u < VW; ++u) vw[rr][u] = 0u;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < SLABS; ++t) {
      uint32_t af[4];
      if constexpr (EB == 1) {
        const uint32_t sel = (t & 1) ? 0x7362u : 0x5140u;
        const uint32_t x01 = prmt(vw[0][t >> 1], vw[1][t >> 1], sel);
        const uint32_t x89 = prmt(vw[2][t >> 1], vw[3][t >> 1], sel);
        af[0] = e4m3x2_to_f16x2(x01 & 0xffffu);
        af[1] = e4m3x2_to_f16x2(x01 >> 16);
        af[2] = e4m3x2_to_f16x2(x89 & 0xffffu);
        af[3] = e4m3x2_to_f16x2(x89 >> 16);
      } else {
        af[0] = prmt(vw[0][t], vw[1][t], 0x5410u);
        af[1] = prmt(vw[0][t], vw[1][t], 0x7632u);
        af[2] = prmt(vw[2][t], vw[3][t], 0x5410u);
        af[3] = prmt(vw[2][t], vw[3][t], 0x7632u);
      }
      mma16816(o[t], af, pb0, pb1, BF);
    }
    // release the stage (shared-memory writes of the fused path are ordered before the next bulk copy)
    if (EB == 1 && new_tok >= t0 && new_tok < t0 + kChunk) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  if (failed) return;

  // ---- reduce the row sums over the 8 lanes that share c, write the partials
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
#pragma unroll
  for (int e = 0; e < 2; ++e) {
    const int hn = nt * 8 + 2 * c + e;
    if (hn >= a.group * a.fold) continue;
    const int tq = hn / a.group;
    const int h = kvh * a.group + (hn - tq * a.group);
    const float m = e ? m1 : m0, l = e ? l1 : l0;
    const int64_t pi = (((int64_t)b * a.fold + tq) * a.hq + h) * a.pmax + p;
    if (g == 0) {
      a.m_part[pi] = m;
      a.l_part[pi] = l;
    }
    float* op = a.o_part + pi * D;
    const float sv_scale = vsc;   // V codes were used unscaled: apply the per-head V scale here
#pragma unroll
    for (int t = 0; t < SLABS; t += 2) {
      const int d = (D / 8) * g + 2 * t;
      float4 v4 = make_float4(o[t][e] * sv_scale, o[t][2 + e] * sv_scale, o[t + 1][e] * sv_scale,
                              o[t + 1][2 + e] * sv_scale);
      *reinterpret_cast<float4*>(op + d) = v4;
    }
    if (a.exp_sums) {
      if (g == 0) {
        store_any(a.exp_sums, a.v2_dtype, pi, l);
        store_any(a.max_logits, a.v2_dtype, pi, m * kLn2);
      }
      const float inv = 1.0f / (l + 1e-6f);
#pragma unroll
      for (int t = 0; t < SLABS; ++t) {
        const int d = (D / 8) * g + 2 * t;
        store_any(a.tmp_out, a.v2_dtype, pi * D + d, o[t][e] * sv_scale * inv);
        store_any(a.tmp_out, a.v2_dtype, pi * D + d + 1, o[t][2 + e] * sv_scale * inv);
      }
    }
  }
}

// float32 caches: exact float32 arithmetic on CUDA cores (the reference's float32 tolerance,
// rtol = atol = 5e-4, is tighter than f16/tf32 tensor-core inputs allow).  One CTA = one
// (query head, sequence, partition); logits live in shared memory; the output loop runs one
// thread per head dimension so V rows are read coalesced.
__global__ void __launch_bounds__(128) paged_decode_f32_kernel(const __grid_constant__ DecodeArgs a, int D) {
  extern __shared__ __align__(16) float fsm[];   // q [D] | logits [part] | rows [part] (int64)
  __shared__ float red[32];
  const int p = blockIdx.x, b = blockIdx.y, h = blockIdx.z;
  const int kvh = h / a.group;
  const int64_t L = seq_len_of(a, b);
  const int64_t t_begin = (int64_t)p * a.part;
  const int64_t pi = ((int64_t)b * a.hq + h) * a.pmax + p;
  if (t_begin >= L) {
    if (a.exp_sums) {
      if (threadIdx.x == 0) {
        store_any(a.exp_sums, a.v2_dtype, pi, 0.0f);
        store_any(a.max_logits, a.v2_dtype, pi, -INFINITY);
      }
      for (int d = threadIdx.x; d < D; d += blockDim.x) store_any(a.tmp_out, a.v2_dtype, pi * D + d, 0.0f);
    }
    return;
  }
  const int64_t t_end = L < t_begin + a.part ? L : t_begin + a.part;
  const int n = (int)(t_end - t_begin);
  float* qs = fsm;
  float* lg = fsm + D;
  int64_t* rows = reinterpret_cast<int64_t*>(fsm + D + a.part);
  for (int d = threadIdx.x; d < D; d += blockDim.x) qs[d] = load_any(a.q, a.q_dtype, ((int64_t)b * a.hq + h) * D + d);
  __syncthreads();
  const float* kc = reinterpret_cast<const float*>(a.k_cache);
  const float* vc = reinterpret_cast<const float*>(a.v_cache);
  const int64_t rowe = (int64_t)a.hkv * D;   // elements per token row
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int64_t row = token_row(a, b, t_begin + i);
    rows[i] = row;
    float acc = 0.0f;
    if (row >= 0) {
      const float4* kr = reinterpret_cast<const float4*>(kc + row * rowe + (int64_t)kvh * D);
      for (int d4 = 0; d4 < D / 4; ++d4) {
        const float4 kv = kr[d4];
        acc = fmaf(kv.x, qs[4 * d4], acc);
        acc = fmaf(kv.y, qs[4 * d4 + 1], acc);
        acc = fmaf(kv.z, qs[4 * d4 + 2], acc);
        acc = fmaf(kv.w, qs[4 * d4 + 3], acc);
      }
    } else {
      atomicOr(&g_tu_status, kStatusBadIndex);
    }
    const float v = acc * a.sm_scale;
    lg[i] = v;
    mx = fmaxf(mx, v);
  }
  // block max of possibly negative logits (block_reduce<true> assumes non-negative values)
  float lmax = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = lmax;
  __syncthreads();
  lmax = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) lmax = fmaxf(lmax, red[w]);
  float ls = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const float e = expf(lg[i] - lmax);
    lg[i] = e;
    ls += e;
  }
  ls = block_reduce<false>(ls, red);
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.0f;
    for (int i = 0; i < n; ++i) {
      const int64_t row = rows[i];
      if (row >= 0) acc = fmaf(lg[i], vc[row * rowe + (int64_t)kvh * D + d], acc);
    }
    a.o_part[pi * D + d] = acc;
    if (a.tmp_out) store_any(a.tmp_out, a.v2_dtype, pi * D + d, acc / (ls + 1e-6f));
  }
  if (threadIdx.x == 0) {
    a.m_part[pi] = lmax * kLog2e;
    a.l_part[pi] = ls;
    if (a.exp_sums) {
      store_any(a.exp_sums, a.v2_dtype, pi, ls);
      store_any(a.max_logits, a.v2_dtype, pi, lmax);
    }
  }
}

// Combines the split-KV partials of one (query row b, query head h) per warp: the lanes take the
// partitions' log2-domain maxima 32 at a time for the global max M, weigh the partition sums
// by 2^(m_p - M) for the total, and accumulate the weighted unnormalised outputs four
// dimensions a lane (float4 loads of the partial rows, which the decode grid has just written
// and which are still in L2), with the weights of each batch of 32 partitions broadcast by
// shuffles (paged_attention_v2.py:163-173; eps = 1e-6 for the v2 normalisation, else 0).  No
// shared memory and no block barrier: a row is one warp's dependent chain.
// With lse, the natural-log sum of exp of the scaled logits of query row b (= sequence b / qtok,
// query token b % qtok) and head h goes to lse[((b / qtok) * hq + h) * qtok + b % qtok].
constexpr int kMergeWarps = 8;
template <int NK>   // float4 columns a lane: head dims up to 128 * NK
__global__ void __launch_bounds__(kMergeWarps * 32) decode_merge_kernel(
    const float* __restrict__ m_part, const float* __restrict__ l_part, const float* __restrict__ o_part,
    const void* seq_lens, int sl64, int rows, int hq, int D, int part, int pmax, float eps, void* out, int out_dtype,
    int qtok, float* __restrict__ lse) {
  // Launched as a programmatic dependent of the decode grid: wait until that grid has
  // completed and its partials are visible (returns at once without a prerequisite grid).
  // (Triggering the next grid after the wait rather than at entry measured faster in
  // back-to-back decode steps.)
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int bh = blockIdx.x * kMergeWarps + (threadIdx.x >> 5);
  if (bh >= rows) return;
  const int b = bh / hq, sq = b / qtok;
  const int64_t L = sl64 ? reinterpret_cast<const int64_t*>(seq_lens)[sq] : (int64_t)reinterpret_cast<const int32_t*>(seq_lens)[sq];
  const int64_t npl = (L + part - 1) / part;
  const int np = (int)(npl < pmax ? npl : pmax);
  const float* mp = m_part + (int64_t)bh * pmax;
  const float* lp = l_part + (int64_t)bh * pmax;
  const float* op = o_part + (int64_t)bh * pmax * D;
  float4 acc[NK];                         // dimensions 4 * lane + 128 * k
#pragma unroll
  for (int k = 0; k < NK; ++k) acc[k] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  // Weighted sum of the partial rows [i0, i1) of the 32-partition chunk at p0; lane i of wl
  // holds the weight of partition p0 + i (0 past np).  Eight rows' loads are in flight before
  // their FMAs.
  auto fma_rows = [&](int k, const float4 (&v)[8], int i0, float wl) {
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float w = __shfl_sync(0xffffffffu, wl, (i0 + u) & 31);
      acc[k].x = fmaf(v[u].x, w, acc[k].x);
      acc[k].y = fmaf(v[u].y, w, acc[k].y);
      acc[k].z = fmaf(v[u].z, w, acc[k].z);
      acc[k].w = fmaf(v[u].w, w, acc[k].w);
    }
  };
  auto load_rows = [&](int k, float4 (&v)[8], int p0, int i0, int i1) {
    const int d = 4 * lane + 128 * k;
#pragma unroll
    for (int u = 0; u < 8; ++u)
      v[u] = (i0 + u < i1 && d < D) ? *reinterpret_cast<const float4*>(op + (int64_t)(p0 + i0 + u) * D + d)
                                    : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  };
  auto accumulate = [&](int p0, int i0, int i1, float wl) {
    for (; i0 < i1; i0 += 8) {
#pragma unroll
      for (int k = 0; k < NK; ++k) {
        float4 v[8];
        load_rows(k, v, p0, i0, i1);
        fma_rows(k, v, i0, wl);
      }
    }
  };
  float M = -INFINITY, Mu, ls = 0.0f;
  if (NK == 1 && np <= 32) {
    // One chunk: the maxima, the sums and the first eight partial rows are requested together
    // (none depends on another), so the row costs one memory round trip, not three.
    const float ml = lane < np ? mp[lane] : -INFINITY;
    const float ll = lane < np ? lp[lane] : 0.0f;
    float4 v0[NK][8];
#pragma unroll
    for (int k = 0; k < NK; ++k) load_rows(k, v0[k], 0, 0, np);
    M = ml;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    Mu = M == -INFINITY ? 0.0f : M;
    const float wl = lane < np ? exp2f(ml - Mu) : 0.0f;
    ls = ll * wl;
#pragma unroll
    for (int k = 0; k < NK; ++k) fma_rows(k, v0[k], 0, wl);
    accumulate(0, 8, np, wl);
  } else {
    for (int p = lane; p < np; p += 32) M = fmaxf(M, mp[p]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    Mu = M == -INFINITY ? 0.0f : M;
    for (int p0 = 0; p0 < np; p0 += 32) {
      const int p = p0 + lane;
      const float wl = p < np ? exp2f(mp[p] - Mu) : 0.0f;
      ls += p < np ? lp[p] * wl : 0.0f;
      accumulate(p0, 0, min(32, np - p0), wl);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
  const float inv = np > 0 ? 1.0f / (ls + eps) : 0.0f;
  if (lse && lane == 0)   // M, in log2 units, plus log2 of the rescaled sum, to natural log
    lse[((int64_t)sq * hq + bh % hq) * qtok + b % qtok] = np > 0 ? (Mu + log2f(ls)) * kLn2 : -INFINITY;
#pragma unroll
  for (int k = 0; k < NK; ++k) {
    const int d = 4 * lane + 128 * k;
    if (d < D) {
      const int64_t o = (int64_t)bh * D + d;
      store_any(out, out_dtype, o, acc[k].x * inv);
      store_any(out, out_dtype, o + 1, acc[k].y * inv);
      store_any(out, out_dtype, o + 2, acc[k].z * inv);
      store_any(out, out_dtype, o + 3, acc[k].w * inv);
    }
  }
}


template <typename KT, int D, int MAXT>
int launch_decode_t(DecodeArgs& a, size_t smem, cudaStream_t st) {
  auto kern = paged_decode_kernel<KT, D, MAXT>;
  static int attr_set_dev = -1;
  static size_t attr_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_set_dev != dev || smem > attr_smem) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "paged_attention: smem attribute: %s", cudaGetErrorString(e));
    attr_set_dev = dev;
    attr_smem = smem;
  }
  const int threads = (a.hc * a.tiles_per_kv + 1) * 32;
  dim3 grid(a.pmax, a.batch / a.fold, a.hkv / a.hc);
  cudaError_t e = launch_pdl(kern, grid, dim3(threads), smem, st, a);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "paged_decode_kernel: %s", cudaGetErrorString(e));
  return check_launch("paged_decode_kernel");
}

// Up to 8 consumer warps (+1 producer) get a 288-thread register budget; more use 544.
template <typename KT, int D>
int launch_decode(DecodeArgs& a, size_t smem, cudaStream_t st) {
  if (a.hc * a.tiles_per_kv <= 8) return launch_decode_t<KT, D, 288>(a, smem, st);
  return launch_decode_t<KT, D, 544>(a, smem, st);
}

template <typename KT>
int launch_decode_d(DecodeArgs& a, int head_dim, size_t smem, cudaStream_t st) {
  if (head_dim == 128) return launch_decode<KT, 128>(a, smem, st);
  if (head_dim == 64) return launch_decode<KT, 64>(a, smem, st);
  return launch_decode<KT, 32>(a, smem, st);
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_paged_attention_auto_partition(int sequences, int64_t max_seq_len) {
  // 512-token partitions, halved down to 64 while the grid has fewer (sequence, partition) CTAs
  // than two for each SM of the current device (148 when there is none)
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
      sms <= 0) {
    cudaGetLastError();
    sms = 148;
  }
  int part = 512;
  while (part > 64 && (int64_t)std::max(sequences, 1) * ((max_seq_len + part - 1) / part) < 2 * (int64_t)sms) part /= 2;
  return part;
}

extern "C" size_t kvb_paged_attention_workspace_size(int batch, int num_q_heads, int head_dim, int max_partitions) {
  const size_t n = (size_t)batch * num_q_heads * max_partitions;
  return (n * (size_t)(head_dim + 2)) * sizeof(float) + 256;
}

static int paged_attention_impl(const void* query, int q_dtype, const void* key_cache, const void* value_cache,
                                   int cache_dtype, const float* k_scale, const float* v_scale, const void* seq_lens,
                                   int seq_lens_dtype, const int32_t* block_table, int64_t bt_stride, int batch,
                                   int num_q_heads, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                   int64_t max_seq_len, float sm_scale, const void* k_new, const void* v_new,
                                   int new_dtype, int partition_size, void* out, int out_dtype, void* exp_sums,
                                   void* max_logits, void* tmp_out, int max_partitions, void* workspace,
                                   size_t workspace_bytes, void* stream, int qtok, float* lse) {
  if (batch < 0 || num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0 || block_size <= 0 || max_seq_len < 0)
    return set_error(KVB_E_ARG, "paged_attention: bad sizes");
  if (batch == 0) return KVB_OK;
  if (!query || !key_cache || !value_cache || !seq_lens || !out || !workspace)
    return set_error(KVB_E_ARG, "paged_attention: null pointer");
  if (num_q_heads % num_kv_heads) return set_error(KVB_E_SHAPE, "paged_attention: num_q_heads %% num_kv_heads != 0");
  if (cache_dtype == KVB_F32 ? (head_dim % 4 != 0 || head_dim > 1024)
                             : (head_dim != 32 && head_dim != 64 && head_dim != 128))
    return set_error(KVB_E_SHAPE, "paged_attention: head_dim %d unsupported (32/64/128; float32 caches: multiples of 4)",
                     head_dim);
  if (!block_table && (int64_t)block_size < max_seq_len)
    return set_error(KVB_E_SHAPE, "paged_attention: without a block table a block must hold a whole sequence");
  if (seq_lens_dtype != KVB_I32 && seq_lens_dtype != KVB_I64) return set_error(KVB_E_DTYPE, "paged_attention: seq_lens dtype");
  if (!is_float_dtype(q_dtype) || !is_float_dtype(out_dtype)) return set_error(KVB_E_DTYPE, "paged_attention: q/out dtype");
  if (cache_dtype == KVB_E4M3 && (!k_scale || !v_scale))
    return set_error(KVB_E_ARG, "paged_attention: e4m3 caches need k_scale and v_scale");
  if ((k_new || v_new) && (!k_new || !v_new || cache_dtype != KVB_E4M3 || !is_float_dtype(new_dtype)))
    return set_error(KVB_E_ARG, "paged_attention: the fused write needs k_new, v_new and an e4m3 cache");
  const int group = num_q_heads / num_kv_heads;
  if (qtok < 1 || batch % qtok) return set_error(KVB_E_ARG, "paged_attention: batch must be a multiple of qtok");
  if ((k_new || v_new) && qtok != 1) return set_error(KVB_E_ARG, "paged_attention: the fused write needs one query per sequence");
  // Query rows of one sequence folded into one CTA row (tensor-core kernels, no v2 outputs): the
  // largest divisor of qtok whose (query row, head) pairs per KV head fill at most 16 tiles of 8,
  // so those rows read the sequence's K/V once between them.
  int fold = 1;
  if (cache_dtype != KVB_F32 && qtok > 1 && !exp_sums)
    for (int f = qtok; f > 1; --f)
      if (qtok % f == 0 && (group * f + 7) / 8 <= 16) { fold = f; break; }
  const int tiles = (group * fold + 7) / 8;
  // KV heads per CTA (tensor-core kernels): all of them when their (kv head, 8-query) tiles fit
  // 16 consumer warps and two 16-token stages of their K/V fit in shared memory; else the
  // largest divisor of num_kv_heads whose tiles fit 8 warps and whose stages fit (heads split
  // over grid.z).
  int hc = num_kv_heads;
  if (cache_dtype != KVB_F32) {
    const size_t head_stage = (size_t)2 * kChunk * head_dim * (cache_dtype == KVB_E4M3 ? 1 : dtype_size(cache_dtype));
    auto fits = [&](int c, int warps) { return c * tiles <= warps && 2 * head_stage * (size_t)c <= 200 * 1024; };
    if (!fits(num_kv_heads, 16)) {
      hc = 0;
      for (int c = num_kv_heads; c >= 1; --c)
        if (num_kv_heads % c == 0 && fits(c, 8)) { hc = c; break; }
      if (hc == 0) {
        if (!fits(1, 16)) return set_error(KVB_E_SHAPE, "paged_attention: more than 128 query heads per KV head");
        hc = 1;
      }
    }
  }
  int part = partition_size;
  if (part <= 0) {
    // automatic: smaller partitions for small grids, unless the workspace was sized for 512
    part = kvb_paged_attention_auto_partition(batch / qtok, max_seq_len);
    const int64_t pm = std::max<int64_t>(1, (max_seq_len + part - 1) / part);
    if (pm > 12288 || kvb_paged_attention_workspace_size(batch, num_q_heads, head_dim, (int)pm) > workspace_bytes)
      part = 512;
  }
  if (part % kChunk) return set_error(KVB_E_SHAPE, "paged_attention: partition_size must be a multiple of 16");
  const int64_t pmax64 = (max_seq_len + part - 1) / part;
  if (pmax64 > 12288)
    return set_error(KVB_E_SHAPE, "paged_attention: %lld partitions (> 12288); use a larger partition_size",
                     (long long)pmax64);
  int pmax = (int)pmax64;
  if (pmax < 1) pmax = 1;
  if (exp_sums || max_logits || tmp_out) {
    if (!exp_sums || !max_logits || !tmp_out) return set_error(KVB_E_ARG, "paged_attention: v2 outputs come together");
    if (max_partitions != pmax)
      return set_error(KVB_E_SHAPE, "paged_attention: max_partitions (%d) != ceil(max_seq_len / partition_size) (%d)",
                       max_partitions, pmax);
  }
  const int esize = cache_dtype == KVB_E4M3 ? 1 : dtype_size(cache_dtype);
  if (esize != 1 && esize != 2 && cache_dtype != KVB_F32)
    return set_error(KVB_E_DTYPE, "paged_attention: cache dtype %d unsupported", cache_dtype);
  const size_t need = kvb_paged_attention_workspace_size(batch, num_q_heads, head_dim, pmax);
  if (workspace_bytes < need) return set_error(KVB_E_WORKSPACE, "paged_attention: workspace %zu < %zu", workspace_bytes, need);
  const int64_t row_bytes = (int64_t)num_kv_heads * head_dim * esize;
  if (row_bytes % 16) return set_error(KVB_E_ALIGN, "paged_attention: a token row must be a multiple of 16 bytes");
  if (!aligned16(key_cache) || !aligned16(value_cache)) return set_error(KVB_E_ALIGN, "paged_attention: caches must be 16-byte aligned");
  const size_t stage_bytes = (size_t)2 * kChunk * (row_bytes / num_kv_heads) * hc;   // this CTA's heads
  int stages = (int)std::min<size_t>(kStagesMax, (200 * 1024) / stage_bytes);
  if (stages > 3 && stage_bytes * 3 >= 96 * 1024) stages = 3;
  if (cache_dtype != KVB_F32 && stages < 2)
    return set_error(KVB_E_SHAPE, "paged_attention: a 16-token chunk (%zu B) does not fit twice in shared memory", stage_bytes);

  DecodeArgs a;
  a.q = query; a.k_cache = key_cache; a.v_cache = value_cache; a.k_scale = k_scale; a.v_scale = v_scale;
  a.seq_lens = seq_lens; a.block_table = block_table; a.bt_stride = bt_stride; a.num_blocks = num_blocks;
  a.k_new = k_new; a.v_new = v_new;
  const size_t n = (size_t)batch * num_q_heads * pmax;
  float* ws = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  a.o_part = ws; a.m_part = ws + n * head_dim; a.l_part = a.m_part + n;   // o_part first: float4-aligned rows
  a.exp_sums = exp_sums; a.max_logits = max_logits; a.tmp_out = tmp_out;
  a.sm_scale = sm_scale;
  a.batch = batch; a.hq = num_q_heads; a.hkv = num_kv_heads; a.group = group; a.bs = block_size; a.part = part;
  a.pmax = pmax; a.tiles_per_kv = tiles; a.stages = stages;
  a.qtok = qtok / fold; a.hc = hc; a.fold = fold;
  a.q_dtype = q_dtype; a.new_dtype = new_dtype; a.sl64 = seq_lens_dtype == KVB_I64; a.v2_dtype = out_dtype;
  const size_t smem = stage_bytes * stages;
  cudaStream_t st = as_stream(stream);
  int rc;
  if (cache_dtype == KVB_E4M3) rc = launch_decode_d<uint8_t>(a, head_dim, smem, st);
  else if (cache_dtype == KVB_F16) rc = launch_decode_d<__half>(a, head_dim, smem, st);
  else if (cache_dtype == KVB_BF16) rc = launch_decode_d<__nv_bfloat16>(a, head_dim, smem, st);
  else {
    const size_t fsmem = (size_t)(head_dim + part) * sizeof(float) + (size_t)part * sizeof(int64_t);
    if (fsmem > 48 * 1024) return set_error(KVB_E_SHAPE, "paged_attention: float32 partitions are limited to 4000 tokens");
    dim3 grid(pmax, batch, num_q_heads);
    paged_decode_f32_kernel<<<grid, 128, fsmem, st>>>(a, head_dim);
    rc = check_launch("paged_decode_f32_kernel");
  }
  if (rc) return rc;
  const float eps = exp_sums ? 1e-6f : 0.0f;
  // Programmatic dependent launch: the merge grid is scheduled while the decode grid drains
  // (every decode CTA allows it as it starts) and waits on the device for its partials, which
  // hides the launch gap between the two kernels.
  cudaLaunchConfig_t cfg = {};
  const int rows = batch * num_q_heads;
  cfg.gridDim = dim3((unsigned)((rows + kMergeWarps - 1) / kMergeWarps));
  cfg.blockDim = dim3(kMergeWarps * 32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float* mp = a.m_part;
  const float* lp = a.l_part;
  const float* op = a.o_part;
  const int sl64 = a.sl64;
  cudaError_t e = cudaLaunchKernelEx(&cfg, head_dim <= 128 ? decode_merge_kernel<1> : decode_merge_kernel<8>, mp, lp, op,
                                     seq_lens, sl64, rows, num_q_heads, head_dim, part, pmax, eps, out, out_dtype, qtok,
                                     lse);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "decode_merge_kernel: %s", cudaGetErrorString(e));
  return check_launch("decode_merge_kernel");
}

extern "C" int kvb_paged_attention(const void* query, int q_dtype, const void* key_cache, const void* value_cache,
                                   int cache_dtype, const float* k_scale, const float* v_scale, const void* seq_lens,
                                   int seq_lens_dtype, const int32_t* block_table, int64_t bt_stride, int batch,
                                   int num_q_heads, int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                   int64_t max_seq_len, float sm_scale, const void* k_new, const void* v_new,
                                   int new_dtype, int partition_size, void* out, int out_dtype, void* exp_sums,
                                   void* max_logits, void* tmp_out, int max_partitions, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  return paged_attention_impl(query, q_dtype, key_cache, value_cache, cache_dtype, k_scale, v_scale, seq_lens,
                              seq_lens_dtype, block_table, bt_stride, batch, num_q_heads, num_kv_heads, head_dim,
                              block_size, num_blocks, max_seq_len, sm_scale, k_new, v_new, new_dtype, partition_size, out,
                              out_dtype, exp_sums, max_logits, tmp_out, max_partitions, workspace, workspace_bytes,
                              stream, 1, nullptr);
}

extern "C" size_t kvb_flash_attn_with_kvcache_workspace_size(int batch, int seq_len_q, int num_heads, int head_dim,
                                                             int64_t seq_len_k) {
  const int part = kvb_paged_attention_auto_partition(batch, seq_len_k);
  const int64_t pmax = seq_len_k > 0 ? (seq_len_k + part - 1) / part : 1;
  return kvb_paged_attention_workspace_size(batch * seq_len_q, num_heads, head_dim, (int)pmax);
}

extern "C" int kvb_flash_attn_with_kvcache(const void* q, const void* k_cache, const void* v_cache, int dtype,
                                          const void* cache_seqlens, int seqlens_dtype, int batch, int seq_len_q,
                                          int64_t seq_len_k, int num_heads, int num_kv_heads, int head_dim,
                                          float softmax_scale, void* out, float* softmax_lse, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  if (batch < 0 || seq_len_q <= 0 || seq_len_k <= 0 || num_heads <= 0 || num_kv_heads <= 0)
    return set_error(KVB_E_ARG, "flash_attn_with_kvcache: bad sizes");
  if (batch == 0) return KVB_OK;
  // Query token i of sequence b is query row b * seq_len_q + i (q is [batch, seq_len_q, heads, D]);
  // all rows of sequence b read block b of the cache, which holds the whole sequence.
  return paged_attention_impl(q, dtype, k_cache, v_cache, dtype, nullptr, nullptr, cache_seqlens, seqlens_dtype,
                              nullptr, 0, batch * seq_len_q, num_heads, num_kv_heads, head_dim, (int)seq_len_k, batch,
                              seq_len_k, softmax_scale, nullptr, nullptr, 0, 0, out, dtype, nullptr, nullptr, nullptr, 0,
                              workspace, workspace_bytes, stream, seq_len_q, softmax_lse);
}

// ---------------------------------------------------------------------------------------------
// Allocation-free variant of kvb_paged_attention.
//
// Its split-KV partials live in this file-scope device array instead of a caller-provided
// workspace.  Every GPU that loads this library's decode module holds the array until the
// process exits, and all calls on a device share it: calls whose work overlaps on the GPU
// (other streams, other host threads) race on it.  Nothing in it needs to start at zero --
// the decode kernel writes every partial the merge kernel reads -- and it keeps whatever
// the last call left there.
#include <mutex>

namespace kvb {
namespace {
static __device__ __align__(256) unsigned char g_noalloc_scratch[KVB_PAGED_ATTENTION_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device
// (the host-side symbol is only a stand-in and must never be passed to a kernel).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "paged_attention_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(KVB_E_DEVICE, "paged_attention_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> g(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(KVB_E_LAUNCH, "paged_attention_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return KVB_OK;
}
}  // namespace
}  // namespace kvb

extern "C" int kvb_paged_attention_noalloc(const void* query, int q_dtype, const void* key_cache,
                                           const void* value_cache, int cache_dtype, const float* k_scale,
                                           const float* v_scale, const void* seq_lens, int seq_lens_dtype,
                                           const int32_t* block_table, int64_t bt_stride, int batch, int num_q_heads,
                                           int num_kv_heads, int head_dim, int block_size, int64_t num_blocks,
                                           int64_t max_seq_len, float sm_scale, const void* k_new, const void* v_new,
                                           int new_dtype, int partition_size, void* out, int out_dtype,
                                           void* exp_sums, void* max_logits, void* tmp_out, int max_partitions,
                                           void* stream) {
  if (batch < 0 || num_q_heads <= 0 || head_dim <= 0 || max_seq_len < 0)
    return set_error(KVB_E_ARG, "paged_attention_noalloc: bad sizes");
  const int part = partition_size > 0 ? partition_size : 512;
  int64_t pmax = (max_seq_len + part - 1) / part;
  if (pmax < 1) pmax = 1;
  const size_t need = kvb_paged_attention_workspace_size(batch, num_q_heads, head_dim, (int)pmax);
  if (need > (size_t)KVB_PAGED_ATTENTION_NOALLOC_SCRATCH_BYTES)
    return set_error(KVB_E_WORKSPACE,
                     "paged_attention_noalloc: this call needs %zu bytes of scratch but the static scratch holds %u "
                     "(batch * num_q_heads * ceil(max_seq_len / partition_size) * (head_dim + 2) * 4 + 256 bytes); "
                     "use a larger partition_size or kvb_paged_attention with a caller workspace",
                     need, (unsigned)KVB_PAGED_ATTENTION_NOALLOC_SCRATCH_BYTES);
  void* ws = nullptr;
  const int rc = noalloc_scratch(&ws);
  if (rc) return rc;
  return kvb_paged_attention(query, q_dtype, key_cache, value_cache, cache_dtype, k_scale, v_scale, seq_lens,
                             seq_lens_dtype, block_table, bt_stride, batch, num_q_heads, num_kv_heads, head_dim,
                             block_size, num_blocks, max_seq_len, sm_scale, k_new, v_new, new_dtype, partition_size, out,
                             out_dtype, exp_sums, max_logits, tmp_out, max_partitions, ws,
                             (size_t)KVB_PAGED_ATTENTION_NOALLOC_SCRATCH_BYTES, stream);
}
