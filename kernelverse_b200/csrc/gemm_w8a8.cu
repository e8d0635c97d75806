// W8A8 int8 GEMM on the 5th-generation tensor cores: out = f(A[M,K] . B[N,K]^T).
//
//   acc[m, n]  = sum_k A[m, k] * B[n, k]                      (exact int32, tcgen05.mma kind::i8, TMEM)
//   acc'[m, n] = acc[m, n] - azp[n] * rowsum(A[m, :])         (optional zero-point correction, exact)
//   out[m, n]  = ((float(acc') * sa[m]) * sb[n] + azp_adj[n]) + bias[n]   (each step one float32 rounding)
//
// or the raw int32 accumulator.  This is the reference's int8_scaled_mm_azp
// (operators/gemm/int8_scaled_mm_azp/int8_scaled_mm_azp.py:61-85, with its dequantise-then-float
// matmul replaced by the exact integer form) and the BASELINE third config (azp off, bias on).
//
// Structure: a persistent, warp-specialised kernel; 128 x BN tiles on one SM, or 256 x BN tiles
// on a CTA pair (cluster of 2, tcgen05 cta_group::2: each CTA loads its 128 rows of A and BN/2
// rows of B and the pair leader issues the MMAs for both); with NSUB = 2 a tile is two such
// N = BN sub-tiles sharing the A tile.
//   warp 0: TMA producer -- A [128 x 128 B] and B [rows x 128 B] K-major boxes with 128-byte
//           swizzle into a STAGES-deep shared-memory ring (mbarrier complete_tx);
//   warp 1: allocates 2 x BN TMEM columns (double-buffered accumulator) and one lane issues
//           4 x tcgen05.mma (K = 32 each) per stage, committing the stage back to the producer
//           and each finished tile to the epilogue;
//   warps 2-9: epilogue -- two warps per TMEM lane quarter, each taking every other 128-byte
//           output chunk: tcgen05.ld 32 columns at a time, scale / bias (optionally a gated
//           activation) / convert, store (direct 16-byte stores, or TMA tensor stores to every
//           rank's buffer for the fused all-gather); then release the accumulator buffer.
// Every mbarrier wait is bounded (kvb_async.cuh); on a timeout the roles drain and the CTA
// frees its TMEM before exiting.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "kvb_common.cuh"
#include "kvb_async.cuh"

namespace kvb {
namespace {

constexpr int kBM = 128;
constexpr int kBK = 128;          // bytes of K per stage = one 128-byte swizzle row
// k-blocks of B requested into L2 ahead of the shared-memory ring (single-wave, small-M launches)
#ifndef KVB_GEMM_PREFETCH_1SM
#define KVB_GEMM_PREFETCH_1SM 1
#endif
constexpr int kPreWaitBlocks = 6;   // k-blocks of B prefetched into L2 before the programmatic wait (small M)
#ifndef KVB_GEMM_PREFETCH_2SM
#define KVB_GEMM_PREFETCH_2SM 0
#endif
constexpr int kUmmaK = 32;        // K of one kind::i8 MMA
constexpr int kEpiWarps = 8;      // two epilogue warps per TMEM lane quarter
constexpr int kThreads = 64 + 32 * kEpiWarps;   // producer, MMA issuer, epilogue warps

struct GemmArgs {
  int M, N, K;
  const float* sa;       // [M]
  const float* sb;       // [N]
  const void* bias;      // [N] or null
  int bias_dtype;
  const float* azp;      // [N] or null (integer-valued)
  const int32_t* rowsum; // [M] (when azp)
  const float* azp_adj;  // [N] or null
  void* out;
  int64_t ldo;
  int out_dtype;         // KVB_BF16 / KVB_F16 / KVB_F32 / KVB_I32
  int n_blocks, m_blocks, tiles;
  int m_fastest;         // tile order: M fastest over every M block (A stays in L2)
  // One tile per CTA (or pair) and no dedicated staging buffer: the epilogue stages its output
  // chunks for the TMA stores in the first 32 KB of the stage ring, idle once the tile's last
  // MMAs have completed (M = 256: 50.9 -> 48.7 us; per-row 16-byte stores put 32 rows ~57 KB
  // apart into every warp store).
  int ring_stage;
  // Fused all-gather: every output tile is also stored into these peer buffers (same layout,
  // columns offset by col_off).  nout == 0 for a plain GEMM.
  int nout;
  int64_t col_off;
  void* outs[8];
  int tma_store;         // 1: full 128-byte output chunks go through TMA tensor stores (omaps)
  int ndest;             // number of valid output maps (destinations) for the TMA-store path
  // Gated activation epilogue (act != 0): B's rows are interleaved in blocks of BN/2 = 128, so
  // accumulator columns [0, 128) of a 256-column tile are the first operand and [128, 256) the
  // second of the same 128 output columns; out = silu(first) * second (act 1, SwiGLU) or
  // first * silu(second) (act 2, mul-and-silu), each operand rounded to the output type first.
  int act;
  int n_out;             // output columns: N, or N / 2 with act
};

// Output tensor maps, one per destination buffer (own buffer first), for TMA stores of
// [32 rows x 128 B] chunks with 128-byte swizzle.
struct OutMaps {
  CUtensorMap m[8];
};

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(map), "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}

template <typename V>
__device__ __forceinline__ V* dst_ptr(const GemmArgs& g, int d, int64_t m, int64_t n) {
  return reinterpret_cast<V*>(d < 0 ? g.out : g.outs[d]) + m * g.ldo + g.col_off + n;
}

// ---------------------------------------------------------------- tcgen05 / TMA wrappers
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], "
      "[%4], %5;"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
// L2 prefetch of one tensor-map tile (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, 8-row atoms of 1024 B.
__device__ __forceinline__ uint64_t smem_desc_k128(const void* p) {
  const uint32_t a = smem_u32(p);
  uint64_t d = 0;
  d |= (uint64_t)((a >> 4) & 0x3FFFu);          // start address
  d |= (uint64_t)1u << 16;                       // leading byte offset: 16 B (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;             // stride byte offset: 1024 B between 8-row groups
  d |= (uint64_t)1u << 46;                       // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                       // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor of tcgen05.mma kind::i8: s32 accumulate, signed A and B, K-major both.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

// ---- CTA-pair (cta_group::2) variants
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of `addr` (a local shared::cta address) in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA load into this CTA's shared memory whose completion is counted on the pair leader's barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(bar_cluster), "l"(policy)
      : "memory");
}
// M = 256 MMA over the CTA pair: A rows 0-127 / 128-255 and B rows [0, N/2) / [N/2, N) come from the
// leader's / the peer's shared memory at the same offsets; D lands in both CTAs' TMEM.
__device__ __forceinline__ void mma_i8_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0),
        "r"(0), "r"(0)
      : "memory");
}
// Completion of this thread's prior MMAs arrives on the barrier at the same offset in both CTAs.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
               ::"r"(smem_u32(bar)), "h"((uint16_t)3)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: this thread gets its lane's 32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Tile order.  When A fits in L2 with room to spare (m_fastest): M fastest over every M block,
// so the CTAs running at the same time share a few B column blocks, each B byte comes from DRAM
// once and A is read from L2 (M = 4096, K = 8192: 316 MB read from DRAM against 268 MB of
// operands; 494 MB with the grouped order).  Otherwise N fastest inside groups of 8 N blocks,
// so A streams from DRAM once per group and B's group stays in L2.
__device__ __forceinline__ void tile_coords(const GemmArgs& g, int t, int& mb, int& nb) {
  if (g.m_fastest) {
    mb = t % g.m_blocks;
    nb = t / g.m_blocks;
    return;
  }
  constexpr int kGroup = 8;
  const int per_group = kGroup * g.m_blocks;
  const int grp = t / per_group;
  const int first_n = grp * kGroup;
  const int gn = min(kGroup, g.n_blocks - first_n);
  const int r = t - grp * per_group;
  mb = r / gn;
  nb = first_n + r % gn;
}

__device__ __forceinline__ float load_bias(const void* p, int dt, int n) {
  if (dt == KVB_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[n]);
  if (dt == KVB_F16) return __half2float(reinterpret_cast<const __half*>(p)[n]);
  return reinterpret_cast<const float*>(p)[n];
}

// Per-column epilogue operands of 32 columns: lane j holds column n0 + j (clamped to the last
// column).  One coalesced load per operand per 32 columns; the values reach the other lanes by
// shuffles.  (Per-element loads of the same address by all 32 lanes serialised behind the L2
// latency and made the epilogue as long as the main loop.)
struct ColVals {
  float sb, bias, azp, adj;
};

__device__ __forceinline__ ColVals load_cols(const GemmArgs& g, int n0, int lane) {
  ColVals c{0.0f, 0.0f, 0.0f, 0.0f};
  if (g.out_dtype == KVB_I32) return c;   // int32-accumulator mode has no column operands
  const int n = min(n0 + lane, g.N - 1);
  c.sb = g.sb[n];
  if (g.bias) c.bias = load_bias(g.bias, g.bias_dtype, n);
  if (g.azp) c.azp = g.azp[n];
  if (g.azp_adj) c.adj = g.azp_adj[n];
  return c;
}

// Scale / bias 32 accumulator columns (operands in c) into float32 values.  All 32 lanes must
// be converged.  The optional operands are template flags: a per-column test around the
// shuffles (convergent operations, which the compiler does not hoist) cost a uniform branch
// per column and made one call ~3000 cycles.
template <bool kAzp, bool kAdj, bool kBias>
__device__ __forceinline__ void epi_values_t(const uint32_t (&r)[32], const ColVals& c, float sa, int32_t rs,
                                             float (&f)[32]) {
  constexpr unsigned kAll = 0xffffffffu;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    int32_t acc = (int32_t)r[j];
    if constexpr (kAzp) acc -= (int32_t)__shfl_sync(kAll, c.azp, j) * rs;
    float y = __fmul_rn(__fmul_rn((float)acc, sa), __shfl_sync(kAll, c.sb, j));
    if constexpr (kAdj) y = __fadd_rn(y, __shfl_sync(kAll, c.adj, j));
    if constexpr (kBias) y = __fadd_rn(y, __shfl_sync(kAll, c.bias, j));
    f[j] = y;
  }
}
__device__ __forceinline__ void epi_values(const GemmArgs& g, const uint32_t (&r)[32], const ColVals& c, float sa,
                                           int32_t rs, float (&f)[32]) {
  const int mask = (g.azp ? 4 : 0) | (g.azp_adj ? 2 : 0) | (g.bias ? 1 : 0);
  switch (mask) {
    case 0: epi_values_t<false, false, false>(r, c, sa, rs, f); break;
    case 1: epi_values_t<false, false, true>(r, c, sa, rs, f); break;
    case 2: epi_values_t<false, true, false>(r, c, sa, rs, f); break;
    case 3: epi_values_t<false, true, true>(r, c, sa, rs, f); break;
    case 4: epi_values_t<true, false, false>(r, c, sa, rs, f); break;
    case 5: epi_values_t<true, false, true>(r, c, sa, rs, f); break;
    case 6: epi_values_t<true, true, false>(r, c, sa, rs, f); break;
    default: epi_values_t<true, true, true>(r, c, sa, rs, f); break;
  }
}

// Output words of 32 float32 values: 32 words for float32 outputs, 16 packed pairs for 16-bit
// (one branch on the type, outside the loops).
__device__ __forceinline__ void pack_out(const GemmArgs& g, const float (&f)[32], uint32_t* w) {
  if (g.out_dtype == KVB_F32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = __float_as_uint(f[j]);
  } else if (g.out_dtype == KVB_BF16) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      __half2 h = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    }
  }
}

// Scale / bias / convert 32 accumulator columns (operands in c) into output words.
__device__ __forceinline__ void epilogue32(const GemmArgs& g, const uint32_t (&r)[32], const ColVals& c, float sa,
                                           int32_t rs, uint32_t* w) {
  if (g.out_dtype == KVB_I32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) w[j] = r[j];
    return;
  }
  float f[32];
  epi_values(g, r, c, sa, rs, f);
  pack_out(g, f, w);
}

// The plain scale / bias epilogue with the tile's column operands in shared memory: cop[j] =
// {sb, bias} of column j, read as broadcasts (every lane reads the same address), two columns
// per 16-byte load -- no shuffles, and no global loads once the accumulator is ready.
template <bool kBias>
__device__ __forceinline__ void epi_values_smem_t(const uint32_t (&r)[32], const float2* cop, float sa, float (&f)[32]) {
#pragma unroll
  for (int j = 0; j < 32; j += 2) {
    const float4 c = *reinterpret_cast<const float4*>(cop + j);
    float y0 = __fmul_rn(__fmul_rn((float)(int32_t)r[j], sa), c.x);
    float y1 = __fmul_rn(__fmul_rn((float)(int32_t)r[j + 1], sa), c.z);
    if constexpr (kBias) {
      y0 = __fadd_rn(y0, c.y);
      y1 = __fadd_rn(y1, c.w);
    }
    f[j] = y0;
    f[j + 1] = y1;
  }
}
__device__ __forceinline__ void epilogue32_smem(const GemmArgs& g, const uint32_t (&r)[32], const float2* cop, float sa,
                                                uint32_t* w) {
  float f[32];
  if (g.bias) epi_values_smem_t<true>(r, cop, sa, f);
  else epi_values_smem_t<false>(r, cop, sa, f);
  pack_out(g, f, w);
}

// Named barrier 1 over the epilogue warps only (barrier 0 is __syncthreads).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(kEpiWarps * 32) : "memory"); }

// Dynamic shared memory of one configuration: the stage ring, the TMA-store staging buffers and,
// when they fit in the 227 KB a CTA may have, one column-operand table per accumulator buffer
// ({sb, bias} per column, the tile's columns rounded up to 32), plus 1 KB for the 1024-byte
// alignment of the ring.
template <int BN, int STAGES, bool kTmaStore, bool k2Sm, int NSUB>
struct GemmSmem {
  static constexpr int kBRows = k2Sm ? BN / 2 : BN;
  static constexpr size_t kStage = (size_t)kBM * kBK + (size_t)NSUB * kBRows * kBK;
  static constexpr size_t kStaging = kTmaStore ? (size_t)kEpiWarps * 4096 : 0;
  static constexpr int kNBuf = NSUB == 1 ? 2 : 1;
  static constexpr int kTabCols = (BN * NSUB + 31) / 32 * 32;
  static constexpr size_t kTabBytes = (size_t)kNBuf * kTabCols * 8;
  static constexpr size_t kBase = STAGES * kStage + kStaging;   // offset of the tables
  static constexpr bool kColSmem = kBase + kTabBytes + 2048 <= 232448;   // + alignment + static smem
  static constexpr size_t kDynamic = kBase + (kColSmem ? kTabBytes : 0) + 1024;
};

// The value the unfused GEMM would have stored, back in float32.
__device__ __forceinline__ float round_out(const GemmArgs& g, float x) {
  if (g.out_dtype == KVB_BF16) return __bfloat162float(__float2bfloat16_rn(x));
  if (g.out_dtype == KVB_F16) return __half2float(__float2half_rn(x));
  return x;
}
// silu(x) = x / (1 + e^-x) in float32 from the fast exponential and the correctly rounded
// reciprocal (a few float32 ulps; the result is then rounded to the 16-bit output type).
__device__ __forceinline__ float silu(float x) { return __fmul_rn(x, __frcp_rn(__fadd_rn(1.0f, __expf(-x)))); }

// Scale and bias of one column per lane (gated epilogue, where there are no zero points).
__device__ __forceinline__ float2 load_sb_bias(const GemmArgs& g, int n0, int lane) {
  const int n = min(n0 + lane, g.N - 1);
  return make_float2(g.sb[n], g.bias ? load_bias(g.bias, g.bias_dtype, n) : 0.0f);
}
__device__ __forceinline__ float2 pick4(const float2 (&v)[4], int k) {   // v[k] without local memory
  return k == 0 ? v[0] : k == 1 ? v[1] : k == 2 ? v[2] : v[3];
}
// Gated-epilogue values of 32 columns: scale / bias with the per-lane column operands c.
__device__ __forceinline__ void act_values(const GemmArgs& g, const uint32_t (&r)[32], float2 c, float sa,
                                           float (&f)[32]) {
  constexpr unsigned kAll = 0xffffffffu;
  if (g.bias) {   // one branch outside the loop (the shuffles are convergent)
#pragma unroll
    for (int j = 0; j < 32; ++j)
      f[j] = __fadd_rn(__fmul_rn(__fmul_rn((float)(int32_t)r[j], sa), __shfl_sync(kAll, c.x, j)),
                       __shfl_sync(kAll, c.y, j));
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) f[j] = __fmul_rn(__fmul_rn((float)(int32_t)r[j], sa), __shfl_sync(kAll, c.x, j));
  }
}

// k2Sm: CTA pairs (cluster of 2) compute 256 x BN tiles with cta_group::2 MMAs; each CTA loads
// its 128 rows of A and BN/2 rows of B, so a k-block moves 32 KB per SM instead of 48 KB.
// NSUB = 2: a tile is two N = BN MMA sub-tiles sharing the A tile (2 x BN > 256 columns, so one
// accumulator buffer in the 512 TMEM columns); a k-block then moves (16 + BN / 8) KB per SM for
// twice the MACs.
template <int BN, int STAGES, bool kTmaStore, bool k2Sm, int NSUB = 1>
__global__ void __launch_bounds__(kThreads, 1) w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a,
                                                                 const __grid_constant__ CUtensorMap tmap_b,
                                                                 const __grid_constant__ GemmArgs g,
                                                                 const __grid_constant__ OutMaps om) {
  constexpr int kTileM = k2Sm ? 2 * kBM : kBM;
  constexpr int TN = BN * NSUB;                 // tile columns
  constexpr int kNBuf = NSUB == 1 ? 2 : 1;      // accumulator buffers in TMEM
  constexpr int kBRows = k2Sm ? BN / 2 : BN;    // B rows this CTA loads per sub-tile
  constexpr uint32_t kABytes = kBM * kBK;
  constexpr uint32_t kBBytes = NSUB * kBRows * kBK;
  constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static_assert(!k2Sm || BN % 32 == 0, "cta_group::2 kind::i8 needs N % 32 == 0");
  // kNBuf accumulator buffers of TN columns; the allocation is a power of two >= 32
  constexpr int kAcc = kNBuf * TN;
  static_assert(kAcc <= 512, "TMEM holds 512 columns");
  constexpr uint32_t kTmemCols = kAcc <= 32 ? 32 : kAcc <= 64 ? 64 : kAcc <= 128 ? 128 : kAcc <= 256 ? 256 : 512;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "tcgen05 kind::i8 with M=128 needs N % 16 == 0, N <= 256");
  constexpr uint32_t kIdesc = idesc_i8(kTileM, BN);
  using SL = GemmSmem<BN, STAGES, kTmaStore, k2Sm, NSUB>;
  static_assert(SL::kStage == kStageBytes && SL::kNBuf == kNBuf, "shared-memory layout");

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2], mma_done;
  __shared__ uint32_t tmem_base_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = (g.K + kBK - 1) / kBK;
  const uint32_t crank = k2Sm ? cluster_ctarank() : 0u;   // 0 = pair leader (issues the MMAs)
  const bool leader = crank == 0;
  const int tile0 = k2Sm ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int tstride = k2Sm ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < kNBuf; ++j) {
      mbar_init(&tmem_full[j], 1);
      mbar_init(&tmem_empty[j], k2Sm ? 2 * kEpiWarps : kEpiWarps);   // every epilogue warp of the pair releases it
    }
    mbar_init(&mma_done, 1);
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_a) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tmap_b) : "memory");
  }
  if (warp == 1) {
    if constexpr (k2Sm) tmem_alloc_pair(&tmem_base_s, kTmemCols);
    else tmem_alloc(&tmem_base_s, kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (k2Sm) {
    __syncwarp();
    cluster_sync_all();    // the peer's barriers are initialised before any remote signal
  }
  tc_fence_after();
  const uint32_t tmem_base = tmem_base_s;
  // Launched as a programmatic dependent of the previous kernel in the stream: everything above
  // (barriers, TMEM, descriptor prefetch) overlaps that kernel's tail; nothing global is read or
  // written before it has completed.  Kernels after this one may be scheduled as SMs free up.
  if (warp == 0 && lane == 0 && g.m_blocks <= 2 && tile0 < g.tiles) {
    // B streams from DRAM once: the first k-blocks of this CTA's first tile start on their way
    // into L2 during that tail (an L2 prefetch returns no data to the SM, so it may precede the
    // wait: a line the previous kernel writes later is updated in L2 before any load reads it).
    // M = 256: 53.9 -> 52.0 us.
    int mb, nb;
    tile_coords(g, tile0, mb, nb);
    const int yb = nb * TN + (int)crank * kBRows;
    for (int kq = 0; kq < KB && kq < kPreWaitBlocks; ++kq)
#pragma unroll
      for (int n = 0; n < NSUB; ++n) tma_prefetch_2d(&tmap_b, kq * kBK, yb + n * BN);
  }
  pdl_wait();
  pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      // A tiles are re-read by every N block: keep them in L2; B is streamed once when M is small.
      const uint64_t pol_a = policy_evict_last();
      const uint64_t pol_b = g.m_blocks <= 2 ? policy_evict_first() : policy_evict_normal();
      for (int t = tile0; t < g.tiles && ok; t += tstride) {
        int mb, nb;
        tile_coords(g, t, mb, nb);
        const int ya = mb * kTileM + (int)crank * kBM, yb = nb * TN + (int)crank * kBRows;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          constexpr int kPrefetchAhead = k2Sm ? KVB_GEMM_PREFETCH_2SM : KVB_GEMM_PREFETCH_1SM;
          if (kPrefetchAhead > 0 && g.m_blocks <= 2 && g.tiles <= tstride) {
            // One wave of tiles streaming B from DRAM once: request k-block kb + kPrefetchAhead
            // into L2 now, before its stage is free, so the DRAM stream is not bound by this
            // SM's stage ring alone (M = 16, one CTA per SM: 42.9 -> 36.7 us at distance 1,
            // 38.3 at 2; CTA pairs at M = 256 and launches of more than one wave run slower
            // with it).
            const int kp = kb + kPrefetchAhead;
            for (int kq = kb == 0 ? STAGES : kp; kq <= kp && kq < KB; ++kq)
#pragma unroll
              for (int n = 0; n < NSUB; ++n) tma_prefetch_2d(&tmap_b, kq * kBK, yb + n * BN);
          }
          const int s = it % STAGES;
          const uint32_t use = it / STAGES;
          if (use > 0 && !mbar_wait_bounded(&empty[s], (use - 1) & 1u)) {
            ok = false;
            break;
          }
          uint8_t* sa_ = smem + s * kStageBytes;
          if constexpr (k2Sm) {
            // both CTAs' bytes complete on the leader's full barrier, which expects them all
            const uint32_t bar = mapa_shared(smem_u32(&full[s]), 0);
            if (leader) mbar_arrive_expect_tx(&full[s], 2 * kStageBytes);
            tma_load_2d_pair(sa_, &tmap_a, kb * kBK, ya, bar, pol_a);
#pragma unroll
            for (int n = 0; n < NSUB; ++n)   // sub-tile n: this CTA's kBRows rows of columns [n BN, n BN + BN)
              tma_load_2d_pair(sa_ + kABytes + n * kBRows * kBK, &tmap_b, kb * kBK, yb + n * BN, bar, pol_b);
          } else {
            mbar_arrive_expect_tx(&full[s], kStageBytes);
            tma_load_2d(sa_, &tmap_a, kb * kBK, ya, &full[s], pol_a);
#pragma unroll
            for (int n = 0; n < NSUB; ++n)
              tma_load_2d(sa_ + kABytes + n * kBRows * kBK, &tmap_b, kb * kBK, yb + n * BN, &full[s], pol_b);
          }
        }
      }
      // drain: every stage issued must have been consumed before this CTA exits
      for (uint32_t i = it > STAGES ? it - STAGES : 0; i < it; ++i)
        mbar_wait_bounded(&empty[i % STAGES], (i / STAGES) & 1u);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int t = tile0; t < g.tiles && ok; t += tstride, ++local) {
        const uint32_t ab = kNBuf == 2 ? (local & 1u) : 0u, v = kNBuf == 2 ? (local >> 1) : local;
        if (v > 0 && !mbar_wait_bounded(&tmem_empty[ab], (v - 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + ab * TN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait_bounded(&full[s], (it / STAGES) & 1u)) {
            ok = false;
            break;
          }
          const uint8_t* a_s = smem + s * kStageBytes;
          const uint8_t* b_s = a_s + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            const uint64_t ad = smem_desc_k128(a_s + kk * kUmmaK);
#pragma unroll
            for (int n = 0; n < NSUB; ++n) {   // sub-tile n -> accumulator columns [n BN, n BN + BN)
              const uint64_t bd = smem_desc_k128(b_s + n * kBRows * kBK + kk * kUmmaK);
              if constexpr (k2Sm) mma_i8_pair(d_tmem + n * BN, ad, bd, kIdesc, (kb | kk) != 0);
              else mma_i8(d_tmem + n * BN, ad, bd, kIdesc, (kb | kk) != 0);
            }
          }
          // stage s is free (in both CTAs) once these MMAs have read it
          if constexpr (k2Sm) mma_commit_pair(&empty[s]);
          else mma_commit(&empty[s]);
        }
        if (!ok) break;
        // accumulator ab is final once every MMA above completes
        if constexpr (k2Sm) mma_commit_pair(&tmem_full[ab]);
        else mma_commit(&tmem_full[ab]);
      }
      // every MMA this thread issued has completed before TMEM may be freed
      if constexpr (k2Sm) mma_commit_pair(&mma_done);
      else mma_commit(&mma_done);
      mbar_wait_bounded(&mma_done, 0);
    } else if (k2Sm && lane == 0) {
      mbar_wait_bounded(&mma_done, 0);   // the leader's MMAs also write this CTA's TMEM
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    // Each warp owns 32 TMEM lanes (= 32 output rows: quarter warp % 4) and every other 128-byte
    // column chunk of them (its half), and one 4 KB staging buffer.
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int ew = warp - 2;                // epilogue warp index
    const int half = ew >> 2;               // which alternate chunks
    const int esize = (g.out_dtype == KVB_I32 || g.out_dtype == KVB_F32) ? 4 : 2;
    const int CW = 128 / esize;             // columns per 128-byte chunk
    uint8_t* stage_buf = smem + (kTmaStore ? (size_t)STAGES * kStageBytes : 0) + (size_t)ew * 4096;
    const bool tma_out = (kTmaStore || g.ring_stage) && g.tma_store;
    // Plain scale / bias epilogue: the eight warps load the tile's column operands into a shared
    // table while the accumulator is computed (every warp of the CTA runs the same tiles, so all
    // take part in every epi_bar, also after a timed-out wait).
    const bool smem_cols = SL::kColSmem && !g.act && !g.azp && !g.azp_adj && g.out_dtype != KVB_I32;
    bool failed = false;
    uint32_t local = 0;
    for (int t = tile0; t < g.tiles; t += tstride, ++local) {
      const uint32_t ab = kNBuf == 2 ? (local & 1u) : 0u, v = kNBuf == 2 ? (local >> 1) : local;
      // The row and column operands are loaded before the accumulator is ready.
      int mb, nb;
      tile_coords(g, t, mb, nb);
      float2* const cop = reinterpret_cast<float2*>(smem + SL::kBase) + ab * SL::kTabCols;
      if (smem_cols) {
        // With one table, every warp must be done with the previous tile's; with two, the
        // barrier after the previous fill already ordered this one behind tile t - 2's readers.
        if constexpr (kNBuf == 1) epi_bar();
        for (int c = ew * 32 + lane; c < SL::kTabCols; c += kEpiWarps * 32) {
          const int n = min(nb * TN + c, g.N - 1);
          cop[c] = make_float2(g.sb[n], g.bias ? load_bias(g.bias, g.bias_dtype, n) : 0.0f);
        }
        epi_bar();
      }
      if (failed) continue;
      const int row0 = mb * kTileM + (int)crank * kBM + q * 32;   // first output row of this warp
      const int m = row0 + lane;
      const bool mrow = m < g.M;
      const float sa = (mrow && g.sa) ? g.sa[m] : 0.0f;   // no scales in int32-accumulator mode
      const int32_t rs = (g.azp && mrow) ? g.rowsum[m] : 0;
      const int OC = g.act ? TN / 2 : TN;   // output columns of a tile (gated: NSUB == 1)
      const uint32_t tm = tmem_base + ((uint32_t)(q * 32) << 16) + ab * TN;   // this warp's accumulator
      ColVals cv0{0.0f, 0.0f, 0.0f, 0.0f}, cv1{0.0f, 0.0f, 0.0f, 0.0f};
      float2 af[4], as[4];                  // gated: the 4 x 32 columns of each operand (OC = 128)
      if (g.act) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          af[k] = load_sb_bias(g, nb * TN + 32 * k, lane);
          as[k] = load_sb_bias(g, nb * TN + OC + 32 * k, lane);
        }
      } else if (!smem_cols) {
        cv0 = load_cols(g, nb * TN + half * CW, lane);
        if (esize == 2 && half * CW + 32 < TN) cv1 = load_cols(g, nb * TN + half * CW + 32, lane);
      }
      if (!mbar_wait_bounded(&tmem_full[ab], v & 1u)) {
        failed = true;   // stop working but keep taking part in the table barriers
        continue;
      }
      tc_fence_after();
#pragma unroll 1
      for (int c0 = half * CW; c0 < OC; c0 += 2 * CW) {
        const int o0 = nb * OC + c0;        // first output column of the chunk
        uint32_t w[32];
        if (g.act) {
          // gated: 32 output columns at a time from accumulator columns c and OC + c
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h * 32 >= CW) break;
            const int c = c0 + 32 * h;
            uint32_t r[32];
            float fa[32], fb[32];
            __syncwarp();                   // tcgen05.ld is .sync.aligned: reconverge first
            tmem_ld32(tm + c, r);
            act_values(g, r, pick4(af, c >> 5), sa, fa);
            __syncwarp();
            tmem_ld32(tm + OC + c, r);
            act_values(g, r, pick4(as, c >> 5), sa, fb);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float x = round_out(g, fa[j]), y = round_out(g, fb[j]);
              fa[j] = g.act == 1 ? __fmul_rn(silu(x), y) : __fmul_rn(x, silu(y));
            }
            pack_out(g, fa, w + 16 * h);    // h > 0 only for 16-bit outputs (16 words per 32 columns)
          }
        } else if (smem_cols) {
          uint32_t r[32];
          __syncwarp();                     // tcgen05.ld is .sync.aligned: reconverge first
          tmem_ld32(tm + c0, r);
          epilogue32_smem(g, r, cop + c0, sa, w);
          if (esize == 2 && c0 + 32 < TN) {
            __syncwarp();
            tmem_ld32(tm + c0 + 32, r);
            epilogue32_smem(g, r, cop + c0 + 32, sa, w + 16);
          }
        } else {
          const int n0 = nb * TN + c0;
          const ColVals cur0 = cv0, cur1 = cv1;
          if (c0 + 2 * CW < TN) {           // prefetch this warp's next chunk's column operands
            cv0 = load_cols(g, n0 + 2 * CW, lane);
            if (esize == 2 && c0 + 2 * CW + 32 < TN) cv1 = load_cols(g, n0 + 2 * CW + 32, lane);
          }
          uint32_t r[32];
          __syncwarp();                     // tcgen05.ld is .sync.aligned: reconverge first
          tmem_ld32(tm + c0, r);
          epilogue32(g, r, cur0, sa, rs, w);
          if (esize == 2 && c0 + 32 < TN) {
            __syncwarp();
            tmem_ld32(tm + c0 + 32, r);
            epilogue32(g, r, cur1, sa, rs, w + 16);
          }
        }
        if (o0 >= g.n_out) continue;
        const bool full_chunk = c0 + CW <= OC && o0 + CW <= g.n_out;
        if (tma_out && full_chunk) {
          // Stage the warp's [32 x 128 B] chunk with the 128-byte swizzle, then one TMA store per
          // destination; rows past M are clipped by the tensor map.
          uint8_t* buf = stage_buf;
          if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // buf is free again
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) =
                make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (lane == 0) {
            for (int d = 0; d < g.ndest; ++d)
              tma_store_2d(&om.m[d], buf, (int)(g.col_off + o0), row0);
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
          }
          continue;
        }
        if (!mrow) continue;
        // Direct stores of the valid columns to every destination: 16-byte vectors for a full,
        // aligned chunk, element stores at a ragged edge.
        const int ncols = min(min(CW, OC - c0), g.n_out - o0);
        for (int d = g.nout ? 0 : -1; d < g.nout; ++d) {
          uint8_t* ob = esize == 4 ? reinterpret_cast<uint8_t*>(dst_ptr<uint32_t>(g, d, m, o0))
                                   : reinterpret_cast<uint8_t*>(dst_ptr<uint16_t>(g, d, m, o0));
          if (ncols == CW && (reinterpret_cast<uintptr_t>(ob) & 15) == 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j)
              reinterpret_cast<uint4*>(ob)[j] = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
            continue;
          }
          if (esize == 4) {
            uint32_t* o = dst_ptr<uint32_t>(g, d, m, o0);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < ncols) o[j] = w[j];
          } else {
            uint16_t* o = dst_ptr<uint16_t>(g, d, m, o0);
#pragma unroll
            for (int j = 0; j < 64; ++j)
              if (j < ncols) o[j] = (uint16_t)(w[j >> 1] >> ((j & 1) * 16));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (k2Sm) mbar_arrive_cluster(mapa_shared(smem_u32(&tmem_empty[ab]), 0));   // the leader's barrier
        else mbar_arrive(&tmem_empty[ab]);
      }
    }
    if (tma_out) {
      if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");   // every output write has landed
      __syncwarp();
    }
  }
  if (g.nout > 1 && warp >= 2) __threadfence_system();   // peer stores visible before the kernel completes
  tc_fence_before();
  __syncthreads();
  if constexpr (k2Sm) {
    __syncwarp();
    cluster_sync_all();    // neither CTA leaves while its peer may still signal it
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (k2Sm) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
}

// rowsum[m] = sum_k A[m, k] (int32), for the zero-point correction.
__global__ void __launch_bounds__(256) rowsum_i8_kernel(const int8_t* __restrict__ a, int M, int K, int32_t* __restrict__ out) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int m = blockIdx.x * warps + (threadIdx.x >> 5); m < M; m += gridDim.x * warps) {
    const int8_t* row = a + (int64_t)m * K;
    int s = 0;
    for (int k = lane * 4; k + 3 < K; k += 128) {
      const int w = *reinterpret_cast<const int*>(row + k);
      s = __dp4a(w, 0x01010101, s);
    }
    for (int k = (K & ~3) + lane; k < K; k += 32) s += row[k];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[m] = s;
  }
}

// B [K, N] (N contiguous) -> Bt [N, K] (K contiguous), 32x32 tiles through shared memory.
__global__ void __launch_bounds__(256) transpose_i8_kernel(const int8_t* __restrict__ b, int K, int N, int8_t* __restrict__ bt) {
  __shared__ int8_t tile[32][33];
  const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int k = k0 + i, n = n0 + threadIdx.x;
    if (k < K && n < N) tile[i][threadIdx.x] = b[(int64_t)k * N + n];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int n = n0 + i, k = k0 + threadIdx.x;
    if (k < K && n < N) bt[(int64_t)n * K + k] = tile[threadIdx.x][i];
  }
}

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D int8 K-major map: rows x K, box [box_rows x 128 B], 128-byte swizzle, zero fill out of bounds.
int make_map(CUtensorMap* map, const void* base, int rows, int K, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(KVB_E_LAUNCH, "w8a8_scaled_mm: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KVB_E_LAUNCH, "w8a8_scaled_mm: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return KVB_OK;
}

int num_sms() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Output map over a [rows, cols] row-major buffer with leading dimension ldo (elements):
// box [32 rows x 128 B], 128-byte swizzle (the epilogue's staging layout).
int make_out_map(CUtensorMap* map, void* base, int out_dtype, int64_t rows, int64_t cols, int64_t ldo) {
  auto fn = encode_fn();
  if (!fn) return set_error(KVB_E_LAUNCH, "w8a8_scaled_mm: cuTensorMapEncodeTiled unavailable");
  const int es = (out_dtype == KVB_I32 || out_dtype == KVB_F32) ? 4 : 2;
  const CUtensorMapDataType dt = out_dtype == KVB_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : out_dtype == KVB_F16  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                 : out_dtype == KVB_F32  ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                         : CU_TENSOR_MAP_DATA_TYPE_INT32;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ldo * es)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), 32u};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KVB_E_LAUNCH, "w8a8_scaled_mm: output tensor map failed (%d)", (int)r);
  return KVB_OK;
}

// TMA stores need 16-byte aligned bases, row pitches and column offsets.
bool tma_store_ok(const GemmArgs& g, void* const* dests, int ndest, int64_t map_cols) {
  const int es = (g.out_dtype == KVB_I32 || g.out_dtype == KVB_F32) ? 4 : 2;
  if ((g.ldo * es) % 16 || (g.col_off * es) % 16 || ndest > 8 || map_cols > g.ldo) return false;
  for (int d = 0; d < ndest; ++d)
    if (!aligned16(dests[d])) return false;
  return true;
}

template <int BN, int STAGES, bool kTmaStore, bool k2Sm, int NSUB = 1>
int launch_gemm(const int8_t* a, const int8_t* b_nk, GemmArgs& g, void* const* dests, int ndest, int64_t map_cols,
                cudaStream_t st) {
  constexpr int kTileM = k2Sm ? 2 * kBM : kBM;
  constexpr int kBRows = k2Sm ? BN / 2 : BN;
  CUtensorMap ma, mb;
  int rc = make_map(&ma, a, g.M, g.K, kBM);
  if (rc) return rc;
  rc = make_map(&mb, b_nk, g.N, g.K, kBRows);
  if (rc) return rc;
  g.m_blocks = (g.M + kTileM - 1) / kTileM;
  g.n_blocks = (g.N + BN * NSUB - 1) / (BN * NSUB);
  g.m_fastest = (int64_t)g.m_blocks * kTileM * g.K <= (int64_t)48 << 20;   // A <= 48 MB of the 126 MB L2
  g.tiles = g.m_blocks * g.n_blocks;
  OutMaps om;
  memset(&om, 0, sizeof(om));
  // Without a staging buffer, a launch of one wave stages output chunks in its idle stage ring.
  static_assert(kTmaStore || STAGES * GemmSmem<BN, STAGES, kTmaStore, k2Sm, NSUB>::kStage >= (size_t)kEpiWarps * 4096,
                "the stage ring holds the epilogue's staging buffers");
  g.ring_stage = !kTmaStore && g.tiles <= (k2Sm ? num_sms() / 2 : num_sms()) ? 1 : 0;
  g.tma_store = (kTmaStore || g.ring_stage) && tma_store_ok(g, dests, ndest, map_cols) ? 1 : 0;
  g.ndest = g.tma_store ? ndest : 0;
  for (int d = 0; d < g.ndest; ++d) {
    rc = make_out_map(&om.m[d], dests[d], g.out_dtype, g.M, map_cols, g.ldo);
    if (rc) return rc;
  }
  const size_t smem = GemmSmem<BN, STAGES, kTmaStore, k2Sm, NSUB>::kDynamic;
  auto kern = w8a8_gemm_kernel<BN, STAGES, kTmaStore, k2Sm, NSUB>;
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "w8a8_scaled_mm: smem attribute: %s", cudaGetErrorString(e));
    set_dev = dev;
  }
  if constexpr (k2Sm) {
    // CTA pairs: a cluster of 2 along x, one pair per two SMs
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see griddepcontrol in the kernel
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(2u * (unsigned)std::min(g.tiles, num_sms() / 2));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, g, om);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "w8a8_gemm_kernel (pairs): %s", cudaGetErrorString(e));
    return check_launch("w8a8_gemm_kernel");
  } else {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see griddepcontrol in the kernel
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)std::min(g.tiles, num_sms()));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, ma, mb, g, om);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "w8a8_gemm_kernel: %s", cudaGetErrorString(e));
    return check_launch("w8a8_gemm_kernel");
  }
}

bool is_sm100() {
  static int cached = -1;
  if (cached < 0) {
    int dev = 0, major = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cached = major == 10;
  }
  return cached == 1;
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_w8a8_scaled_mm_allgather(const int8_t* a, const int8_t* b_shard, const float* a_scales,
                                            const float* b_scales_shard, const void* bias_shard, int bias_dtype,
                                            int64_t M, int64_t N_shard, int64_t K, void* const* out_ptrs, int world,
                                            int rank, int64_t ldo, int out_dtype, void* stream) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world) return set_error(KVB_E_ARG, "w8a8_allgather: world 1..8, 0 <= rank < world");
  if (!out_ptrs) return set_error(KVB_E_ARG, "w8a8_allgather: null out_ptrs");
  for (int r = 0; r < world; ++r)
    if (!out_ptrs[r]) return set_error(KVB_E_ARG, "w8a8_allgather: null output pointer of rank %d", r);
  if (M < 0 || N_shard < 0 || K <= 0) return set_error(KVB_E_ARG, "w8a8_allgather: bad sizes");
  if (M > 0x7fffffff || N_shard > 0x7fffffff || K > 0x7fffffff)
    return set_error(KVB_E_SHAPE, "w8a8_allgather: size too large");
  if (bias_shard && bias_dtype != KVB_BF16 && bias_dtype != KVB_F16 && bias_dtype != KVB_F32)
    return set_error(KVB_E_DTYPE, "w8a8_allgather: bias dtype %d", bias_dtype);
  if (M == 0 || N_shard == 0) return KVB_OK;
  if (ldo < (int64_t)world * N_shard) return set_error(KVB_E_SHAPE, "w8a8_allgather: ldo < world * N_shard");
  if (!a || !b_shard || (out_dtype != KVB_I32 && (!a_scales || !b_scales_shard)))
    return set_error(KVB_E_ARG, "w8a8_allgather: null pointer");
  if (out_dtype != KVB_BF16 && out_dtype != KVB_F16 && out_dtype != KVB_F32 && out_dtype != KVB_I32)
    return set_error(KVB_E_DTYPE, "w8a8_allgather: out dtype %d", out_dtype);
  if (K % 16 != 0) return set_error(KVB_E_SHAPE, "w8a8_allgather: K must be a multiple of 16");
  if (!aligned16(a) || !aligned16(b_shard)) return set_error(KVB_E_ALIGN, "w8a8_allgather: A/B must be 16-byte aligned");
  if (!is_sm100()) return set_error(KVB_E_DEVICE, "w8a8_allgather: needs an sm_100 device");
  GemmArgs g{};
  g.M = (int)M; g.N = (int)N_shard; g.K = (int)K;
  g.sa = a_scales; g.sb = b_scales_shard; g.bias = bias_shard; g.bias_dtype = bias_dtype;
  g.out = out_ptrs[rank]; g.ldo = ldo; g.out_dtype = out_dtype;
  g.n_out = g.N;
  g.nout = world;
  g.col_off = (int64_t)rank * N_shard;
  void* dests[8];
  for (int d = 0; d < world; ++d) dests[d] = g.outs[d] = out_ptrs[(rank + d) % world];   // own buffer first, then peers
  cudaStream_t st = as_stream(stream);
  // Peer destinations: stage output chunks and write them with TMA tensor stores (large NVLink writes).
  if (M <= 256) return launch_gemm<208, 4, true, false>(a, b_shard, g, dests, world, ldo, st);
  return launch_gemm<256, 6, true, true>(a, b_shard, g, dests, world, ldo, st);
}

extern "C" size_t kvb_w8a8_workspace_size(int64_t M, int64_t N, int64_t K, int b_layout, int has_azp) {
  size_t n = 256;
  if (b_layout == 1) n += (size_t)N * K + 256;      // transposed B
  if (has_azp) n += (size_t)M * 4 + 256;            // row sums of A
  return n;
}

extern "C" int kvb_w8a8_scaled_mm(const int8_t* a, const int8_t* b, int b_layout, const float* a_scales,
                                  const float* b_scales, const void* bias, int bias_dtype, const float* azp,
                                  const float* azp_adj, int64_t M, int64_t N, int64_t K, void* out, int out_dtype,
                                  int64_t ldo, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 0 || N < 0 || K < 0) return set_error(KVB_E_ARG, "w8a8_scaled_mm: negative size");
  if (M == 0 || N == 0) return KVB_OK;
  if (!a || !b || !out) return set_error(KVB_E_ARG, "w8a8_scaled_mm: null pointer");
  if (out_dtype != KVB_I32 && (!a_scales || !b_scales)) return set_error(KVB_E_ARG, "w8a8_scaled_mm: scales required");
  if (out_dtype != KVB_BF16 && out_dtype != KVB_F16 && out_dtype != KVB_F32 && out_dtype != KVB_I32)
    return set_error(KVB_E_DTYPE, "w8a8_scaled_mm: out dtype %d", out_dtype);
  if (bias && bias_dtype != KVB_BF16 && bias_dtype != KVB_F16 && bias_dtype != KVB_F32)
    return set_error(KVB_E_DTYPE, "w8a8_scaled_mm: bias dtype %d", bias_dtype);
  if (b_layout != 0 && b_layout != 1) return set_error(KVB_E_ARG, "w8a8_scaled_mm: b_layout must be 0 ([N,K]) or 1 ([K,N])");
  if (K % 16 != 0 || K == 0) return set_error(KVB_E_SHAPE, "w8a8_scaled_mm: K must be a positive multiple of 16");
  if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return set_error(KVB_E_SHAPE, "w8a8_scaled_mm: size too large");
  if (ldo < N) return set_error(KVB_E_SHAPE, "w8a8_scaled_mm: ldo < N");
  if (!aligned16(a) || (b_layout == 0 && !aligned16(b))) return set_error(KVB_E_ALIGN, "w8a8_scaled_mm: A/B must be 16-byte aligned");
  if (!is_sm100()) return set_error(KVB_E_DEVICE, "w8a8_scaled_mm: needs an sm_100 device");
  const size_t need = kvb_w8a8_workspace_size(M, N, K, b_layout, azp != nullptr);
  if ((b_layout == 1 || azp) && (!workspace || workspace_bytes < need))
    return set_error(KVB_E_WORKSPACE, "w8a8_scaled_mm: workspace %zu < %zu", workspace_bytes, need);
  cudaStream_t st = as_stream(stream);
  uint8_t* ws = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  const int8_t* b_nk = b;
  if (b_layout == 1) {
    int8_t* bt = reinterpret_cast<int8_t*>(ws);
    ws += ((size_t)N * K + 255) & ~size_t(255);
    dim3 grid((unsigned)((N + 31) / 32), (unsigned)((K + 31) / 32));
    transpose_i8_kernel<<<grid, dim3(32, 8), 0, st>>>(b, (int)K, (int)N, bt);
    int rc = check_launch("transpose_i8_kernel");
    if (rc) return rc;
    b_nk = bt;
  }
  GemmArgs g{};
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.sa = a_scales; g.sb = b_scales; g.bias = bias; g.bias_dtype = bias_dtype;
  g.azp = azp; g.azp_adj = azp_adj; g.out = out; g.ldo = ldo; g.out_dtype = out_dtype;
  g.n_out = g.N;
  if (azp) {
    int32_t* rs = reinterpret_cast<int32_t*>(ws);
    rowsum_i8_kernel<<<(unsigned)std::min<int64_t>((M + 7) / 8, 148 * 16), 256, 0, st>>>(a, (int)M, (int)K, rs);
    int rc = check_launch("rowsum_i8_kernel");
    if (rc) return rc;
    g.rowsum = rs;
  }
  // M <= 128 streams B from HBM: 208-column tiles make N = 28672 exactly 138 tiles (one wave on
  // 148 SMs).  M <= 256: CTA pairs with 256 x 448 tiles (two N = 224 MMAs per k-step sharing A:
  // 64 tiles for N = 28672, one wave on 128 SMs; 54.3 us at M = 256 against 57.9 with 256 x 512
  // tiles on 112 SMs and 60.0 with 256 x 256 tiles in two waves).  Larger M: CTA pairs with
  // 256 x 256 tiles and a double-buffered accumulator, so each tile's epilogue overlaps the next
  // tile's main loop (the single-buffered 512-column tiles lose 5-15 % there).
  void* dests[1] = {out};
  if (M <= 128) return launch_gemm<208, 5, false, false>(a, b_nk, g, dests, 1, N, st);
  if (M <= 256) return launch_gemm<224, 5, false, true, 2>(a, b_nk, g, dests, 1, N, st);
  return launch_gemm<256, 6, false, true>(a, b_nk, g, dests, 1, N, st);
}

namespace {
// Checks shared by the gated-activation entry points (N here is the weight row count).
int check_act_args(const char* who, const int8_t* a, const int8_t* b, const float* sa, const float* sb, int bias_dtype,
                   const void* bias, int64_t M, int64_t N, int64_t K, int act, int out_dtype) {
  if (M < 0 || N < 0 || K <= 0) return set_error(KVB_E_ARG, "%s: bad sizes", who);
  if (act != 1 && act != 2) return set_error(KVB_E_ARG, "%s: act must be 1 (silu(first) * second) or 2 (first * silu(second))", who);
  if (N % 256 != 0) return set_error(KVB_E_SHAPE, "%s: weight rows (%lld) must be a multiple of 256", who, (long long)N);
  if (out_dtype != KVB_BF16 && out_dtype != KVB_F16 && out_dtype != KVB_F32)
    return set_error(KVB_E_DTYPE, "%s: out dtype %d (bf16, f16 or f32)", who, out_dtype);
  if (bias && bias_dtype != KVB_BF16 && bias_dtype != KVB_F16 && bias_dtype != KVB_F32)
    return set_error(KVB_E_DTYPE, "%s: bias dtype %d", who, bias_dtype);
  if (K % 16 != 0) return set_error(KVB_E_SHAPE, "%s: K must be a multiple of 16", who);
  if (M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) return set_error(KVB_E_SHAPE, "%s: size too large", who);
  if (M > 0 && (!a || !b || !sa || !sb)) return set_error(KVB_E_ARG, "%s: null pointer", who);
  if (M > 0 && (!aligned16(a) || !aligned16(b))) return set_error(KVB_E_ALIGN, "%s: A/B must be 16-byte aligned", who);
  if (!is_sm100()) return set_error(KVB_E_DEVICE, "%s: needs an sm_100 device", who);
  return KVB_OK;
}
}  // namespace

extern "C" int kvb_w8a8_scaled_mm_act(const int8_t* a, const int8_t* b_nk, const float* a_scales, const float* b_scales,
                                      const void* bias, int bias_dtype, int64_t M, int64_t N, int64_t K, int act,
                                      void* out, int out_dtype, int64_t ldo, void* stream) {
  int rc = check_act_args("w8a8_scaled_mm_act", a, b_nk, a_scales, b_scales, bias_dtype, bias, M, N, K, act, out_dtype);
  if (rc) return rc;
  if (M == 0 || N == 0) return KVB_OK;
  if (!out) return set_error(KVB_E_ARG, "w8a8_scaled_mm_act: null output");
  if (ldo < N / 2) return set_error(KVB_E_SHAPE, "w8a8_scaled_mm_act: ldo < N / 2");
  GemmArgs g{};
  g.M = (int)M; g.N = (int)N; g.K = (int)K;
  g.sa = a_scales; g.sb = b_scales; g.bias = bias; g.bias_dtype = bias_dtype;
  g.out = out; g.ldo = ldo; g.out_dtype = out_dtype;
  g.act = act; g.n_out = (int)(N / 2);
  cudaStream_t st = as_stream(stream);
  void* dests[1] = {out};
  if (M <= 128) return launch_gemm<256, 4, false, false>(a, b_nk, g, dests, 1, N / 2, st);
  return launch_gemm<256, 6, false, true>(a, b_nk, g, dests, 1, N / 2, st);
}

extern "C" int kvb_w8a8_scaled_mm_act_allgather(const int8_t* a, const int8_t* b_shard, const float* a_scales,
                                                const float* b_scales_shard, const void* bias_shard, int bias_dtype,
                                                int64_t M, int64_t N_shard, int64_t K, int act, void* const* out_ptrs,
                                                int world, int rank, int64_t ldo, int out_dtype, void* stream) {
  if (world < 1 || world > 8 || rank < 0 || rank >= world)
    return set_error(KVB_E_ARG, "w8a8_act_allgather: world 1..8, 0 <= rank < world");
  int rc = check_act_args("w8a8_act_allgather", a, b_shard, a_scales, b_scales_shard, bias_dtype, bias_shard, M,
                          N_shard, K, act, out_dtype);
  if (rc) return rc;
  if (!out_ptrs) return set_error(KVB_E_ARG, "w8a8_act_allgather: null out_ptrs");
  for (int r = 0; r < world; ++r)
    if (!out_ptrs[r]) return set_error(KVB_E_ARG, "w8a8_act_allgather: null output pointer of rank %d", r);
  if (M == 0 || N_shard == 0) return KVB_OK;
  const int64_t out_shard = N_shard / 2;
  if (ldo < (int64_t)world * out_shard) return set_error(KVB_E_SHAPE, "w8a8_act_allgather: ldo < world * N_shard / 2");
  GemmArgs g{};
  g.M = (int)M; g.N = (int)N_shard; g.K = (int)K;
  g.sa = a_scales; g.sb = b_scales_shard; g.bias = bias_shard; g.bias_dtype = bias_dtype;
  g.out = out_ptrs[rank]; g.ldo = ldo; g.out_dtype = out_dtype;
  g.act = act; g.n_out = (int)out_shard;
  g.nout = world;
  g.col_off = (int64_t)rank * out_shard;
  void* dests[8];
  for (int d = 0; d < world; ++d) dests[d] = g.outs[d] = out_ptrs[(rank + d) % world];   // own buffer first, then peers
  cudaStream_t st = as_stream(stream);
  if (M <= 128) return launch_gemm<256, 4, true, false>(a, b_shard, g, dests, world, ldo, st);
  return launch_gemm<256, 6, true, true>(a, b_shard, g, dests, world, ldo, st);
}

