// Packed causal prefill attention on the 5th-generation tensor cores (16-bit inputs).
// Same contract as prefill.cu (operators/attention/batched_prefill_attention/batched_prefill_attention.py:30-73);
// this kernel serves f16 / bf16 with head_dim a multiple of 16 up to 128.
//
// One CTA per (128 query rows of one request, one query head), warp-specialised:
//   warp 0     TMA producer: the Q tile once, then K and V tiles of 128 keys into a 3-deep ring
//              (3-D tensor maps over [tokens, heads, D], boxes of 64 D-elements x 128 tokens with
//              the 128-byte swizzle; rows past the tensors are zero-filled);
//   warp 1     allocates TMEM (three S buffers of 128 columns + O of D columns) and one lane
//              issues the MMAs: S_j = Q K_j^T (kind::f16, M = 128, N = 128, both K-major) into
//              S[j % 3], then O += P_j V_j (M = 128, N = D, K = 128; P read from tensor memory,
//              where the softmax wrote it over S_j; V MN-major).  S_{j+1} is issued ahead of PV_j,
//              so the softmax of tile j+1 overlaps PV_j, and with three buffers S_{j+1} never
//              waits for a PV that is still running;
//   warps 2-5  softmax, one query row per thread (TMEM lane = row): the row's 128 scores in one
//              load, the row max (log2 domain, causal mask), P = 2^(s - m) rounded to the input
//              type and packed two keys per column over the scores, the running sum, and the O
//              rescale; the max is only moved when it grows by more than 2^8 (the sum and O then
//              scale by the same factor, so the result is unchanged and most tiles skip the
//              rescale); finally O / l to global memory.
// Every mbarrier wait is bounded; on a timeout the roles stop, the producer waits for its own
// copies, the MMA lane for its MMAs, and the CTA frees its TMEM before exiting.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>

#include "kvb_common.cuh"
#include "kvb_async.cuh"

namespace kvb {
namespace {

constexpr int kTcRows = 128;               // query rows per CTA (TMEM lanes)
constexpr int kTcKeys = 128;               // keys per K/V tile
constexpr int kTcThreads = 192;            // producer, MMA, four softmax warps
constexpr int kRing = 3;                   // K / V stages = S / P buffers in TMEM
constexpr uint32_t kChunkBytes = 16384;    // [128 rows x 64 elements] of a 16-bit operand
constexpr float kLazyMax = 8.0f;           // log2 growth of the row max that forces a rescale
constexpr unsigned int kStatusBadIndptrTc = 4u;

struct TcArgs {
  const int32_t* qo;
  const int32_t* kvp;
  void* out;
  int64_t total_q, total_kv;
  int batch, hq, hkv, group, D;
  float scale_log2;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// K-major operand with the 128-byte swizzle: rows of 128 B, 8-row atoms of 1024 B.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                  // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;        // stride byte offset: 8-row groups
  d |= (uint64_t)1u << 46;                  // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                  // SWIZZLE_128B
  return d;
}
// MN-major operand with the 128-byte swizzle: 64 MN-elements per 128-byte row, one row per K
// index; 8-row (K) groups 1024 B apart (stride offset), 64-element MN blocks `mn_block` B apart
// (leading offset).
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t saddr, uint32_t mn_block) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((mn_block >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}
// Instruction descriptor of kind::f16 with float32 accumulation; A K-major, B K-major or MN-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool bf16, bool b_mn_major) {
  return (1u << 4) | (bf16 ? (1u << 7) | (1u << 10) : 0u) | (b_mn_major ? (1u << 16) : 0u) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
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
// 32 lanes x 128 consecutive 32-bit columns in one load (one round trip): this thread gets its
// lane's 128 columns.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,"
      "%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,"
      "%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,"
      "%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,"
      "%121,%122,%123,%124,%125,%126,%127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]),
        "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
        "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]),
        "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]),
        "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]), "=r"(r[64]),
        "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]), "=r"(r[72]),
        "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]), "=r"(r[80]),
        "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]), "=r"(r[88]),
        "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]), "=r"(r[96]),
        "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]), "=r"(r[104]),
        "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
        "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]),
        "=r"(r[119]), "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]),
        "=r"(r[126]), "=r"(r[127])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// 32 lanes x 64 consecutive 32-bit columns stored in one instruction.
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,"
      "%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
        "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]), "r"(r[32]), "r"(r[33]), "r"(r[34]),
        "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]), "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]),
        "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]), "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]),
        "r"(r[53]), "r"(r[54]), "r"(r[55]), "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]),
        "r"(r[62]), "r"(r[63])
      : "memory");
}
// tcgen05.mma kind::f16 with A (M = 128 lanes x 16 K-elements, two 16-bit elements per 32-bit
// column, the lower K index in the low half) read from tensor memory.
__device__ __forceinline__ void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accum), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}
__device__ __forceinline__ float ex2_approx(float x) {   // 2^x (MUFU.EX2; ex2(-inf) = +0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
template <bool kBf>
__device__ __forceinline__ uint32_t pack2h(float lo, float hi) {
  if constexpr (kBf) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
// Every lane waits; the warp goes on only if all of them saw the phase complete.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait_bounded(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

// DC: 64-element chunks of D (1 or 2).  Shared memory: V ring, K ring and Q, each stage DC
// chunks of 16 KB.
template <typename T, int DC>
__global__ void __launch_bounds__(kTcThreads, 1) prefill_tc_kernel(const __grid_constant__ CUtensorMap tq,
                                                                   const __grid_constant__ CUtensorMap tk,
                                                                   const __grid_constant__ CUtensorMap tv,
                                                                   const __grid_constant__ TcArgs a) {
  constexpr bool kBf = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kOpBytes = DC * kChunkBytes;          // one Q / K / V tile
  constexpr uint32_t kV0 = 0, kK0 = kRing * kOpBytes, kQ0 = 2 * kRing * kOpBytes;
  constexpr uint32_t kTmemCols = 512;
  constexpr uint32_t kO = kRing * kTcKeys;                  // O's first TMEM column (after the S buffers)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  // One P-ready barrier per buffer (like S and PV): with a single one, a softmax that finished
  // tile j+1 before the MMA lane had seen tile j would complete two phases and the MMA lane
  // would wait for a third.
  __shared__ uint64_t q_full, k_full[kRing], v_full[kRing], kv_empty[kRing], s_full[kRing], pv_done[kRing], p_full[kRing],
      mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kRing; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&pv_done[s], 1);
    }
    for (int s = 0; s < kRing; ++s) mbar_init(&p_full[s], 4);
    mbar_init(&mma_done, 1);
    s_abort = 0;
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tq) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tk) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tv) : "memory");
  }
  pdl_trigger();
  pdl_wait();            // launched as a programmatic dependent: global data from here on

  // (request, query tile) of this CTA: request b's tiles, last first.
  int b = -1, tile = 0;
  {
    int rem = (int)blockIdx.y;
    for (int r = 0; r < a.batch; ++r) {
      const int ql = a.qo[r + 1] - a.qo[r];
      const int nt = ql > 0 ? (ql + kTcRows - 1) / kTcRows : 0;
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
    if (threadIdx.x == 0) atomicOr(&g_tu_status, kStatusBadIndptrTc);
    return;
  }
  const int i0 = tile * kTcRows;
  const int rows = min(kTcRows, ql - i0);
  const int off = kl - ql;                                 // position of query row i = off + i
  const int last = min(off + i0 + rows - 1, kl - 1);       // last key the tile attends
  const int n = last >= 0 ? last / kTcKeys + 1 : 0;        // key tiles
  const int kvh = h / a.group;
  const int D = a.D;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&q_full, kOpBytes);
      for (int c = 0; c < DC; ++c) tma_load_3d(sbase + kQ0 + c * kChunkBytes, &tq, c * 64, h, q0 + i0, &q_full);
      int issued = 0;
      for (int j = 0, s = 0, ph = 0; j < n; ++j) {            // stage s = j % kRing, ph = (j / kRing) & 1
        if (j >= kRing && !mbar_wait_bounded(&kv_empty[s], ph ^ 1)) {
          s_abort = 1;
          break;
        }
        if (s_abort) break;
        const int kt = k0 + j * kTcKeys;
        mbar_arrive_expect_tx(&k_full[s], kOpBytes);
        for (int c = 0; c < DC; ++c)
          tma_load_3d(sbase + kK0 + s * kOpBytes + c * kChunkBytes, &tk, c * 64, kvh, kt, &k_full[s]);
        mbar_arrive_expect_tx(&v_full[s], kOpBytes);
        for (int c = 0; c < DC; ++c)
          tma_load_3d(sbase + kV0 + s * kOpBytes + c * kChunkBytes, &tv, c * 64, kvh, kt, &v_full[s]);
        issued = j + 1;
        if (++s == kRing) {
          s = 0;
          ph ^= 1;
        }
      }
      // every copy this CTA issued has landed before it exits
      mbar_wait_bounded(&q_full, 0);
      for (int j = issued > kRing ? issued - kRing : 0; j < issued; ++j) {
        mbar_wait_bounded(&k_full[j % kRing], (j / kRing) & 1);
        mbar_wait_bounded(&v_full[j % kRing], (j / kRing) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(kTcRows, kTcKeys, kBf, false);
      const uint32_t id_pv = idesc_f16(kTcRows, D, kBf, true);
      const int ksteps = D / 16;
      // S_j into S buffer j % kRing once K_j has landed and PV_{j-kRing} has consumed the P that
      // buffer held
      auto issue_s = [&](int j) -> bool {
        const int s = j % kRing;
        const uint32_t ph = (uint32_t)(j / kRing) & 1u;
        if (!mbar_wait_bounded(&k_full[s], ph)) return false;
        if (j >= kRing && !mbar_wait_bounded(&pv_done[s], ph ^ 1u)) return false;
        tc_fence_after();
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint32_t off_b = (uint32_t)(ks >> 2) * kChunkBytes + (uint32_t)(ks & 3) * 32u;
          mma_f16(tmem + (uint32_t)s * kTcKeys, desc_kmajor(sbase + kQ0 + off_b),
                  desc_kmajor(sbase + kK0 + s * kOpBytes + off_b), kIdS, ks > 0);
        }
        mma_commit(&s_full[s]);
        return true;
      };
      bool ok = n == 0 || (mbar_wait_bounded(&q_full, 0) && issue_s(0));
      for (int j = 0; j < n && ok && !s_abort; ++j) {
        if (j + 1 < n && !issue_s(j + 1)) {
          ok = false;
          break;
        }
        const int s = j % kRing;
        if (!mbar_wait_bounded(&p_full[s], (j / kRing) & 1) || !mbar_wait_bounded(&v_full[s], (j / kRing) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vs = sbase + kV0 + s * kOpBytes;
#pragma unroll
        for (int ks = 0; ks < kTcKeys / 16; ++ks)   // P_j: 16 keys = 8 packed columns of S buffer s
          mma_f16_ts(tmem + kO, tmem + (uint32_t)s * kTcKeys + (uint32_t)ks * 8u,
                     desc_mnmajor(vs + (uint32_t)ks * 2048u, kChunkBytes), id_pv, (j | ks) != 0);
        mma_commit(&pv_done[s]);
        mma_commit(&kv_empty[s]);
      }
      if (!ok) s_abort = 1;
      mma_commit(&mma_done);                 // every MMA issued above has completed before TMEM is freed
      mbar_wait_bounded(&mma_done, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax (warps 2-5)
    const int quarter = warp & 3;                          // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;                   // query row of the tile = TMEM lane
    const int pos = off + i0 + row;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const float sc = a.scale_log2;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j % kRing;                            // S / P buffer of tile j
      if (__shfl_sync(0xffffffffu, s_abort, 0) || !warp_wait(&s_full[sb], (j / kRing) & 1)) {   // warp-uniform
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = tmem + lane_addr + (uint32_t)sb * kTcKeys;
      const int kb = j * kTcKeys;
      const bool mask = kb + kTcKeys - 1 > off + i0 + quarter * 32;   // some key of the tile may pass a row
      // the row's 128 scores in one load
      uint32_t r[128];
      tmem_ld128(sa, r);
      if (mask) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kb + i > pos) r[i] = __float_as_uint(sc >= 0.0f ? -INFINITY : INFINITY);
      }
      // the tile's row max in the log2 domain (the raw extreme times the scale)
      float mx;
      if (sc >= 0.0f) {
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 128; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(r[i]));
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      } else {
        float m4[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
#pragma unroll
        for (int i = 0; i < 128; ++i) m4[i & 3] = fminf(m4[i & 3], __uint_as_float(r[i]));
        mx = fminf(fminf(m4[0], m4[1]), fminf(m4[2], m4[3]));
      }
      mx *= sc;
      const bool grow = mx > m_used + kLazyMax;
      const float alpha = grow ? ex2_approx(m_used - mx) : 1.0f;
      if (grow) m_used = mx;
      l *= alpha;
      // P = 2^(s * scale - m) in the input type (masked scores give 2^-inf = 0), two keys per
      // 32-bit column over the first 64 columns of the row's scores: the A operand of PV_j
      const float neg_m = -m_used;
      float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint32_t w[64];
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(r[i]), sc, neg_m));
        const float p1 = ex2_approx(fmaf(__uint_as_float(r[i + 1]), sc, neg_m));
        l4[(i >> 1) & 3] += p0 + p1;
        w[i >> 1] = pack2h<kBf>(p0, p1);
      }
      tmem_st64(sa, w);
      l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      // O *= alpha where the max moved (whole warp, when any of its rows needs it), once PV_{j-1}
      // has completed
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        if (!warp_wait(&pv_done[(j - 1) % kRing], ((j - 1) / kRing) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int c = 0; c < (D + 31) / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_addr + kO + c * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          tmem_st32(tmem + lane_addr + kO + c * 32, r);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    if (!ok) s_abort = 1;
    // O / l of the valid rows
    if (ok && (n == 0 || warp_wait(&pv_done[(n - 1) % kRing], ((n - 1) / kRing) & 1))) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const bool valid = i0 + row < ql;
      T* orow = reinterpret_cast<T*>(a.out) + ((int64_t)q0 + i0 + row) * a.hq * D + (int64_t)h * D;
      for (int c = 0; c < (D + 31) / 32; ++c) {
        uint32_t r[32];
        if (n > 0) tmem_ld32(tmem + lane_addr + kO + c * 32, r);
        else
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = 0u;
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          w[i >> 1] = pack2h<kBf>(__uint_as_float(r[i]) * inv, __uint_as_float(r[i + 1]) * inv);
        if (valid) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (c * 32 + u * 8 < D)
              *reinterpret_cast<uint4*>(orow + c * 32 + u * 8) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
        }
      }
    } else {
      s_abort = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// Two query tiles per CTA (ping-pong): rows [i0, i0 + 256) of one request and one query head as
// tiles A = [i0, i0 + 128) and B = [i0 + 128, i0 + 256), sharing every K / V tile.  Each tile has
// one S buffer and its O in tensor memory (S_A | O_A | S_B | O_B = 512 columns), its own group
// of four softmax warps (warps 2-5: A, 6-9: B), and its chain S_j -> softmax -> PV_j -> S_{j+1};
// the MMA lane interleaves the two chains, so one tile's exponentials overlap the other tile's
// MMAs, and each K / V byte staged in shared memory serves 256 query rows.
constexpr int kPpThreads = 320;            // producer, MMA, two softmax groups of four warps
constexpr int kPpRing = 2;                 // K / V stages
#ifndef KVB_PREFILL_PP_MIN_BLOCKS
#define KVB_PREFILL_PP_MIN_BLOCKS 148
#endif
constexpr int kPpMinBlocks = KVB_PREFILL_PP_MIN_BLOCKS;   // (head, 256-row block) items from which auto picks it

template <typename T, int DC>
__global__ void __launch_bounds__(kPpThreads, 1) prefill_pp_kernel(const __grid_constant__ CUtensorMap tq,
                                                                   const __grid_constant__ CUtensorMap tk,
                                                                   const __grid_constant__ CUtensorMap tv,
                                                                   const __grid_constant__ TcArgs a) {
  constexpr bool kBf = std::is_same<T, __nv_bfloat16>::value;
  constexpr uint32_t kOpBytes = DC * kChunkBytes;          // one Q / K / V tile
  constexpr uint32_t kV0 = 0, kK0 = kPpRing * kOpBytes, kQ0 = 2 * kPpRing * kOpBytes;   // Q tile t at kQ0 + t * kOpBytes
  constexpr uint32_t kTmemCols = 512;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  // s_full / p_full / pv_done: one per query tile, one phase per key tile of that query tile.
  __shared__ uint64_t q_full, k_full[kPpRing], v_full[kPpRing], kv_empty[kPpRing], s_full[2], p_full[2], pv_done[2],
      mma_done;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int s_abort;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x;
  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int s = 0; s < kPpRing; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_full[t], 4);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(&mma_done, 1);
    s_abort = 0;
    fence_mbar_init();
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tq) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tk) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&tv) : "memory");
  }
  pdl_trigger();
  pdl_wait();            // launched as a programmatic dependent: global data from here on

  // (request, 256-row block) of this CTA: request b's blocks, last first.
  int b = -1, blk = 0;
  {
    int rem = (int)blockIdx.y;
    for (int r = 0; r < a.batch; ++r) {
      const int ql = a.qo[r + 1] - a.qo[r];
      const int nb = ql > 0 ? (ql + 2 * kTcRows - 1) / (2 * kTcRows) : 0;
      if (rem < nb) {
        b = r;
        blk = nb - 1 - rem;
        break;
      }
      rem -= nb;
    }
  }
  if (b < 0) return;
  const int q0 = a.qo[b], ql = a.qo[b + 1] - q0;
  const int k0 = a.kvp[b], kl = a.kvp[b + 1] - k0;
  if (q0 < 0 || (int64_t)q0 + ql > a.total_q || k0 < 0 || kl < 0 || (int64_t)k0 + kl > a.total_kv) {
    if (threadIdx.x == 0) atomicOr(&g_tu_status, kStatusBadIndptrTc);
    return;
  }
  const int i0 = blk * 2 * kTcRows;
  const int off = kl - ql;                                 // position of query row i = off + i
  int nt[2];                                               // key tiles of query tile t (0: tile empty)
  for (int t = 0; t < 2; ++t) {
    const int rows = min(kTcRows, ql - (i0 + t * kTcRows));
    const int last = min(off + i0 + t * kTcRows + rows - 1, kl - 1);   // last key the tile attends
    nt[t] = (rows > 0 && last >= 0) ? last / kTcKeys + 1 : 0;
  }
  const int n = max(nt[0], nt[1]);                          // key tiles of the CTA
  const bool two = ql - i0 > kTcRows;                        // tile B holds rows
  const int kvh = h / a.group;
  const int D = a.D;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(&q_full, (two ? 2u : 1u) * kOpBytes);
      for (int t = 0; t < (two ? 2 : 1); ++t)
        for (int c = 0; c < DC; ++c)
          tma_load_3d(sbase + kQ0 + t * kOpBytes + c * kChunkBytes, &tq, c * 64, h, q0 + i0 + t * kTcRows, &q_full);
      int issued = 0;
      for (int j = 0, s = 0, ph = 0; j < n; ++j) {            // stage s = j % kPpRing, ph = (j / kPpRing) & 1
        if (j >= kPpRing && !mbar_wait_bounded(&kv_empty[s], ph ^ 1)) {
          s_abort = 1;
          break;
        }
        if (s_abort) break;
        const int kt = k0 + j * kTcKeys;
        mbar_arrive_expect_tx(&k_full[s], kOpBytes);
        for (int c = 0; c < DC; ++c)
          tma_load_3d(sbase + kK0 + s * kOpBytes + c * kChunkBytes, &tk, c * 64, kvh, kt, &k_full[s]);
        mbar_arrive_expect_tx(&v_full[s], kOpBytes);
        for (int c = 0; c < DC; ++c)
          tma_load_3d(sbase + kV0 + s * kOpBytes + c * kChunkBytes, &tv, c * 64, kvh, kt, &v_full[s]);
        issued = j + 1;
        if (++s == kPpRing) {
          s = 0;
          ph ^= 1;
        }
      }
      // every copy this CTA issued has landed before it exits
      mbar_wait_bounded(&q_full, 0);
      for (int j = issued > kPpRing ? issued - kPpRing : 0; j < issued; ++j) {
        mbar_wait_bounded(&k_full[j % kPpRing], (j / kPpRing) & 1);
        mbar_wait_bounded(&v_full[j % kPpRing], (j / kPpRing) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdS = idesc_f16(kTcRows, kTcKeys, kBf, false);
      const uint32_t id_pv = idesc_f16(kTcRows, D, kBf, true);
      const int ksteps = D / 16;
      // S_j of tile t into its S buffer (K_j has landed; the caller has seen PV_{j-1} of the tile,
      // which read the P this buffer held, complete)
      auto issue_s = [&](int t, int j) -> bool {
        const int s = j % kPpRing;
        if (!mbar_wait_bounded(&k_full[s], (uint32_t)(j / kPpRing) & 1u)) return false;
        tc_fence_after();
        for (int ks = 0; ks < ksteps; ++ks) {
          const uint32_t off_b = (uint32_t)(ks >> 2) * kChunkBytes + (uint32_t)(ks & 3) * 32u;
          mma_f16(tmem + (uint32_t)t * 256u, desc_kmajor(sbase + kQ0 + t * kOpBytes + off_b),
                  desc_kmajor(sbase + kK0 + s * kOpBytes + off_b), kIdS, ks > 0);
        }
        mma_commit(&s_full[t]);
        return true;
      };
      bool ok = mbar_wait_bounded(&q_full, 0);
      for (int t = 0; t < 2 && ok; ++t)
        if (nt[t] > 0) ok = issue_s(t, 0);
      for (int j = 0; j < n && ok && !s_abort; ++j) {
        const int s = j % kPpRing;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= nt[t]) continue;
          if (!mbar_wait_bounded(&p_full[t], (uint32_t)j & 1u) ||
              !mbar_wait_bounded(&v_full[s], (uint32_t)(j / kPpRing) & 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t vs = sbase + kV0 + s * kOpBytes;
#pragma unroll
          for (int ks = 0; ks < kTcKeys / 16; ++ks)   // P_j: 16 keys = 8 packed columns of the tile's S buffer
            mma_f16_ts(tmem + (uint32_t)t * 256u + 128u, tmem + (uint32_t)t * 256u + (uint32_t)ks * 8u,
                       desc_mnmajor(vs + (uint32_t)ks * 2048u, kChunkBytes), id_pv, (j | ks) != 0);
          mma_commit(&pv_done[t]);
          if (j + 1 < nt[t]) {
            // S_{j+1} overwrites the P that PV_j reads: wait for PV_j first
            if (!mbar_wait_bounded(&pv_done[t], (uint32_t)j & 1u)) {
              ok = false;
              break;
            }
            ok = issue_s(t, j + 1);
          }
        }
        mma_commit(&kv_empty[s]);              // K_j and V_j are free once the MMAs above complete
      }
      if (!ok) s_abort = 1;
      mma_commit(&mma_done);                   // every MMA issued above has completed before TMEM is freed
      mbar_wait_bounded(&mma_done, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax (warps 2-5: tile A, 6-9: tile B)
    const int t = (warp - 2) >> 2;                         // query tile of this warp
    const int quarter = warp & 3;                          // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;                   // query row of the tile = TMEM lane
    const int ti0 = i0 + t * kTcRows;                      // first query row of the tile
    const int pos = off + ti0 + row;
    const int nj = nt[t];
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    const uint32_t s_col = (uint32_t)t * 256u, o_col = s_col + 128u;
    const float sc = a.scale_log2;
    float m_used = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < nj; ++j) {
      if (__shfl_sync(0xffffffffu, s_abort, 0) || !warp_wait(&s_full[t], (uint32_t)j & 1u)) {   // warp-uniform
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = tmem + lane_addr + s_col;
      const int kb = j * kTcKeys;
      const bool mask = kb + kTcKeys - 1 > off + ti0 + quarter * 32;   // some key of the tile may pass a row
      uint32_t r[128];
      tmem_ld128(sa, r);
      if (mask) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kb + i > pos) r[i] = __float_as_uint(sc >= 0.0f ? -INFINITY : INFINITY);
      }
      float mx;
      if (sc >= 0.0f) {
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < 128; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(r[i]));
        mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      } else {
        float m4[4] = {INFINITY, INFINITY, INFINITY, INFINITY};
#pragma unroll
        for (int i = 0; i < 128; ++i) m4[i & 3] = fminf(m4[i & 3], __uint_as_float(r[i]));
        mx = fminf(fminf(m4[0], m4[1]), fminf(m4[2], m4[3]));
      }
      mx *= sc;
      const bool grow = mx > m_used + kLazyMax;
      const float alpha = grow ? ex2_approx(m_used - mx) : 1.0f;
      if (grow) m_used = mx;
      l *= alpha;
      const float neg_m = -m_used;
      float l4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {                    // 64 keys -> 32 packed columns at a time
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < 64; i += 2) {
          const float p0 = ex2_approx(fmaf(__uint_as_float(r[64 * hf + i]), sc, neg_m));
          const float p1 = ex2_approx(fmaf(__uint_as_float(r[64 * hf + i + 1]), sc, neg_m));
          l4[(i >> 1) & 3] += p0 + p1;
          w[i >> 1] = pack2h<kBf>(p0, p1);
        }
        tmem_st32(sa + 32u * hf, w);
      }
      l += (l4[0] + l4[1]) + (l4[2] + l4[3]);
      // O *= alpha where the max moved (whole warp, when any of its rows needs it), once PV_{j-1}
      // has completed
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        if (!warp_wait(&pv_done[t], (uint32_t)(j - 1) & 1u)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int c = 0; c < (D + 31) / 32; ++c) {
          uint32_t r2[32];
          tmem_ld32(tmem + lane_addr + o_col + c * 32, r2);
#pragma unroll
          for (int i = 0; i < 32; ++i) r2[i] = __float_as_uint(__uint_as_float(r2[i]) * alpha);
          tmem_st32(tmem + lane_addr + o_col + c * 32, r2);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[t]);
    }
    if (!ok) s_abort = 1;
    // O / l of the valid rows
    if (ok && (nj == 0 || warp_wait(&pv_done[t], (uint32_t)(nj - 1) & 1u))) {
      tc_fence_after();
      const float inv = 1.0f / l;
      const bool valid = ti0 + row < ql;
      T* orow = reinterpret_cast<T*>(a.out) + ((int64_t)q0 + ti0 + row) * a.hq * D + (int64_t)h * D;
      for (int c = 0; c < (D + 31) / 32; ++c) {
        uint32_t r2[32];
        if (nj > 0) tmem_ld32(tmem + lane_addr + o_col + c * 32, r2);
        else
#pragma unroll
          for (int i = 0; i < 32; ++i) r2[i] = 0u;
        uint32_t w[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          w[i >> 1] = pack2h<kBf>(__uint_as_float(r2[i]) * inv, __uint_as_float(r2[i + 1]) * inv);
        if (valid) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            if (c * 32 + u * 8 < D)
              *reinterpret_cast<uint4*>(orow + c * 32 + u * 8) = make_uint4(w[4 * u], w[4 * u + 1], w[4 * u + 2], w[4 * u + 3]);
        }
      }
    } else {
      s_abort = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_tiled() {
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

// [tokens, heads, D] 16-bit tensor; box of 64 D-elements x 1 head x 128 tokens, 128-byte swizzle,
// zero fill out of bounds.
int make_head_map(CUtensorMap* map, const void* base, bool bf16, int64_t tokens, int heads, int D) {
  auto fn = encode_tiled();
  if (!fn) return set_error(KVB_E_LAUNCH, "batched_prefill_attention: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)heads, (cuuint64_t)tokens};
  cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)heads * D * 2};
  cuuint32_t box[3] = {64u, 1u, (cuuint32_t)kTcRows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(KVB_E_LAUNCH, "batched_prefill_attention: tensor map failed (%d)", (int)r);
  return KVB_OK;
}

template <typename T, int DC>
int launch_tc(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const TcArgs& a, int tiles_ub,
              cudaStream_t st) {
  constexpr size_t smem = (2 * kRing + 1) * (size_t)DC * kChunkBytes + 1024;
  auto kern = prefill_tc_kernel<T, DC>;
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "batched_prefill_attention: smem attribute: %s", cudaGetErrorString(e));
    set_dev = dev;
  }
  cudaError_t e = launch_pdl(kern, dim3((unsigned)a.hq, (unsigned)tiles_ub), dim3(kTcThreads), smem, st, mq, mk, mv, a);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "prefill_tc_kernel: %s", cudaGetErrorString(e));
  return check_launch("prefill_tc_kernel");
}

template <typename T, int DC>
int launch_pp(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const TcArgs& a, int blocks_ub,
              cudaStream_t st) {
  constexpr size_t smem = (2 * kPpRing + 2) * (size_t)DC * kChunkBytes + 1024;
  auto kern = prefill_pp_kernel<T, DC>;
  static int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (set_dev != dev) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "batched_prefill_attention: smem attribute: %s", cudaGetErrorString(e));
    set_dev = dev;
  }
  cudaError_t e = launch_pdl(kern, dim3((unsigned)a.hq, (unsigned)blocks_ub), dim3(kPpThreads), smem, st, mq, mk, mv, a);
  if (e != cudaSuccess) return set_error(KVB_E_LAUNCH, "prefill_pp_kernel: %s", cudaGetErrorString(e));
  return check_launch("prefill_pp_kernel");
}

}  // namespace

// Host entry used by prefill.cu for 16-bit inputs with head_dim % 16 == 0 and <= 128.  kernel: 0
// = automatic, 1 = one query tile per CTA, 2 = two query tiles per CTA.
int prefill_tcgen05(const void* q, const void* k, const void* v, bool bf16, const int32_t* qo, const int32_t* kvp,
                    int batch, int64_t total_q, int64_t total_kv, int hq, int hkv, int D, float scale_log2, void* out,
                    int kernel, cudaStream_t st) {
  const int64_t tiles_ub = total_q / kTcRows + batch;
  if (tiles_ub > 65535) return set_error(KVB_E_SHAPE, "batched_prefill_attention: too many query tiles");
  CUtensorMap mq, mk, mv;
  int rc = make_head_map(&mq, q, bf16, total_q, hq, D);
  if (!rc) rc = make_head_map(&mk, k, bf16, total_kv, hkv, D);
  if (!rc) rc = make_head_map(&mv, v, bf16, total_kv, hkv, D);
  if (rc) return rc;
  TcArgs a{};
  a.qo = qo; a.kvp = kvp; a.out = out; a.total_q = total_q; a.total_kv = total_kv;
  a.batch = batch; a.hq = hq; a.hkv = hkv; a.group = hq / hkv; a.D = D; a.scale_log2 = scale_log2;
  // Two query tiles per CTA once the (head, 256-row block) items fill the SMs (bf16, 32 / 8 heads,
  // D = 128: 118.0 -> 107.2 us at q_lens [2048, 1536, 1024, 512], 650 -> 593 us at [8192, 512,
  // 128, 32], 106.4 -> 101.0 us for 4 x 512 queries on 4096-1024 keys); smaller inputs keep one
  // tile per CTA for the parallelism.
  const int64_t blocks_ub = total_q / (2 * kTcRows) + batch;
  const bool pp = kernel == 2 || (kernel == 0 && (int64_t)hq * (total_q / (2 * kTcRows)) >= kPpMinBlocks);
  if (pp) {
    if (D <= 64) return bf16 ? launch_pp<__nv_bfloat16, 1>(mq, mk, mv, a, (int)blocks_ub, st)
                             : launch_pp<__half, 1>(mq, mk, mv, a, (int)blocks_ub, st);
    return bf16 ? launch_pp<__nv_bfloat16, 2>(mq, mk, mv, a, (int)blocks_ub, st)
                : launch_pp<__half, 2>(mq, mk, mv, a, (int)blocks_ub, st);
  }
  if (D <= 64) return bf16 ? launch_tc<__nv_bfloat16, 1>(mq, mk, mv, a, (int)tiles_ub, st)
                           : launch_tc<__half, 1>(mq, mk, mv, a, (int)tiles_ub, st);
  return bf16 ? launch_tc<__nv_bfloat16, 2>(mq, mk, mv, a, (int)tiles_ub, st)
              : launch_tc<__half, 2>(mq, mk, mv, a, (int)tiles_ub, st);
}

}  // namespace kvb
