// Paged KV-cache writes.
//
// * kvb_paged_kv_cache_update: the reference's clone-then-scatter
//   (operators/kv_cache/paged_kv_cache_update/paged_kv_cache_update.py:27-31): an optional
//   vectorised copy of the whole cache into the output, then token i overwrites flat slot
//   slot_mapping[i] (skipped when negative).
// * kvb_paged_fp8_kv_write: the BASELINE fourth config's write -- token i, head h is stored
//   as e4m3(clamp(x / scale[h], +-448)) codes in slot slot_mapping[i].
// * kvb_kv_cache_write: operators/kv_cache/kv_cache_write/kv_cache_write.py:24-58 -- copies
//   of the [batch, heads, max_seq_len, head_dim] caches with the new rows scattered in at
//   their positions.
// Slots are bounds-checked on the device: an index >= num_slots is skipped and recorded in
// the status word (kvb_device_status bit 1).
#include "kvb_common.cuh"
#include "kvb_async.cuh"

namespace kvb {
namespace {

constexpr unsigned int kStatusBadSlot = 2u;

__device__ __forceinline__ int64_t load_slot(const void* sm, int idx64, int64_t i) {
  return idx64 ? reinterpret_cast<const int64_t*>(sm)[i] : (int64_t)reinterpret_cast<const int32_t*>(sm)[i];
}

__global__ void __launch_bounds__(256) copy16_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, int64_t n16) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __ldcs(src + i);
}
__global__ void __launch_bounds__(256) copy1_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// One CTA per token; the slot row (slot_bytes) is copied with 16-byte (or byte) accesses.
__global__ void __launch_bounds__(128) scatter_rows_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ cache,
                                                           const void* slot_mapping, int idx64, int64_t num_slots,
                                                           int64_t slot_bytes, int vec16) {
  const int64_t i = blockIdx.x;
  const int64_t slot = load_slot(slot_mapping, idx64, i);
  if (slot < 0) return;
  if (slot >= num_slots) {
    if (threadIdx.x == 0) atomicOr(&g_tu_status, kStatusBadSlot);
    return;
  }
  const uint8_t* s = src + i * slot_bytes;
  uint8_t* d = cache + slot * slot_bytes;
  if (vec16) {
    for (int64_t k = threadIdx.x; k < slot_bytes / 16; k += blockDim.x)
      reinterpret_cast<uint4*>(d)[k] = reinterpret_cast<const uint4*>(s)[k];
  } else {
    for (int64_t k = threadIdx.x; k < slot_bytes; k += blockDim.x) d[k] = s[k];
  }
}

// One thread per (token, head, 8 elements).
template <typename T>
__global__ void __launch_bounds__(256) fp8_kv_write_kernel(const T* __restrict__ x, uint8_t* __restrict__ cache,
                                                           const void* slot_mapping, int idx64, const float* __restrict__ scales,
                                                           int64_t num_tokens, int64_t num_slots, int heads, int head_dim) {
  const int vec_per_head = head_dim / 8;
  const int64_t total = num_tokens * heads * vec_per_head;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < total; v += (int64_t)gridDim.x * blockDim.x) {
    const int64_t tok = v / (heads * vec_per_head);
    const int h = (int)((v / vec_per_head) % heads);
    const int64_t slot = load_slot(slot_mapping, idx64, tok);
    if (slot < 0) continue;
    if (slot >= num_slots) {
      atomicOr(&g_tu_status, kStatusBadSlot);
      continue;
    }
    Vec8<T> a;
    a.load(x + v * 8);
    float f[8];
    a.unpack(f);
    const Divisor d = make_divisor(scales[h]);
    const uint32_t lo = quant_e4m3x2(f[0], f[1], d) | ((uint32_t)quant_e4m3x2(f[2], f[3], d) << 16);
    const uint32_t hi = quant_e4m3x2(f[4], f[5], d) | ((uint32_t)quant_e4m3x2(f[6], f[7], d) << 16);
    const int64_t within = v % ((int64_t)heads * vec_per_head);
    *reinterpret_cast<uint2*>(cache + slot * (int64_t)heads * head_dim + within * 8) = make_uint2(lo, hi);
  }
}

// kv_cache_write: one warp per written row (b, h, w) of K (blockIdx.y == 0) or V (1); the row of
// head_dim elements goes to position positions[w] (shared) or positions[b, w] (per batch).
__global__ void __launch_bounds__(128) kv_write_rows_kernel(const uint8_t* __restrict__ key, const uint8_t* __restrict__ value,
                                                            uint8_t* __restrict__ k_out, uint8_t* __restrict__ v_out,
                                                            const void* positions, int idx64, int per_batch, int64_t rows,
                                                            int64_t heads, int64_t max_seq_len, int64_t write_len,
                                                            int64_t row_bytes, int vec16) {
  const int64_t r = (int64_t)blockIdx.x * 4 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t w = r % write_len, bh = r / write_len, b = bh / heads;
  int64_t pos = load_slot(positions, idx64, per_batch ? b * write_len + w : w);
  if (pos < 0) pos += max_seq_len;                 // torch indexing: negative positions count from the end
  if (pos < 0 || pos >= max_seq_len) {
    if (lane == 0) atomicOr(&g_tu_status, kStatusBadSlot);
    return;
  }
  const uint8_t* src = (blockIdx.y ? value : key) + r * row_bytes;
  uint8_t* dst = (blockIdx.y ? v_out : k_out) + (bh * max_seq_len + pos) * row_bytes;
  if (vec16) {
    for (int64_t k = lane; k < row_bytes / 16; k += 32)
      reinterpret_cast<uint4*>(dst)[k] = reinterpret_cast<const uint4*>(src)[k];
  } else {
    for (int64_t k = lane; k < row_bytes; k += 32) dst[k] = src[k];
  }
}

int grid_for(int64_t work, int threads) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t g = (work + threads - 1) / threads;
  if (g > (int64_t)sms * 8) g = (int64_t)sms * 8;
  return (int)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace kvb

using namespace kvb;

extern "C" int kvb_paged_kv_cache_update(const void* to_cache, const void* kv_cache_in, void* kv_cache_out,
                                         const void* slot_mapping, int index_dtype, int dtype, int64_t num_tokens,
                                         int64_t num_slots, int64_t slot_elems, void* stream) {
  if (num_tokens < 0 || num_slots < 0 || slot_elems < 0) return set_error(KVB_E_ARG, "paged_kv_cache_update: negative size");
  if (index_dtype != KVB_I32 && index_dtype != KVB_I64) return set_error(KVB_E_DTYPE, "paged_kv_cache_update: index dtype");
  const int es = dtype == KVB_E4M3 ? 1 : dtype_size(dtype);
  if (es <= 0) return set_error(KVB_E_DTYPE, "paged_kv_cache_update: dtype %d", dtype);
  if (!kv_cache_out || (num_tokens > 0 && (!to_cache || !slot_mapping)))
    return set_error(KVB_E_ARG, "paged_kv_cache_update: null pointer");
  cudaStream_t st = as_stream(stream);
  const int64_t slot_bytes = slot_elems * es;
  if (kv_cache_in && kv_cache_in != kv_cache_out) {
    const int64_t n = num_slots * slot_bytes;
    if (aligned16(kv_cache_in) && aligned16(kv_cache_out) && n % 16 == 0) {
      copy16_kernel<<<grid_for(n / 16, 256), 256, 0, st>>>(reinterpret_cast<const uint4*>(kv_cache_in),
                                                          reinterpret_cast<uint4*>(kv_cache_out), n / 16);
    } else {
      copy1_kernel<<<grid_for(n, 256), 256, 0, st>>>(reinterpret_cast<const uint8_t*>(kv_cache_in),
                                                    reinterpret_cast<uint8_t*>(kv_cache_out), n);
    }
    int rc = check_launch("copy_kernel");
    if (rc) return rc;
  }
  if (num_tokens == 0 || slot_bytes == 0) return KVB_OK;
  if (num_tokens > 0x7fffffffLL) return set_error(KVB_E_SHAPE, "paged_kv_cache_update: too many tokens");
  const int vec16 = slot_bytes % 16 == 0 && aligned16(to_cache) && aligned16(kv_cache_out);
  scatter_rows_kernel<<<(unsigned)num_tokens, 128, 0, st>>>(reinterpret_cast<const uint8_t*>(to_cache),
                                                            reinterpret_cast<uint8_t*>(kv_cache_out), slot_mapping,
                                                            index_dtype == KVB_I64, num_slots, slot_bytes, vec16);
  return check_launch("scatter_rows_kernel");
}

namespace {
int copy_cache(const void* in, void* out, int64_t n, cudaStream_t st) {
  if (!in || in == out || n == 0) return KVB_OK;
  if (aligned16(in) && aligned16(out) && n % 16 == 0)
    copy16_kernel<<<grid_for(n / 16, 256), 256, 0, st>>>(reinterpret_cast<const uint4*>(in), reinterpret_cast<uint4*>(out),
                                                        n / 16);
  else
    copy1_kernel<<<grid_for(n, 256), 256, 0, st>>>(reinterpret_cast<const uint8_t*>(in), reinterpret_cast<uint8_t*>(out), n);
  return check_launch("copy_kernel");
}
}  // namespace

extern "C" int kvb_kv_cache_write(const void* key, const void* value, const void* k_cache_in, const void* v_cache_in,
                                  void* k_cache_out, void* v_cache_out, const void* positions, int index_dtype,
                                  int per_batch, int dtype, int64_t batch, int64_t heads, int64_t max_seq_len,
                                  int64_t write_len, int64_t head_dim, void* stream) {
  if (batch < 0 || heads < 0 || max_seq_len < 0 || write_len < 0 || head_dim < 0)
    return set_error(KVB_E_ARG, "kv_cache_write: negative size");
  if (index_dtype != KVB_I32 && index_dtype != KVB_I64) return set_error(KVB_E_DTYPE, "kv_cache_write: index dtype");
  const int es = dtype == KVB_E4M3 ? 1 : dtype_size(dtype);
  if (es <= 0) return set_error(KVB_E_DTYPE, "kv_cache_write: dtype %d", dtype);
  if (!k_cache_out || !v_cache_out) return set_error(KVB_E_ARG, "kv_cache_write: null output");
  const int64_t rows = batch * heads * write_len, row_bytes = head_dim * es;
  if (rows > 0 && (!key || !value || !positions)) return set_error(KVB_E_ARG, "kv_cache_write: null pointer");
  cudaStream_t st = as_stream(stream);
  const int64_t cache_bytes = batch * heads * max_seq_len * row_bytes;
  int rc = copy_cache(k_cache_in, k_cache_out, cache_bytes, st);
  if (!rc) rc = copy_cache(v_cache_in, v_cache_out, cache_bytes, st);
  if (rc || rows == 0 || row_bytes == 0) return rc;
  if ((rows + 3) / 4 > 0x7fffffffLL) return set_error(KVB_E_SHAPE, "kv_cache_write: too many rows");
  const int vec16 = row_bytes % 16 == 0 && aligned16(key) && aligned16(value) && aligned16(k_cache_out) &&
                    aligned16(v_cache_out);
  dim3 grid((unsigned)((rows + 3) / 4), 2);
  kv_write_rows_kernel<<<grid, 128, 0, st>>>(reinterpret_cast<const uint8_t*>(key), reinterpret_cast<const uint8_t*>(value),
                                             reinterpret_cast<uint8_t*>(k_cache_out), reinterpret_cast<uint8_t*>(v_cache_out),
                                             positions, index_dtype == KVB_I64, per_batch, rows, heads, max_seq_len,
                                             write_len, row_bytes, vec16);
  return check_launch("kv_write_rows_kernel");
}

extern "C" int kvb_paged_fp8_kv_write(const void* x_new, int x_dtype, void* cache, const void* slot_mapping,
                                      int index_dtype, const float* head_scales, int64_t num_tokens, int64_t num_slots,
                                      int num_heads, int head_dim, void* stream) {
  if (num_tokens < 0 || num_slots < 0 || num_heads <= 0 || head_dim <= 0)
    return set_error(KVB_E_ARG, "paged_fp8_kv_write: bad sizes");
  if (num_tokens == 0) return KVB_OK;
  if (!x_new || !cache || !slot_mapping || !head_scales) return set_error(KVB_E_ARG, "paged_fp8_kv_write: null pointer");
  if (head_dim % 8) return set_error(KVB_E_SHAPE, "paged_fp8_kv_write: head_dim must be a multiple of 8");
  if (index_dtype != KVB_I32 && index_dtype != KVB_I64) return set_error(KVB_E_DTYPE, "paged_fp8_kv_write: index dtype");
  if (!aligned16(x_new) || !aligned8(cache)) return set_error(KVB_E_ALIGN, "paged_fp8_kv_write: x 16-byte / cache 8-byte alignment");
  cudaStream_t st = as_stream(stream);
  const int64_t work = num_tokens * num_heads * (head_dim / 8);
  const int idx64 = index_dtype == KVB_I64;
  uint8_t* c = reinterpret_cast<uint8_t*>(cache);
  switch (x_dtype) {
    case KVB_BF16:
      fp8_kv_write_kernel<__nv_bfloat16><<<grid_for(work, 256), 256, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(x_new), c, slot_mapping, idx64, head_scales, num_tokens, num_slots,
          num_heads, head_dim);
      break;
    case KVB_F16:
      fp8_kv_write_kernel<__half><<<grid_for(work, 256), 256, 0, st>>>(reinterpret_cast<const __half*>(x_new), c,
                                                                       slot_mapping, idx64, head_scales, num_tokens,
                                                                       num_slots, num_heads, head_dim);
      break;
    case KVB_F32:
      fp8_kv_write_kernel<float><<<grid_for(work, 256), 256, 0, st>>>(reinterpret_cast<const float*>(x_new), c,
                                                                      slot_mapping, idx64, head_scales, num_tokens,
                                                                      num_slots, num_heads, head_dim);
      break;
    default: return set_error(KVB_E_DTYPE, "paged_fp8_kv_write: x dtype %d", x_dtype);
  }
  return check_launch("fp8_kv_write_kernel");
}
