/*
 * kvb.h -- C ABI of libkvb.so, the B200 (sm_100a) kernels of the quantised
 * decoder-layer hot path of KernelVerse.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are raw DEVICE pointers to contiguous row-major
 *     buffers; sizes are element counts.  No torch types cross this boundary.
 *   - The caller owns all memory (inputs, outputs and any workspace); entry
 *     points never allocate and never synchronise the host.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream); all work is
 *     stream-ordered on it.
 *   - The return value is KVB_OK (0) or a positive KVB_E_* status; the message
 *     for the calling thread's last failure is kvb_last_error().
 *   - Every reference interface an entry point replaces is cited as
 *     path:line inside the KernelVerse tree.
 */
#ifndef KVB_H_
#define KVB_H_

#include <stddef.h>
#include <stdint.h>

#if defined(KVB_BUILD) && defined(__GNUC__)
#define KVB_API __attribute__((visibility("default")))
#else
#define KVB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define KVB_OK 0
#define KVB_E_ARG 1        /* null pointer / bad enum / negative size */
#define KVB_E_SHAPE 2      /* shape outside what the kernel supports */
#define KVB_E_ALIGN 3      /* pointer or stride alignment violated */
#define KVB_E_DTYPE 4      /* unsupported dtype combination */
#define KVB_E_LAUNCH 5     /* CUDA launch / driver error */
#define KVB_E_TIMEOUT 6    /* a bounded device-side wait gave up */
#define KVB_E_WORKSPACE 7  /* workspace missing or too small */
#define KVB_E_DEVICE 8     /* device is not sm_100 */

/* element types */
#define KVB_F32 0
#define KVB_F16 1
#define KVB_BF16 2
#define KVB_I8 3
#define KVB_U8 4
#define KVB_I32 5
#define KVB_I64 6
#define KVB_E4M3 7         /* float8_e4m3fn codes (OCP FP8 E4M3, no inf, max 448) */

/* Message for the last non-zero status returned on this host thread. */
KVB_API const char* kvb_last_error(void);
/* ABI version: bumped on any signature change. */
KVB_API int kvb_abi_version(void);

/*
 * Diagnostics (no reference counterpart).  kvb_device_status synchronises the
 * current device and returns the OR of the library's device status words:
 * bit 0 = a bounded device-side wait gave up (its kernel drained and exited
 * early; outputs of that launch are invalid).  reset != 0 clears the words.
 * Returns 0x80000000 if the device itself reports an error.
 */
KVB_API unsigned int kvb_device_status(int reset);
/* out[i] = a[i] / b[i] through the kernels' FMA-corrected division (test hook). */
KVB_API int kvb_selftest_div_rn(const float* a, const float* b, float* out, int64_t n, void* stream);

/* ---------------------------------------------------------------- quantisation */

/* Bytes of workspace kvb_dynamic_scaled_int8_quant needs (a 256-byte-aligned block). */
KVB_API size_t kvb_dynamic_scaled_int8_quant_workspace_size(void);

/*
 * Per-tensor dynamic int8 quantisation.
 * Replaces operators/quantization/dynamic_scaled_int8_quant/dynamic_scaled_int8_quant.py:21-26
 * (constants helpers.py:7-8):
 *   scale = max(float32(dtype(amax|x| / 127)), 1/(448*512));
 *   q = round_half_even(clamp(x / scale, -127, 127)); azp = 0.
 * x: `numel` elements of x_dtype (KVB_F32/F16/BF16).  q: numel int8.  scale: 1 float.
 * azp: 1 int32 (may be NULL).  workspace: >= kvb_dynamic_scaled_int8_quant_workspace_size()
 * bytes of device memory (the running amax); it is re-initialised on every call.
 * Two kernels are launched (amax, then quantise) after a 4-byte memset.
 */
KVB_API int kvb_dynamic_scaled_int8_quant(const void* x, int x_dtype, int64_t numel,
                                  int8_t* q, float* scale, int32_t* azp,
                                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Per-token, per-group dynamic int8 quantisation.
 * Replaces operators/quantization/per_token_group_quant_int8/per_token_group_quant_int8.py:23-32:
 *   scales[t, g] = max(amax|x[t, g*G:(g+1)*G]| / 127, eps)   (float32)
 *   q = clamp(round_half_even(x / scales), -127, 127)
 * x: [tokens, hidden] of x_dtype; hidden % group_size == 0.  q: [tokens, hidden] int8;
 * scales: [tokens, hidden / group_size] float32.  group_size == hidden gives per-token
 * quantisation (the BASELINE first config).
 */
KVB_API int kvb_per_token_group_quant_int8(const void* x, int x_dtype, int64_t tokens, int64_t hidden,
                                   int64_t group_size, float eps, int8_t* q, float* scales,
                                   void* stream);

/* ---------------------------------------------------------------- residual add + RMSNorm */

/*
 * out = dtype((s * rsqrt(mean(s^2) + eps)) * w), s = x + residual, all in float32.
 * Replaces operators/normalization/add_rmsnorm/add_rmsnorm.py:24-35 (correctness
 * compute mode, :17-22).  x, residual, out: [rows, hidden] of `dtype`; weight: [hidden].
 */
KVB_API int kvb_add_rmsnorm(const void* x, const void* residual, const void* weight, int dtype,
                    int64_t rows, int64_t hidden, float eps, void* out, void* stream);

/*
 * Fused residual add + RMSNorm + dynamic per-row quantisation (one HBM pass).
 * No single reference operator: composes add_rmsnorm.py:24-35 with the per-row
 * quantisation of the BASELINE second config.
 *   residual_out = dtype(x + residual)                     (may alias `residual`)
 *   y = (s * rsqrt(mean(s^2) + eps)) * w                   (float32)
 *   scales[r] = max(amax|y_r| / Q, 1/(448*512)),  Q = 448 (KVB_E4M3) or 127 (KVB_I8)
 *   codes = e4m3fn(clamp(y / scale, +-448))  or  clamp(round_half_even(y / scale), +-127)
 * residual_out may be NULL (not written).  codes: [rows, hidden] bytes; scales: [rows].
 */
KVB_API int kvb_add_rmsnorm_quant(const void* x, const void* residual, const void* weight, int dtype,
                          int64_t rows, int64_t hidden, float eps, void* residual_out,
                          void* codes, int code_dtype, float* scales, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* KVB_H_ */
