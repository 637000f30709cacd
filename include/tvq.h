/*
 * tvq.h -- C ABI of libtvq, the B200 (sm_100a) implementation of
 * TokenVector.Inference's post-training-quantized (PTQ) linear path.
 *
 * The boundary follows the reference's native-call convention
 * (docs/SPEC_FUSED_SDPA_BWD.md:89, docs/SIMD_NOTES.md:8-18 of that
 * repository): plain pointers, int64_t sizes, float scalars, an int status
 * (0 = OK).  The reference turned a non-zero status into an interpreted
 * fallback; this library has no fallback -- callers raise on non-zero.
 *
 * Two families of entry points:
 *  - tvq_*      HOST buffers (the reference's list backing arrays).  The call
 *               stages them to the current CUDA device, runs, copies results
 *               back and synchronises.  Mirrors tv.quantization.* one to one.
 *  - tvq_dev_*  DEVICE buffers, asynchronous on the given cudaStream_t
 *               (NULL = legacy default stream); scales that the GPU produces
 *               (calibration) are passed by device pointer so that chains of
 *               calls need no host round trip.
 * And a session API (tvq_session_*) holding device-resident weights and a
 * captured launch sequence for a GPT-2-shaped stack of QuantizedGemm layers.
 *
 * Semantics of every numeric entry point match the reference bit for bit
 * (int8 tensors, int32 accumulators, fp32 epilogue outputs) except where a
 * comment states a tolerance.  Thread safety: each call is independent; a
 * session handle must not be used from two threads at once.
 */
#ifndef TVQ_H_
#define TVQ_H_

#include <stdint.h>

#if defined(__GNUC__)
#define TVQ_API __attribute__((visibility("default")))
#else
#define TVQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes */
#define TVQ_OK 0
#define TVQ_ERR_INVALID (-1)     /* null pointer, negative size, bad mode          */
#define TVQ_ERR_SIZE (-2)        /* a buffer or scale list is too small (ValueError) */
#define TVQ_ERR_CUDA (-3)        /* CUDA runtime / driver error                     */
#define TVQ_ERR_TIMEOUT (-4)     /* a device-side bounded wait ran out             */
#define TVQ_ERR_UNSUPPORTED (-5) /* no sm_100 device, unaligned or unsupported shape */
#define TVQ_ERR_HANDLE (-6)      /* unknown or destroyed session handle            */

/* ---- activation codes of the GEMM epilogue
 * tv/optimization/kernels.tkv:2-7 numbers its ActivationFunction enum the same
 * way for 0..2; GELU_ERF is the erf form used by tv/training/gpt2_ref.tkv. */
#define TVQ_ACT_NONE 0
#define TVQ_ACT_RELU 1
#define TVQ_ACT_GELU_TANH 2 /* ActivationFunction_GELU, kernels.tkv:22-24        */
#define TVQ_ACT_GELU_ERF 6  /* gelu_erf, tv/training/tensor.tkv:189-190 (fp32 math) */

/* ---- FP8 encoder modes */
#define TVQ_FP8_REF 0 /* reference encoder, tv/quantization/types.tkv:154-191 (quirks kept) */
#define TVQ_FP8_HW 1  /* hardware cvt.rn.satfinite (OCP E4M3), not the reference's          */

/* ---- library / device */
TVQ_API int tvq_version(void);
/* Copies the last error message of the calling thread (NUL-terminated). */
TVQ_API int tvq_last_error(char* buf, int64_t len);
TVQ_API int tvq_device_count(int* n);
/* Reads and clears the device error word of the current device (bounded
 * waits record there); returns TVQ_OK or TVQ_ERR_TIMEOUT. */
TVQ_API int tvq_device_error(void* stream);
/* Failure-detection self test (no reference counterpart: the reference has no
 * device code).  Launches one kernel whose bounded mbarrier wait -- the wait
 * every tensor-core kernel uses -- runs out after limit_us (1 .. 10^6) because
 * nothing arrives, then reads the device error word like any call: returns
 * TVQ_ERR_TIMEOUT with the word cleared and the context still usable. */
TVQ_API int tvq_selftest_wait_timeout(int64_t limit_us, void* stream);

/* ================================================================ host buffers
 * tv/quantization/engine.tkv */

/* calibrate_minmax(data, symmetric), engine.tkv:13-36 -> QuantParams fields. */
TVQ_API int tvq_calibrate_minmax(const float* data, int64_t n, int symmetric, float* scale, int64_t* zero_point,
                         float* min_val, float* max_val);
/* calibrate_minmax over several batches (running min/max), as the caller of
 * engine.tkv:13-36 does for BASELINE config 1's 8 calibration batches. */
TVQ_API int tvq_calibrate_minmax_batches(const float* const* batches, const int64_t* sizes, int64_t n_batches,
                                 int symmetric, float* scale, int64_t* zero_point, float* min_val,
                                 float* max_val);
/* calibrate_kl, engine.tkv:42-122 (TensorRT-style KL over a num_bins histogram
 * of |x|, candidate thresholds every 16 bins from target_bins); symmetric
 * result.  num_bins <= 4096.  max |x| < 1e-8 returns calibrate_minmax(data, 1). */
TVQ_API int tvq_calibrate_kl(const float* data, int64_t n, int64_t num_bins, int64_t target_bins, float* scale,
                             int64_t* zero_point, float* min_val, float* max_val);
/* calibrate_percentile, engine.tkv:125-162: clip at the percentile of |x|
 * (exact rank int(min(n-1, percentile/100 n)) of |x|; inputs without NaN);
 * TVQ_ERR_SIZE (ValueError) for percentile outside (0, 100]. */
TVQ_API int tvq_calibrate_percentile(const float* data, int64_t n, float percentile, int symmetric, float* scale,
                                     int64_t* zero_point, float* min_val, float* max_val);
/* calibrate_mse, engine.tkv:165-197: the threshold am*c/num (c = 1..num, num
 * >= 4) with the least mean squared quantization error; symmetric result. */
TVQ_API int tvq_calibrate_mse(const float* data, int64_t n, int64_t num_candidates, float* scale,
                              int64_t* zero_point, float* min_val, float* max_val);
/* Device form of calibrate_mse that also writes the per-candidate mean squared
 * errors (curve_dev[num_candidates], f64) and the result to out4_dev
 * {scale, zero point, min, max}; *fallback = 1 when max |x| < 1e-8 (then
 * nothing is written: the reference returns calibrate_minmax). */
TVQ_API int tvq_dev_calibrate_mse_curve(const float* x, int64_t n, int64_t num_candidates, double* curve_dev,
                                        float* out4_dev, int* fallback, void* stream);
/* calibrate_per_channel_minmax(data, rows, cols, 1), engine.tkv:202-213: the
 * per-row symmetric scales (fl32(max|W[r,:]|/127), floor 1e-8). */
TVQ_API int tvq_calibrate_per_channel_minmax(const float* data, int64_t len, int64_t rows, int64_t cols,
                                     float* scales, int64_t n_scales);
/* calibrate_per_channel_minmax(data, rows, cols, symmetric), engine.tkv:
 * 202-213, with every QuantParams field per row (one launch): scale, zero
 * point, and the row's own min / max as calibrate_minmax stores them
 * (engine.tkv:13-36; symmetric: -am / am). */
TVQ_API int tvq_calibrate_per_channel_params(const float* data, int64_t len, int64_t rows, int64_t cols,
                                             int symmetric, float* scales, int64_t* zero_points, float* min_vals,
                                             float* max_vals, int64_t n);
/* quantize_int8_symmetric, engine.tkv:216-226 */
TVQ_API int tvq_quantize_int8_symmetric(const float* src, int64_t n, int8_t* dst, int64_t dst_len, float scale);
/* dequantize_int8_symmetric, engine.tkv:229-234 */
TVQ_API int tvq_dequantize_int8_symmetric(const int8_t* src, int64_t n, float* dst, int64_t dst_len, float scale);
/* quantize_int8_per_channel, engine.tkv:237-250 */
TVQ_API int tvq_quantize_int8_per_channel(const float* src, int64_t src_len, int8_t* dst, int64_t dst_len, int64_t rows,
                                  int64_t cols, const float* scales, int64_t n_scales);
/* dequantize_int8_per_channel, engine.tkv:253-262 */
TVQ_API int tvq_dequantize_int8_per_channel(const int8_t* src, int64_t src_len, float* dst, int64_t dst_len,
                                    int64_t rows, int64_t cols, const float* scales, int64_t n_scales);
/* quantize_dynamic_int8_rowwise, engine.tkv:266-285 */
TVQ_API int tvq_quantize_dynamic_int8_rowwise(const float* src, int64_t src_len, int8_t* dst, int64_t dst_len,
                                      int64_t rows, int64_t cols, float* scales_out, int64_t n_scales);

/* ================================================================ host buffers
 * tv/quantization/matmul.tkv -- A int8 [m,k] row-major, W int8 [n,k]
 * row-major ("TN"), bias f32 [n] (n_bias == 0: none), Y f32 [m,n]. */

/* matmul_int8_per_channel, matmul.tkv:17-29 (+ optional activation, which the
 * reference's QuantizedGemm node ignores: pass TVQ_ACT_NONE for parity). */
TVQ_API int tvq_matmul_int8_per_channel(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y,
                                int64_t m, int64_t n, int64_t k, float scale_a, const float* scales_w,
                                int64_t n_scales, int act);
/* matmul_int8_symmetric, matmul.tkv:4-15 */
TVQ_API int tvq_matmul_int8_symmetric(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y,
                              int64_t m, int64_t n, int64_t k, float scale_a, float scale_w, int act);
/* Raw int32 accumulators acc[m,n] = sum_k A[m,k]*W[n,k] (_dot_int8,
 * matmul.tkv:116-127), for bit-exact verification. */
TVQ_API int tvq_gemm_i8_acc(const int8_t* A, const int8_t* W, int32_t* acc, int64_t m, int64_t n, int64_t k);

/* quantize_fp8_e4m3, matmul.tkv:60-66 (byte form; mode TVQ_FP8_REF|HW). */
TVQ_API int tvq_quantize_fp8_e4m3(const float* src, int64_t n, uint8_t* dst, int64_t dst_len, int mode);
/* Scaled FP8 quantize: dst = encode(fl32(src * (1/scale))),
 * scales per row (per_row = 1, n_scales >= rows) or one per tensor. */
TVQ_API int tvq_quantize_fp8_e4m3_scaled(const float* src, int64_t rows, int64_t cols, uint8_t* dst,
                                 const float* scales, int64_t n_scales, int per_row, int mode);
/* dequantize_fp8_e4m3, matmul.tkv:68-73 (reference decoder, byte form). */
TVQ_API int tvq_dequantize_fp8_e4m3(const uint8_t* src, int64_t n, float* dst, int64_t dst_len);
/* matmul_fp8_e4m3, matmul.tkv:46-58, on E4M3 bytes, with the optional
 * scale_a * scales_w[n] factor of config 3 (scales_w NULL and scale_a 1 =
 * the reference's unscaled form).  fp32 tensor-core accumulation: results
 * agree with the reference's exact f64 sum within the documented FP8
 * tolerance; subnormal E4M3 operands use the OCP value (the reference
 * decoder halves them, types.tkv:221). */
TVQ_API int tvq_matmul_fp8_e4m3(const uint8_t* A, const uint8_t* W, const float* bias, int64_t n_bias, float* Y,
                        int64_t m, int64_t n, int64_t k, float scale_a, const float* scales_w, int act);

/* matmul_int8_asymmetric, matmul.tkv:31-44: acc = sum_k (a - zp_a)(w - zp_w)
 * exact, y = fl32(fl64(acc * fl64(scale_a*scale_w)) + bias[n]).  On the
 * tensor cores: the int32 dot product, then in the epilogue acc = dot -
 * zp_w sum_k a - zp_a sum_k w + k zp_a zp_w in binary64 (every term an exact
 * integer).  |zp_a|, |zp_w| <= 2^17 (TVQ_ERR_UNSUPPORTED beyond). */
TVQ_API int tvq_matmul_int8_asymmetric(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y,
                               int64_t m, int64_t n, int64_t k, float scale_a, int64_t zp_a, float scale_w,
                               int64_t zp_w);

/* matmul_fp16, matmul.tkv:79-96: A [m,k] and W [n,k] fp16 bit patterns,
 * y = fl32(sum_k a w + bias[n]).  kind::f16 tensor cores with fp32
 * accumulation, partial sums of 192 k promoted to registers: within
 * (k/16 + 2) 2^-23 sum_k |a w| of the reference's binary64 sum.  An fp16 NaN
 * operand stays NaN here; the reference's decoder reads it as +-Inf
 * (f32_bits_to_f64 maps exponent 255 to 2^129). */
TVQ_API int tvq_matmul_fp16(const uint16_t* A, const uint16_t* W, const float* bias, int64_t n_bias, float* Y,
                    int64_t m, int64_t n, int64_t k);
/* quantize_fp16, matmul.tkv:106-114: the reference's encoder
 * (native_f16_encode, types.tkv:95-127; its departures from IEEE rounding
 * are kept: see tvq_f16.h) of n floats, dst_len >= n. */
TVQ_API int tvq_quantize_fp16(const float* src, int64_t n, uint16_t* dst, int64_t dst_len);

/* ---- list[i32] compatibility forms: the reference stores int8 values in
 * list[i32] (engine.tkv:216, session.tkv:158-170) and FP8 bytes as
 * byte - 128 (matmul.tkv:65, :76).  These convert at the boundary. */
TVQ_API int tvq_quantize_int8_symmetric_i32(const float* src, int64_t n, int32_t* dst, int64_t dst_len, float scale);
TVQ_API int tvq_matmul_int8_per_channel_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias,
                                    float* Y, int64_t m, int64_t n, int64_t k, float scale_a,
                                    const float* scales_w, int64_t n_scales);
TVQ_API int tvq_quantize_fp8_e4m3_i32(const float* src, int64_t n, int32_t* dst, int64_t dst_len);
TVQ_API int tvq_matmul_fp8_e4m3_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias, float* Y,
                            int64_t m, int64_t n, int64_t k);
TVQ_API int tvq_matmul_int8_asymmetric_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias,
                                   float* Y, int64_t m, int64_t n, int64_t k, float scale_a, int64_t zp_a,
                                   float scale_w, int64_t zp_w);
/* FP16 as the reference stores it: two list entries per element, low byte
 * first (A [2 m k], W [2 n k]; each entry & 255, matmul.tkv:84-87) */
TVQ_API int tvq_matmul_fp16_i32(const int32_t* A, const int32_t* W, const float* bias, int64_t n_bias, float* Y,
                        int64_t m, int64_t n, int64_t k);
/* dst [2 n]: the two bytes of each fp16 as signed values (_to_sbyte, matmul.tkv:98-114) */
TVQ_API int tvq_quantize_fp16_i32(const float* src, int64_t n, int32_t* dst, int64_t dst_len);

/* ================================================================ device buffers
 * Asynchronous on `stream`.  minmax_dev is float[2] = {min, max} in an
 * order-preserving encoding; reset it with tvq_dev_minmax_reset before the
 * first batch, accumulate any number of batches, then finalize. */
TVQ_API int tvq_dev_minmax_reset(uint32_t* minmax_dev, void* stream);
TVQ_API int tvq_dev_minmax_accumulate(const float* x, int64_t n, uint32_t* minmax_dev, float* first_dev, void* stream);
/* Writes QuantParams {scale, zero_point(as float), min, max} to params_dev[4]. */
TVQ_API int tvq_dev_minmax_finalize(const uint32_t* minmax_dev, const float* first_dev, int symmetric, float* params_dev,
                            void* stream);
/* Per-tensor quantize with a device scale (scale_dev[0]). */
TVQ_API int tvq_dev_quantize_int8(const float* x, int8_t* q, int64_t n, const float* scale_dev, void* stream);
/* quantize_fp16 on device buffers (fp16 bit patterns out). */
TVQ_API int tvq_dev_quantize_fp16(const float* x, uint16_t* q, int64_t n, void* stream);
/* matmul_fp16 on device buffers: k a multiple of 8, A and W 16-byte aligned;
 * bias [n] or NULL. */
TVQ_API int tvq_dev_matmul_fp16(const uint16_t* A, const uint16_t* W, const float* bias, float* Y, int64_t m, int64_t n,
                        int64_t k, void* stream);
/* matmul_int8_asymmetric on device buffers: k a multiple of 16, A and W
 * 16-byte aligned; scale_a_dev / scale_w_dev device float[1].  Allocates its
 * (m + n)-int row-sum scratch stream-ordered (cudaMallocAsync). */
TVQ_API int tvq_dev_matmul_int8_asymmetric(const int8_t* A, const int8_t* W, const float* bias, float* Y, int64_t m,
                                   int64_t n, int64_t k, const float* scale_a_dev, int64_t zp_a,
                                   const float* scale_w_dev, int64_t zp_w, void* stream);
/* Per-channel weight calibrate + quantize, fused: scales_dev[r] and q[r,:]. */
TVQ_API int tvq_dev_calibrate_quantize_per_channel(const float* w, int8_t* q, float* scales_dev, int64_t rows,
                                           int64_t cols, void* stream);
TVQ_API int tvq_dev_quantize_int8_per_channel(const float* w, int8_t* q, const float* scales_dev, int64_t rows,
                                      int64_t cols, void* stream);
TVQ_API int tvq_dev_quantize_dynamic_rowwise(const float* x, int8_t* q, float* scales_dev, int64_t rows, int64_t cols,
                                     void* stream);
TVQ_API int tvq_dev_quantize_fp8(const float* x, uint8_t* q, int64_t rows, int64_t cols, const float* scales_dev,
                         int scale_mode /*0 none, 1 per tensor, 2 per row*/, int mode, void* stream);
TVQ_API int tvq_dev_dequantize_fp8(const uint8_t* q, float* y, int64_t n, void* stream);

/* Quantized GEMM on tcgen05 tensor cores.  kind 0 = INT8 (A,W int8), 1 = FP8
 * E4M3 (A,W bytes).  scale_a_dev: device float[1]; scales_w_dev: device
 * float[n] (per_channel = 1) or float[1].  Epilogue, in order:
 *   y = fl32(acc * scale_a * scale_w[n] + bias[n])      (f64, the reference's)
 *   y = act(y)                                          (TVQ_ACT_*)
 *   y = fl32(y + residual[m,n])   if residual != NULL
 *   Y[m,n] = y                    if Y != NULL          (f32, ldy = n)
 *   Yq[m,n] = clamp(round(y * (1/scale_out)), +-127)   if Yq != NULL
 *   atomicMax(|y|) into amax_dev  if amax_dev != NULL   (calibration)
 * k must be a multiple of 16 and pointers 16-byte aligned. */
TVQ_API int tvq_dev_gemm(int kind, const void* A, const void* W, const float* bias, const float* residual, float* Y,
                 int8_t* Yq, int64_t m, int64_t n, int64_t k, const float* scale_a_dev,
                 const float* scales_w_dev, int per_channel, int act, const float* scale_out_dev,
                 uint32_t* amax_dev, void* stream);

/* fp32 GEMM Y[m,n] = A[m,k] W[n,k]^T on the tcgen05 tensor cores with split
 * precision: each operand is given as high + low parts (tvq_dev_split_tf32),
 * and Y accumulates xh*wh + xh*wl + xl*wh in f32 (relative error about 2^-21
 * per product, the size of an fp32 GEMM's own accumulation error).  Used for
 * the tied LM head (gpt2_ref.tkv:603-610).  k*4 must be a multiple of 16 and
 * all pointers 16-byte aligned. */
TVQ_API int tvq_dev_gemm_f32x3(const float* A_hi, const float* A_lo, const float* W_hi, const float* W_lo, float* Y,
                               int64_t m, int64_t n, int64_t k, void* stream);
/* x ~ hi + lo with both parts on the TF32 grid: hi = tf32(x), lo =
 * tf32(x - hi), |x - hi - lo| <= 2^-22 |x|. */
TVQ_API int tvq_dev_split_tf32(const float* x, float* hi, float* lo, int64_t n, void* stream);

/* fp32 GEMM Y[m,n] = A[m,k] W[n,k]^T on the FP16 tensor cores (kind::f16):
 * each row of A and of W is split by tvq_dev_split_f16_rows into fp16
 * high + low parts under a power-of-two row scale, Y accumulates xh*wh +
 * xh*wl + xl*wh in f32 and the epilogue multiplies by A_rscale[m] *
 * W_rscale[n] (exact).  Twice the K per instruction and half the operand
 * bytes of tvq_dev_gemm_f32x3 at the same accuracy.  k must be a multiple
 * of 8 and all pointers 16-byte aligned.  Used for the tied LM head
 * (gpt2_ref.tkv:603-610). */
TVQ_API int tvq_dev_gemm_f16x3(const void* A_hi, const void* A_lo, const float* A_rscale, const void* W_hi,
                               const void* W_lo, const float* W_rscale, float* Y, int64_t m, int64_t n, int64_t k,
                               void* stream);
/* Row-scaled fp16 split of x [rows, k] (f32): per row the power of two s
 * with max|x| * s in [2^14, 2^15), hi = fp16(x*s), lo = fp16(x*s - hi)
 * (fp16 bit patterns, [rows, k] each), rscale[row] = 1/s (1 for k = 0).
 * |x*s - hi - lo| <= max(2^-22 |x*s|, 2^-25).  A row with Inf or NaN gets
 * s = 1. */
TVQ_API int tvq_dev_split_f16_rows(const float* x, void* hi, void* lo, float* rscale, int64_t rows, int64_t k,
                                   void* stream);

/* ================================================================ fp32 glue, device buffers
 * gpt2_layernorm, tv/training/gpt2_ref.tkv:50-78 (f64 statistics): y (f32)
 * and/or q = int8 with the static scale qscale_dev[0]; amax_dev records
 * max|y| (calibration). */
TVQ_API int tvq_dev_layernorm(const float* x, const float* gamma, const float* beta, float* y, int8_t* q,
                              const float* qscale_dev, uint32_t* amax_dev, int64_t rows, int64_t d, double eps,
                              void* stream);
/* Causal multi-head attention of gpt2_attention (gpt2_ref.tkv:360-395, no
 * projection) over packed sequences seg[0..n_seg] (host offsets): qkv f32
 * [T, 3d] rows [Q|K|V]; out f32 [T, d] and/or outq int8 (scale qscale_dev).
 * tiles_dev: device scratch of tiles_cap entries of 4 x int32, 16-byte
 * aligned; a call needs one entry per 64-row query tile, or with head dim 64
 * (tensor-core kernel, FP16 hi/lo products) two per 128-row tile -- at most
 * ceil(len / 64) + 1 entries per sequence either way.  fp32-accurate: within
 * 1e-4 relative / 2e-6 absolute of the f64 oracle. */
TVQ_API int tvq_dev_attention(const float* qkv, const int64_t* seg, int64_t n_seg, int64_t d, int64_t n_heads,
                              int32_t* tiles_dev, int64_t tiles_cap, float* out, int8_t* outq,
                              const float* qscale_dev, uint32_t* amax_dev, void* stream);
/* tvq_dev_attention for callers that cannot allocate device memory when they
 * call (a host runtime whose device memory all belongs to its own pool, a
 * serving loop that must not allocate): no counterpart in the reference.  The
 * query-tile scratch is a fixed 512 KiB device array inside the library
 * (every GPU that loads it holds it until exit), so at most 32768 tiles of
 * 64 tokens per sequence fit in one call; larger calls fail with
 * TVQ_ERR_SIZE.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) once.  All calls share the array: calls
 * that overlap on the GPU race on it.  No
 * cudaMalloc or cudaFree is called.  The tile list is copied into the array
 * from host memory, so the call blocks the calling thread until the work
 * already queued on `stream` has finished.  It always runs the fp32 SIMT
 * kernel (head dims 16, 32, 48, 64): bit-identical to tvq_dev_attention at
 * head dims 16-48, within the same 1e-4 / 2e-6 tolerance of it at head dim
 * 64, where tvq_dev_attention takes the tensor-core kernel. */
TVQ_API int tvq_dev_attention_noalloc(const float* qkv, const int64_t* seg, int64_t n_seg, int64_t d,
                                      int64_t n_heads, float* out, int8_t* outq, const float* qscale_dev,
                                      uint32_t* amax_dev, void* stream);

/* ================================================================ ONNX QDQ operators
 * The quantized-operator family of the reference runtime's fp32 graph
 * executor (tv/runtime/session.tkv), reached from ExecutionNode.execute
 * (:642-675).  Quantize / dequantize take the tensor split at its axis into
 * (outer, dim, inner) (session.tkv:1926-1940, qlinear_axis); n_scales == 1 is
 * per tensor, n_scales == dim per channel (else TVQ_ERR_SIZE).  B of the two
 * matmuls is row-major [K, N] as in the reference.  Host-buffer forms first,
 * then device-buffer forms (stream-ordered). */
/* _exec_quantize_linear, session.tkv:1896-1953: y = clamp(int(round(x / s))
 * + zero_point, -128, 127), s = max(scale, 1e-12). */
TVQ_API int tvq_quantize_linear(const float* x, int8_t* y, int64_t outer, int64_t dim, int64_t inner,
                                const float* scales, int64_t n_scales, int64_t zero_point);
/* _exec_dequantize_linear, session.tkv:1955-1990: y = (x - zero_point) * scale. */
TVQ_API int tvq_dequantize_linear(const int8_t* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                                  const float* scales, int64_t n_scales, int64_t zero_point);
/* _exec_matmul_integer, session.tkv:2789-2851: y int32 [m, n] = a [m, k] x b [k, n]. */
TVQ_API int tvq_matmul_integer(const int8_t* a, const int8_t* b, int32_t* y, int64_t m, int64_t k, int64_t n);
/* _exec_qlinear_matmul, session.tkv:1992-2071: y = clamp(int(round(sum (a - zp_a)(b - zp_b)
 * * scale_a * scale_b / scale_y)) + zp_y, -128, 127) (scale_y == 0 -> 1). */
TVQ_API int tvq_qlinear_matmul(const int8_t* a, float scale_a, int64_t zp_a, const int8_t* b, float scale_b,
                               int64_t zp_b, float scale_y, int64_t zp_y, int8_t* y, int64_t m, int64_t k, int64_t n);
/* _exec_dyn_quant, session.tkv:2853-2905: uint8 asymmetric over the tensor, stored as
 * int8 (q - 128); y_scale = (max(mx,0) - min(mn,0)) / 255, y_zero_point in [0, 255]. */
TVQ_API int tvq_dynamic_quantize_linear(const float* x, int64_t n, int8_t* y, float* y_scale, float* y_zero_point);
TVQ_API int tvq_dev_quantize_linear(const float* x, int8_t* y, int64_t outer, int64_t dim, int64_t inner,
                                    const float* scales_dev, int64_t n_scales, int64_t zero_point, void* stream);
TVQ_API int tvq_dev_dequantize_linear(const int8_t* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                                      const float* scales_dev, int64_t n_scales, int64_t zero_point, void* stream);
TVQ_API int tvq_dev_matmul_integer(const int8_t* a, const int8_t* b, int32_t* y, int64_t m, int64_t k, int64_t n,
                                   void* stream);
TVQ_API int tvq_dev_qlinear_matmul(const int8_t* a, float scale_a, int64_t zp_a, const int8_t* b, float scale_b,
                                   int64_t zp_b, float scale_y, int64_t zp_y, int8_t* y, int64_t m, int64_t k,
                                   int64_t n, void* stream);
TVQ_API int tvq_dev_dynamic_quantize_linear(const float* x, int64_t n, int8_t* y, float* y_scale_dev,
                                            float* y_zp_dev, void* stream);

/* ================================================================ group-wise INT4 (int4.tkv)
 * Weights [rows, cols] -> packed bytes [rows, cols/2] (two nibbles per byte,
 * low nibble first; the reference's list[i32] holds the same byte values),
 * scales f32 [rows, cols/group_size], and for the AWQ-style asymmetric form
 * zero points int64 [rows, cols/group_size] (zps NULL = symmetric).  cols
 * must be an even multiple of group_size (else TVQ_ERR_SIZE, the reference's
 * ValueError).  Bit-exact with the reference's f64 arithmetic.
 *   quantize_int4_grouped        int4.tkv:27-48 (scales :18-29)
 *   dequantize_int4_grouped      int4.tkv:51-64
 *   quantize_int4_grouped_asym   int4.tkv:68-150
 *   dequantize_int4_grouped_asym int4.tkv:153-164
 *   permute_cols / inv_permute_cols (inverse = 1)  int4.tkv:169-184
 *   matmul_int4_grouped (perm NULL) / matmul_int4_grouped_ordered (act
 *     order, A columns gathered by perm)  int4.tkv:187-239: Y[m,n] = sum_k
 *     A[m, perm[k]] * (nib - 8) * scale[n, k/gs] + bias[n], f32 A [m,k],
 *     packed W [n, k/2]; on the tensor cores with fp32 accuracy (A split
 *     into fp16 hi/lo under power-of-two row scales, the weights' integers
 *     exact in fp16, each group's partial sum times its scale in registers).
 * Device forms take device pointers and a stream; host forms are synchronous. */
TVQ_API int tvq_dev_quantize_int4_grouped(const float* src, int64_t rows, int64_t cols, int64_t group_size,
                                          uint8_t* packed, float* scales, int64_t* zps, void* stream);
TVQ_API int tvq_dev_dequantize_int4_grouped(const uint8_t* packed, float* dst, int64_t rows, int64_t cols,
                                            int64_t group_size, const float* scales, const int64_t* zps,
                                            void* stream);
TVQ_API int tvq_dev_permute_cols(const float* src, float* dst, int64_t rows, int64_t cols, const int64_t* perm,
                                 int inverse, void* stream);
TVQ_API int tvq_dev_matmul_int4_grouped(const float* A, const uint8_t* packed_w, const float* bias, float* Y,
                                        int64_t m, int64_t n, int64_t k, int64_t group_size, const float* scales_w,
                                        const int64_t* perm, void* stream);
TVQ_API int tvq_quantize_int4_grouped(const float* src, int64_t rows, int64_t cols, int64_t group_size,
                                      uint8_t* packed_out, float* scales_out, int64_t* zps_out);
TVQ_API int tvq_dequantize_int4_grouped(const uint8_t* packed, float* dst, int64_t rows, int64_t cols,
                                        int64_t group_size, const float* scales, int64_t n_scales,
                                        const int64_t* zps);
TVQ_API int tvq_permute_cols(const float* src, float* dst, int64_t rows, int64_t cols, const int64_t* perm,
                             int64_t n_perm, int inverse);
TVQ_API int tvq_matmul_int4_grouped(const float* A, const uint8_t* packed_w, const float* bias, int64_t n_bias,
                                    float* Y, int64_t m, int64_t n, int64_t k, int64_t group_size,
                                    const float* scales_w, int64_t n_scales, const int64_t* perm);

/* ================================================================ sessions
 * Device-resident GPT-2-shaped INT8 PTQ stack: embeddings, n_layers blocks of
 * (ln_1, c_attn, attention, c_proj, ln_2, c_fc, GELU-erf, mlp c_proj) with the
 * four linears as QuantizedGemm (session.tkv:678-697), ln_f and the tied fp32
 * LM head (gpt2_ref.tkv:575-610).  Replaces InferenceSession construction +
 * run (session.tkv:3376-3436) for graphs of this shape.  One handle per GPU.
 * vocab 0 makes a layer stack without embeddings, ln_f or LM head: it runs
 * through tvq_session_run_layers only. */
TVQ_API int tvq_session_create(int device, int64_t vocab, int64_t d_model, int64_t n_heads, int64_t n_layers,
                               int64_t d_ffn, int64_t max_pos, double ln_eps, int64_t max_tokens, int64_t* handle);
TVQ_API int tvq_session_destroy(int64_t handle);
/* wte f32 [vocab, d] (also the LM head), wpe f32 [max_pos, d], host. */
TVQ_API int tvq_session_set_embeddings(int64_t handle, const float* wte, const float* wpe);
/* layer -1 = ln_f; which 0 = ln_1, 1 = ln_2. */
TVQ_API int tvq_session_set_layernorm(int64_t handle, int64_t layer, int64_t which, const float* gamma,
                                      const float* beta);
/* which 0 c_attn [3d x d], 1 attn c_proj [d x d], 2 c_fc [ffn x d], 3 mlp
 * c_proj [d x ffn]; f32 weights quantized on the GPU per output channel
 * (calibrate_per_channel_minmax + quantize_int8_per_channel, engine.tkv:202-250).
 * layout 0 = [k, n] (HF Conv1D, gpt2_ref.tkv:91-117), 1 = [n, k]. */
TVQ_API int tvq_session_set_linear_f32(int64_t handle, int64_t layer, int64_t which, const float* w,
                                       const float* bias, int layout);
/* Pre-quantized weights [n, k] with per-channel scales (the QuantizedGemm
 * node's initializers_int8 + scales_w, session.tkv:3149, 497-505). */
TVQ_API int tvq_session_set_linear_i8(int64_t handle, int64_t layer, int64_t which, const int8_t* w_nk,
                                      const float* scales_w, const float* bias);
TVQ_API int tvq_session_get_linear_i8(int64_t handle, int64_t layer, int64_t which, int8_t* w_nk, float* scales_w);
/* Static activation scales, 4 per layer: ln_1 out, attention context, ln_2
 * out, GELU out (the scale_a of the four QuantizedGemm nodes). */
TVQ_API int tvq_session_set_act_scales(int64_t handle, const float* scales, int64_t n);
TVQ_API int tvq_session_get_act_scales(int64_t handle, float* scales, int64_t n);
/* Batch layout: seg[0..n_seg] packed sequence offsets (seg[0] = 0, total
 * tokens seg[n_seg] <= max_tokens); logits_mode 0 = logits for every token,
 * 1 = for the last token of each sequence. */
TVQ_API int tvq_session_prepare(int64_t handle, const int64_t* seg, int64_t n_seg, int logits_mode);
/* Calibration forward on ids (host or device): records max|x| at the four
 * quantization points of every layer (running max unless reset) and sets
 * the static scales from it. */
TVQ_API int tvq_session_calibrate(int64_t handle, const int64_t* ids, int ids_on_device, int reset);
/* One INT8 forward (CUDA graph) on `stream` (NULL: the session's own).
 * ids NULL = reuse the resident ids.  logits NULL = keep them on the device
 * (see tvq_session_logits).  Host buffers make the call synchronous.  With a
 * host logits buffer, logits_mode 0 and >= 512 tokens, the LM head runs in
 * 256-row chunks after the captured body and each chunk's logits are copied
 * to the host on a second stream while the next chunk computes (same bits
 * as the one-launch LM head). */
TVQ_API int tvq_session_forward(int64_t handle, const int64_t* ids, int ids_on_device, float* logits,
                                int64_t logits_len, int logits_on_device, void* stream);
/* tvq_session_forward with host logits, queued without waiting: the call
 * returns once the work is on `stream` (NULL: the session's own), so calls
 * can be issued back to back and the next forward's body runs while this
 * one's logits cross PCIe (the copy, ~206 MB per 1024-token step of GPT-2
 * 124M, bounds the blocking form).  Before the LM head overwrites a range of
 * the device logits, the stream waits until the previous call's copy of that
 * range is done.  ids: host (pinned for an asynchronous copy) or device;
 * logits: host memory (pinned), left untouched by the caller until
 * tvq_session_wait returns.  No counterpart in the reference: its
 * InferenceSession.run (session.tkv:3403-3436) is synchronous; each call's
 * logits are those of tvq_session_forward on the same ids. */
TVQ_API int tvq_session_forward_async(int64_t handle, const int64_t* ids, int ids_on_device, float* logits,
                                      int64_t logits_len, void* stream);
/* Makes `stream` wait (without blocking the host) until every logits copy
 * queued by the session so far is done. */
TVQ_API int tvq_session_join(int64_t handle, void* stream);
/* tvq_session_join, then blocks until `stream` reaches that point and
 * reports a device error of the queued calls (bad token ids and the like).
 * Call it before reading the host logits and before any other call on the
 * session. */
TVQ_API int tvq_session_wait(int64_t handle, void* stream);
TVQ_API int tvq_session_logits(int64_t handle, float** logits_dev, int64_t* rows, int64_t* cols);
/* The transformer blocks alone (a CUDA graph of their own) on hidden states
 * x f32 [T, d_model] (T = the prepared layout's tokens; host or device; NULL
 * = the resident hidden states, tvq_session_hidden), written to y (NULL =
 * keep them on the device).  dynamic 0 uses the static activation scales;
 * dynamic 1 calibrates every quantization point on this call's activations
 * (calibrate_minmax, engine.tkv:13-36, then quantize_int8_symmetric, per
 * layer on the GPU) and leaves those scales as the static ones.  Host
 * buffers make the call synchronous. */
TVQ_API int tvq_session_run_layers(int64_t handle, const float* x, int x_on_device, float* y, int y_on_device,
                                   int dynamic, void* stream);
/* Device pointer of the resident hidden states [max_tokens, d_model]. */
TVQ_API int tvq_session_hidden(int64_t handle, float** x_dev);
/* Kernel launches of the last tvq_session_forward or tvq_session_run_layers
 * for the prepared layout (kernel nodes of its captured CUDA graph, plus the
 * LM-head chunk launches of the host-logits path; memset and profiling event
 * nodes excluded); needs one to have run since the last prepare / profiling
 * change. */
TVQ_API int tvq_session_launches(int64_t handle, int64_t* kernels);
TVQ_API int tvq_session_sync(int64_t handle);
/* Profiling: with enable = 1 the captured forward records a CUDA event after
 * every stage; tvq_session_stage_times then returns the last forward's time
 * per stage class in ms: [0] embedding, [1] layernorms, [2] c_attn GEMMs,
 * [3] attention, [4] attn c_proj GEMMs, [5] c_fc GEMMs, [6] mlp c_proj GEMMs,
 * [7] LM head, [8] calibrate-then-quantize passes (calibrating / dynamic
 * runs).  n >= 9. */
TVQ_API int tvq_session_set_profiling(int64_t handle, int enable);
TVQ_API int tvq_session_stage_times(int64_t handle, float* ms, int64_t n);

#ifdef __cplusplus
}
#endif

#endif /* TVQ_H_ */
