// tvq_kernels.h -- internal launcher declarations of libtvq (not part of the
// C ABI; the exported surface is include/tvq.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace tvq {

// tvq_quant.cu
int launch_minmax_reset(uint32_t* mm, cudaStream_t st);
int launch_minmax_accumulate(const float* x, int64_t n, uint32_t* mm, float* first, cudaStream_t st);
int launch_minmax_finalize(const uint32_t* mm, const float* first, int symmetric, float* params, cudaStream_t st);
int launch_quantize_i8(const float* x, int8_t* q, int64_t n, const float* scale_dev, cudaStream_t st);
// Calibrate-then-quantize: scale = fl32(max(*amax, 1e-8) / 127) (stored to
// *scale_out), then quantize_int8_symmetric with it; one launch.
int launch_quantize_i8_amax(const float* x, int8_t* q, int64_t n, const uint32_t* amax, float* scale_out,
                            cudaStream_t st);
int launch_dequantize_i8(const int8_t* q, float* y, int64_t rows, int64_t cols, const float* scales_dev,
                         int per_row, cudaStream_t st);
// calibrate_per_channel_minmax with all four QuantParams fields per row
// (scale, zero point, min, max), symmetric or asymmetric.
int launch_rowwise_params(const float* x, int64_t rows, int64_t cols, int symmetric, float* scale, int64_t* zp,
                          float* mn, float* mx, cudaStream_t st);
// mode 0: per-channel calibrate+quantize, 1: per-channel quantize with given
// scales, 2: dynamic row-wise
int launch_rowwise(int mode, const float* x, int8_t* q, float* scales, int64_t rows, int64_t cols,
                   cudaStream_t st);
int launch_fp8_encode(const float* x, uint8_t* q, int64_t rows, int64_t cols, const float* scales, int scale_mode,
                      int hw, cudaStream_t st);
int launch_fp8_decode(const uint8_t* q, float* y, int64_t n, cudaStream_t st);
int launch_widen(const void* src, int32_t* dst, int64_t n, int is_unsigned, int32_t off, cudaStream_t st);
int launch_narrow(const int32_t* src, void* dst, int64_t n, int32_t off, cudaStream_t st);
float e4m3_decode_host(uint32_t v);
uint8_t e4m3_encode_host(float x);

// tvq_gemm.cu
// GEMM_W4: fp32 activations (fp16 hi / lo under row scales, A / A2,
// scale_a [m]) times group-wise INT4 weights given as their integer values
// nib - 8 in fp16 (W [n, k]), scales_w [n, k / group_size]; Y = sum over
// groups of scale * partial, then * scale_a[m] + bias[n].
enum GemmKind { GEMM_I8 = 0, GEMM_F8 = 1, GEMM_TF32X3 = 2, GEMM_F16X3 = 3, GEMM_W4 = 4 };

struct GemmArgs {
    int kind = GEMM_I8;
    const void* A = nullptr;          // [m,k] 8-bit, row-major
    const void* W = nullptr;          // [n,k] 8-bit, row-major
    // GEMM_TF32X3 / GEMM_F16X3: low parts of A and W (A, W hold the high
    // parts: f32 on the TF32 grid / fp16).  GEMM_F16X3 also reads scale_a [m]
    // and scales_w [n]: the rows' power-of-two scales (launch_split_f16_rows).
    const void* A2 = nullptr;
    const void* W2 = nullptr;
    const float* bias = nullptr;      // [n] or null
    const float* residual = nullptr;  // [m,n] or null
    float* Y = nullptr;               // [m,n] or null
    int8_t* Yq = nullptr;             // [m,n] or null
    int32_t* acc_out = nullptr;       // [m,n] raw accumulators or null (verification)
    int64_t m = 0, n = 0, k = 0;
    const float* scale_a = nullptr;   // device [1]
    const float* scales_w = nullptr;  // device [n] or [1]
    int per_channel = 1;
    int act = 0;
    const float* scale_out = nullptr; // device [1], needed with Yq
    uint32_t* amax = nullptr;         // device [1] or null
    int force_bn = 0;                 // 0 = heuristic, else 64/128/256
    int group_size = 0;               // GEMM_W4: k elements per weight scale (a multiple of 16)
    // c_attn only: also write Q, K [m, kvd] and V^T [kvd, vt_pitch] of qkv as
    // fp16 hi / lo under per-head power-of-two scales (the tensor-core
    // attention's operands); kv_bound [6 kvd / 64] holds the per-head bounds
    // of launch_kv_head_bound, kv_exp [3 kvd / 64] receives the exponents
    void *qh = nullptr, *ql = nullptr, *kh = nullptr, *kl = nullptr, *vth = nullptr, *vtl = nullptr;
    int kvd = 0, vt_pitch = 0;
    int* kv_exp = nullptr;
    const float* kv_bound = nullptr;
    // with the operand split: max |V| of each V column [kvd] (float bits,
    // atomicMax; zeroed by the caller), the attention's exact-int8 error bound
    uint32_t* kv_vmax = nullptr;
    // GEMM_I8, per-tensor scales: zero points (matmul_int8_asymmetric).
    // zp_rows [m] = sum_k A[m, k], zp_cols [n] = sum_k W[n, k] (int32, any k
    // padding included: zeros), zp_k the unpadded k; |zp_a|, |zp_w| <= 2^17
    const int* zp_rows = nullptr;
    const int* zp_cols = nullptr;
    int64_t zp_a = 0, zp_w = 0, zp_k = 0;
};
// GEMM_F16X3 with A2 = W2 = null: the plain fp16 product y = A W^T + bias
// (fp16 operands given directly, scale_a / scales_w unused; matmul_fp16).
int launch_gemm(const GemmArgs& g, cudaStream_t st);
// quantize_fp16: the reference's FP16 encoder (tvq_f16.h) of n floats
int launch_f16_encode(const float* x, uint16_t* q, int64_t n, cudaStream_t st);
// sum over k of each row of a [rows, k] int8 matrix (row pitch k)
int launch_row_sums_i8(const int8_t* a, int64_t rows, int64_t k, int* out, cudaStream_t st);
// Tensor map of a row-major f32 matrix [rows, cols] (row pitch `pitch`
// elements, 0 = cols): box of 32 columns (128 bytes) x box_rows rows,
// 128-byte swizzle.
int make_tma_f32_sw128(CUtensorMap* map, const float* ptr, int64_t rows, int64_t cols, int box_rows,
                       int64_t pitch = 0);
// The same for fp16 [rows, cols]: box of 64 columns x box_rows rows.
int make_tma_f16_sw128(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_rows,
                       int64_t pitch = 0);
// x = hi + lo with hi rounded to TF32 precision (10 explicit mantissa bits)
int launch_split_tf32(const float* x, float* hi, float* lo, int64_t n, cudaStream_t st);
// tvq_int4.cu: group-wise INT4 (int4.tkv).  zps == nullptr: symmetric
// (quantize_int4_grouped / dequantize_int4_grouped), else the AWQ-style
// asymmetric form with per-group zero points.  packed [rows, cols / 2]
// bytes, scales / zps [rows, cols / gs].
int launch_int4_quantize(const float* src, int64_t rows, int64_t cols, int64_t gs, uint8_t* packed, float* scales,
                         int64_t* zps, cudaStream_t st);
int launch_int4_dequantize(const uint8_t* packed, float* dst, int64_t rows, int64_t cols, int64_t gs,
                           const float* scales, const int64_t* zps, cudaStream_t st);
// dst[r, c] = src[r, perm[c]] (inverse: dst[r, perm[c]] = src[r, c])
int launch_permute_cols(const float* src, float* dst, int64_t rows, int64_t cols, const int64_t* perm, int inverse,
                        cudaStream_t st);
// packed [n, k / 2] -> nib - 8 as fp16 [n, k] (GEMM_W4's weights)
int launch_int4_unpack_f16(const uint8_t* packed, void* q, int64_t n, int64_t k, cudaStream_t st);

// Row-scaled fp16 split of x [rows, k]: per row s = 2^e with max|x|*s in
// [2^14, 2^15); hi = fp16(x*s), lo = fp16(x*s - hi); rscale[row] = 1/s.
int launch_split_f16_rows(const float* x, void* hi, void* lo, float* rscale, int64_t rows, int64_t k,
                          cudaStream_t st, const int64_t* perm = nullptr);

// tvq_qdq.cu: the ONNX QDQ operator family (session.tkv:1896-2071, 2789-2905).
// Quantize / dequantize split the tensor at its axis into (outer, dim, inner);
// nsc == 1 is per tensor, nsc == dim per channel.  B of the two matmuls is
// [K, N] row-major as in the reference.
int launch_quantize_linear(const float* x, int8_t* y, int64_t outer, int64_t dim, int64_t inner, const float* scales,
                           int64_t nsc, int64_t zp, cudaStream_t st);
int launch_dequantize_linear(const int8_t* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                             const float* scales, int64_t nsc, int64_t zp, cudaStream_t st);
int launch_matmul_integer(const int8_t* a, const int8_t* b, int32_t* y, int64_t m, int64_t k, int64_t n,
                          cudaStream_t st);
int launch_qlinear_matmul(const int8_t* a, float sa, int64_t zpa, const int8_t* b, float sw, int64_t zpw, float sy,
                          int64_t zpy, int8_t* y, int64_t m, int64_t k, int64_t n, cudaStream_t st);
int launch_dynamic_quantize_linear(const float* x, int64_t n, int8_t* y, float* y_scale, float* y_zp,
                                   cudaStream_t st);

// tvq_calib.cu: calibrate_kl / _percentile / _mse (engine.tkv:42-197).
// out4 (device) = {scale, zero point, min, max}; *fallback = 1 when max |x| <
// 1e-8, where the reference returns calibrate_minmax(data, 1) instead.
int launch_calibrate_kl(const float* x, int64_t n, int num_bins, int target_bins, float* out4, int* fallback,
                        cudaStream_t st);
int launch_calibrate_percentile(const float* x, int64_t n, float percentile, int symmetric, float* out4,
                                cudaStream_t st);
int launch_calibrate_mse(const float* x, int64_t n, int num_candidates, float* out4, double* curve, int* fallback,
                         cudaStream_t st);

}  // namespace tvq
