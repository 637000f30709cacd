/*
 * tvq_oracle.c -- CPU restatement of TokenVector.Inference's post-training-
 * quantization (PTQ) linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * tokenvector/inference_b200: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * never calls it and has no CPU fallback.
 *
 * Every function restates one function of the reference (.tkv source, cited as
 * path:line relative to the reference repository root).  The reference is
 * written in TokenVector, compiled to .NET IL by an external compiler that is
 * not available here, so it cannot be run; this file is the executable model.
 *
 * Numeric model (the reference compiler's, see docs/HANDOFF.md:3663 "JIT widen
 * f64, truncate at the typed boundary"): untyped locals and every arithmetic
 * expression are binary64; a value is rounded to binary32 only where it is
 * stored into something typed 'f32' (list[f32] elements, f32 fields, f32
 * parameters and return values).  `round` is .NET Math.Round (half to even),
 * `int()` truncates and, as on .NET 9+, saturates with NaN -> 0.  The file is
 * compiled with -ffp-contract=off so no multiply-add is fused.
 *
 * Parity pins: calibrate_minmax, quantize/dequantize round trip and the FP8
 * round trip are pinned by the reference's own tests (tv/tests/gap_tests.tkv:
 * 159-240); MatMulInteger and DynamicQuantizeLinear by
 * tv/tests/inference_tests.tkv:847-989.  The INT8 GEMM, per-channel quantize
 * and the f64 epilogue model have no reference test or fixture: their parity
 * is unpinned beyond this restatement.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#include <immintrin.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TVO_API __attribute__((visibility("default")))

/* ---------------------------------------------------------------------- */
/* .NET-style conversions                                                  */
/* ---------------------------------------------------------------------- */

/* int(round(v)) with .NET 9+ saturating conversion (NaN -> 0). */
static inline int64_t net_round_to_i64(double v) {
    if (isnan(v)) return 0;
    double r = nearbyint(v);               /* half to even in the default mode */
    if (r >= 9.2233720368547758e18) return INT64_MAX;
    if (r <= -9.2233720368547758e18) return INT64_MIN;
    return (int64_t)r;
}

static inline int64_t clamp_i64(int64_t v, int64_t lo, int64_t hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

/* ---------------------------------------------------------------------- */
/* tv/runtime/f32_bits.tkv                                                 */
/* ---------------------------------------------------------------------- */

/* f64_to_f32_bits, tv/runtime/f32_bits.tkv:6-57.  The loop is kept as the
 * reference writes it.  Two inputs never finish there: +/-Inf loops forever in
 * `while a >= 2.0` and NaN falls through to an undefined int(NaN).  For those
 * this restatement returns the binary32 Inf / quiet-NaN pattern instead, so
 * that the FP8 encoder below reaches its own ex == 255 branch. */
TVO_API uint32_t tvo_f64_to_f32_bits(double x) {
    if (x == 0.0) return 0;                       /* -0.0 also gives 0 */
    uint32_t s = 0;
    double a = x;
    if (isnan(x)) return 0x7FC00000u;
    if (x < 0.0) { s = 2147483648u; a = 0.0 - x; }
    if (isinf(a)) return s + 255u * 8388608u;
    int64_t e = 0;
    while (a >= 2.0) { a = a / 2.0; e = e + 1; }
    while (a < 1.0) { a = a * 2.0; e = e - 1; }
    int64_t ex = e + 127;
    if (ex >= 255) return s + 255u * 8388608u;
    if (ex <= 0) {
        int64_t sh = e + 149;
        if (sh <= 0) return s;
        return s + (uint32_t)(int64_t)(a * pow(2.0, (double)sh) + 0.5);
    }
    double t = (a - 1.0) * 8388608.0;
    int64_t f = (int64_t)t;
    double r = t - (double)f;
    int64_t m;
    if (r > 0.5) m = f + 1;
    else if (r < 0.5) m = f;
    else { m = f; if (f % 2 != 0) m = f + 1; }
    if (m > 8388607) {
        m = 0;
        ex = ex + 1;
        if (ex >= 255) return s + 255u * 8388608u;
    }
    return s + (uint32_t)ex * 8388608u + (uint32_t)m;
}

/* f32_bits_to_f64, tv/runtime/f32_bits.tkv:60-74 (ex == 255 gives 2^129,
 * i.e. +/-Inf after the f32 return boundary). */
TVO_API double tvo_f32_bits_to_f64(uint32_t b) {
    uint32_t s = b & 2147483648u;
    int64_t ex = (b >> 23) & 255;
    int64_t mant = b & 8388607;
    double v;
    if (ex == 0) v = (double)mant * pow(2.0, 0.0 - 149.0);
    else if (ex == 255) v = pow(2.0, 128.0) * 2.0;
    else v = (1.0 + (double)mant / 8388608.0) * pow(2.0, (double)(ex - 127));
    if (s != 0) v = 0.0 - v;
    return v;
}

/* ---------------------------------------------------------------------- */
/* tv/quantization/types.tkv -- FP8 / FP16 codecs                          */
/* ---------------------------------------------------------------------- */

/* _qt_rne_rshift, tv/quantization/types.tkv:71-93 */
TVO_API int64_t tvo_rne_rshift(int64_t v, int64_t s) {
    if (s > 40) return 0;
    if (s <= 0) return v;
    int64_t half = (int64_t)1 << (s - 1);
    int64_t q = v >> s;
    int64_t rem = v - (q << s);
    if (rem > half) return q + 1;
    if (rem < half) return q;
    if ((q & 1) == 1) return q + 1;
    return q;
}

/* _qt_fp8_encode, tv/quantization/types.tkv:154-191 */
TVO_API int tvo_fp8_encode(float x, int bias, int w, int emax_field, int has_inf, int sat_bits) {
    uint32_t b = tvo_f64_to_f32_bits((double)x);
    int64_t sign = (b >> 31) & 1;
    int64_t ex = (b >> 23) & 255;
    int64_t man = b & 8388607;
    if (ex == 255) {
        if (man != 0) {
            if (has_inf == 1) return (int)((sign << 7) | sat_bits);
            return (int)((sign << 7) | 127);
        }
        if (has_inf == 1) return (int)((sign << 7) | emax_field);
        return (int)((sign << 7) | 127);
    }
    int64_t e, full;
    if (ex == 0) { e = -126; full = man; }
    else { e = ex - 127; full = man | 8388608; }
    int64_t e8 = e + bias;
    if (e8 >= emax_field) return (int)((sign << 7) | sat_bits);
    if (e8 <= 0) {
        int64_t m = tvo_rne_rshift(full, 24 - w - e8);
        int64_t lim = ((int64_t)1 << w) - 1;
        if (m > lim) m = lim;
        return (int)((sign << 7) | m);
    }
    int64_t r = tvo_rne_rshift(full, 23 - w);
    int64_t base = (int64_t)1 << w;
    if (r >= base * 2) {
        r = base;
        e8 = e8 + 1;
        if (e8 >= emax_field) return (int)((sign << 7) | sat_bits);
    }
    return (int)((sign << 7) | (e8 << w) | (r - base));
}

/* _qt_fp8_decode, tv/quantization/types.tkv:193-226 (f32 return boundary). */
TVO_API float tvo_fp8_decode(int v, int bias, int w, int emax_field, int has_inf) {
    int64_t sign = (v >> 7) & 1;
    int ebits = (emax_field == 15) ? 4 : 5;
    int64_t emask = ((int64_t)1 << ebits) - 1;
    int64_t e8 = (v >> w) & emask;
    int64_t m8 = v & (((int64_t)1 << w) - 1);
    int64_t base = (int64_t)1 << w;
    int64_t e32, man32;
    if (e8 == emax_field) {
        if (has_inf == 0) {
            if (m8 == 7)
                return (float)tvo_f32_bits_to_f64((uint32_t)((sign << 31) | 2139095040 | 4194304));
        } else {
            if (m8 != 0)
                return (float)tvo_f32_bits_to_f64((uint32_t)((sign << 31) | 2139095040 | 4194304));
            return (float)tvo_f32_bits_to_f64((uint32_t)((sign << 31) | 2139095040));
        }
    }
    if (e8 == 0) {
        if (m8 == 0) return (float)tvo_f32_bits_to_f64((uint32_t)(sign << 31));
        int64_t t = m8, n = 0;
        while (t < base) { t = t * 2; n = n + 1; }
        e32 = 127 - bias - n;
        man32 = (t - base) << (23 - w);
    } else {
        e32 = e8 - bias + 127;
        man32 = m8 << (23 - w);
    }
    return (float)tvo_f32_bits_to_f64((uint32_t)((sign << 31) | (e32 << 23) | man32));
}

/* native_fp8_e4m3_encode / _decode, tv/quantization/types.tkv:228-233 */
TVO_API int tvo_e4m3_encode(float x) { return tvo_fp8_encode(x, 7, 3, 15, 0, 126); }
TVO_API float tvo_e4m3_decode(int v) { return tvo_fp8_decode(v, 7, 3, 15, 0); }
/* native_fp8_e5m2_encode / _decode, tv/quantization/types.tkv:235-240 */
TVO_API int tvo_e5m2_encode(float x) { return tvo_fp8_encode(x, 15, 2, 31, 1, 252); }
TVO_API float tvo_e5m2_decode(int v) { return tvo_fp8_decode(v, 15, 2, 31, 1); }

/* native_f16_encode, tv/quantization/types.tkv:95-127 */
TVO_API int tvo_f16_encode(float x) {
    uint32_t b = tvo_f64_to_f32_bits((double)x);
    int64_t sign = (b >> 31) & 1, ex = (b >> 23) & 255, man = b & 8388607;
    if (ex == 255) {
        if (man != 0) return (int)((sign << 15) | 31744 | 512);
        return (int)((sign << 15) | 31744);
    }
    int64_t e, full;
    if (ex == 0) { e = -126; full = man; } else { e = ex - 127; full = man | 8388608; }
    int64_t e16 = e + 15;
    if (e16 >= 31) return (int)((sign << 15) | 31744);
    if (e16 <= 0) {
        int64_t m = tvo_rne_rshift(full, 24 - 10 - e16);
        if (m > 1023) m = 1023;
        return (int)((sign << 15) | m);
    }
    int64_t r = tvo_rne_rshift(full, 23 - 10);
    if (r >= 2048) {
        r = 1024;
        e16 = e16 + 1;
        if (e16 >= 31) return (int)((sign << 15) | 31744);
    }
    return (int)((sign << 15) | (e16 << 10) | (r - 1024));
}

/* native_f16_decode, tv/quantization/types.tkv:129-152 */
TVO_API float tvo_f16_decode(int v) {
    int64_t sign = (v >> 15) & 1, e16 = (v >> 10) & 31, m16 = v & 1023, e32, man32;
    if (e16 == 31) {
        if (m16 != 0) return (float)tvo_f32_bits_to_f64((uint32_t)((sign << 31) | 2139095040 | 4194304));
        return (float)tvo_f32_bits_to_f64((uint32_t)((sign << 31) | 2139095040));
    }
    if (e16 == 0) {
        if (m16 == 0) return (float)tvo_f32_bits_to_f64((uint32_t)(sign << 31));
        int64_t t = m16, n = 0;
        while (t < 1024) { t = t * 2; n = n + 1; }
        e32 = 127 - 14 - n;
        man32 = (t - 1024) << 13;
    } else {
        e32 = e16 - 15 + 127;
        man32 = m16 << 13;
    }
    return (float)tvo_f32_bits_to_f64((uint32_t)((sign << 31) | (e32 << 23) | man32));
}

/* ---------------------------------------------------------------------- */
/* tv/quantization/engine.tkv -- calibration and INT8 quantize             */
/* ---------------------------------------------------------------------- */

typedef struct {
    float scale;          /* QuantParams.scale      'f32' */
    int64_t zero_point;   /* QuantParams.zero_point 'i64' */
    float min_val;        /* QuantParams.min_val    'f32' */
    float max_val;        /* QuantParams.max_val    'f32' */
} tvo_qparams;

/* _quant_identity, tv/quantization/engine.tkv:9-10 */
static tvo_qparams quant_identity(void) {
    tvo_qparams p = {1.0f, 0, -FLT_MAX, FLT_MAX};
    return p;
}

/* calibrate_minmax, tv/quantization/engine.tkv:13-36.  Locals are f64; the
 * QuantParams fields round to f32.  NaN elements compare false and are
 * skipped unless data[0] is NaN, exactly as the comparison chain does. */
TVO_API tvo_qparams tvo_calibrate_minmax(const float* data, int64_t n, int symmetric) {
    if (n == 0) return quant_identity();
    double mn = data[0], mx = data[0];
    for (int64_t i = 1; i < n; i++) {
        double v = data[i];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
    }
    tvo_qparams p;
    if (symmetric) {
        double am = fabs(mx);
        if (fabs(mn) > am) am = fabs(mn);
        if (am < 0.00000001) am = 0.00000001;
        p.scale = (float)(am / 127.0);
        p.zero_point = 0;
        p.min_val = (float)(-am);
        p.max_val = (float)am;
        return p;
    }
    if (fabs(mx - mn) < 0.00000001) mx = mn + 0.00000001;
    double scale = (mx - mn) / 255.0;
    int64_t zp = net_round_to_i64(-mn / scale) - 128;
    zp = clamp_i64(zp, -128, 127);
    p.scale = (float)scale;
    p.zero_point = zp;
    p.min_val = (float)mn;
    p.max_val = (float)mx;
    return p;
}

/* Running calibration over several batches (8 seeded
 * batches).  calibrate_minmax over the concatenation equals this max-of-maxes,
 * which is how the caller composes it. */
TVO_API tvo_qparams tvo_calibrate_minmax_batches(const float* const* batches, const int64_t* sizes,
                                                 int64_t nb, int symmetric) {
    int64_t total = 0;
    for (int64_t b = 0; b < nb; b++) total += sizes[b];
    float* cat = (float*)malloc(sizeof(float) * (size_t)(total > 0 ? total : 1));
    int64_t o = 0;
    for (int64_t b = 0; b < nb; b++) {
        memcpy(cat + o, batches[b], sizeof(float) * (size_t)sizes[b]);
        o += sizes[b];
    }
    tvo_qparams p = tvo_calibrate_minmax(cat, total, symmetric);
    free(cat);
    return p;
}

/* calibrate_per_channel_minmax, tv/quantization/engine.tkv:202-213.
 * Returns 0, or -1 for the reference's ValueError cases. */
TVO_API int tvo_calibrate_per_channel_minmax(const float* data, int64_t len, int64_t rows, int64_t cols,
                                             int symmetric, tvo_qparams* out) {
    if (rows <= 0 || cols <= 0) return -1;
    if (len < rows * cols) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) out[r] = tvo_calibrate_minmax(data + r * cols, cols, symmetric);
    return 0;
}

/* quantize_int8_symmetric, tv/quantization/engine.tkv:216-226 */
TVO_API int tvo_quantize_int8_symmetric(const float* src, int64_t n, int8_t* dst, int64_t dst_len, float scale) {
    if (dst_len < n) return -1;
    double inv;
    if ((double)scale > 0.00000001) inv = 1.0 / (double)scale;
    else inv = 1.0 / 0.00000001;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        int64_t q = net_round_to_i64((double)src[i] * inv);
        dst[i] = (int8_t)clamp_i64(q, -127, 127);
    }
    return 0;
}

/* dequantize_int8_symmetric, tv/quantization/engine.tkv:229-234 */
TVO_API int tvo_dequantize_int8_symmetric(const int8_t* src, int64_t n, float* dst, int64_t dst_len, float scale) {
    if (dst_len < n) return -1;
    for (int64_t i = 0; i < n; i++) dst[i] = (float)((double)src[i] * (double)scale);
    return 0;
}

/* quantize_int8_per_channel, tv/quantization/engine.tkv:237-250 */
TVO_API int tvo_quantize_int8_per_channel(const float* src, int64_t src_len, int8_t* dst, int64_t dst_len,
                                          int64_t rows, int64_t cols, const float* scales, int64_t n_scales) {
    if (dst_len < rows * cols || src_len < rows * cols) return -1;
    if (n_scales < rows) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        double sc = scales[r];
        if (sc <= 0.00000001) sc = 0.00000001;
        double inv = 1.0 / sc;
        for (int64_t c = 0; c < cols; c++) {
            int64_t i = r * cols + c;
            dst[i] = (int8_t)clamp_i64(net_round_to_i64((double)src[i] * inv), -127, 127);
        }
    }
    return 0;
}

/* dequantize_int8_per_channel, tv/quantization/engine.tkv:253-262 */
TVO_API int tvo_dequantize_int8_per_channel(const int8_t* src, int64_t src_len, float* dst, int64_t dst_len,
                                            int64_t rows, int64_t cols, const float* scales, int64_t n_scales) {
    if (dst_len < rows * cols || src_len < rows * cols) return -1;
    if (n_scales < rows) return -1;
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++) {
            int64_t i = r * cols + c;
            dst[i] = (float)((double)src[i] * (double)scales[r]);
        }
    return 0;
}

/* quantize_dynamic_int8_rowwise, tv/quantization/engine.tkv:266-285.  The
 * stored scale rounds to f32 but the quantizer uses the f64 `sc`. */
TVO_API int tvo_quantize_dynamic_int8_rowwise(const float* src, int64_t src_len, int8_t* dst, int64_t dst_len,
                                              int64_t rows, int64_t cols, float* scales_out, int64_t n_scales) {
    if (dst_len < rows * cols || src_len < rows * cols) return -1;
    if (n_scales < rows) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        double am = 0.0;
        for (int64_t c = 0; c < cols; c++) {
            double a = fabs((double)src[r * cols + c]);
            if (a > am) am = a;
        }
        if (am < 0.00000001) am = 0.00000001;
        double sc = am / 127.0;
        scales_out[r] = (float)sc;
        double inv = 1.0 / sc;
        for (int64_t c = 0; c < cols; c++) {
            int64_t i = r * cols + c;
            dst[i] = (int8_t)clamp_i64(net_round_to_i64((double)src[i] * inv), -127, 127);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------- */
/* tv/quantization/matmul.tkv -- quantized GEMMs                           */
/* ---------------------------------------------------------------------- */

/* _dot_int8, tv/quantization/matmul.tkv:116-127: K unrolled by 32 with an
 * i64 accumulator, then the tail. */
TVO_API int64_t tvo_dot_int8(const int8_t* a, const int8_t* b, int64_t k) {
    int64_t acc = 0, kk = 0, limit = k - 31;
    while (kk < limit) {
        for (int l = 0; l < 32; l++) acc += (int64_t)a[kk + l] * (int64_t)b[kk + l];
        kk += 32;
    }
    while (kk < k) { acc += (int64_t)a[kk] * (int64_t)b[kk]; kk++; }
    return acc;
}

/* Raw accumulators acc[m,n] = _dot_int8(A[m,:], W[n,:]) as int32 (exact
 * for k < 133143), for bit-exact checks of the tensor-core accumulator. */
TVO_API int tvo_gemm_i8_acc_i32(const int8_t* A, const int8_t* W, int32_t* acc, int64_t m, int64_t n, int64_t k) {
#pragma omp parallel for schedule(static)
    for (int64_t mm = 0; mm < m; mm++)
        for (int64_t nn = 0; nn < n; nn++) acc[mm * n + nn] = (int32_t)tvo_dot_int8(A + mm * k, W + nn * k, k);
    return 0;
}

/* matmul_int8_per_channel, tv/quantization/matmul.tkv:17-29:
 * py = acc * scale_a * scales_w[nn] + bias, evaluated left to right in f64 and
 * rounded to f32 on the list[f32] store.  n_bias == 0 means "no bias". */
TVO_API int tvo_matmul_int8_per_channel(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias,
                                        float* Y, int64_t m, int64_t n, int64_t k, float scale_a,
                                        const float* scales_w, int64_t n_scales) {
    if (n_scales < n) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t mm = 0; mm < m; mm++)
        for (int64_t nn = 0; nn < n; nn++) {
            int64_t acc = tvo_dot_int8(A + mm * k, W + nn * k, k);
            double b = (n_bias > 0) ? (double)bias[nn] : 0.0;
            Y[mm * n + nn] = (float)((double)acc * (double)scale_a * (double)scales_w[nn] + b);
        }
    return 0;
}

/* The faithful scalar form of matmul_int8_per_channel (matmul.tkv:17-29 with
 * _dot_int8, :116-127): one thread, the reference's loop order, the 32-way
 * unrolled i64 accumulation without vectorisation.  It is the single-core CPU
 * baseline of the INT8 GEMM (same results as the OpenMP form above: integer
 * sums are exact in any order). */
__attribute__((optimize("no-tree-vectorize"))) static int64_t dot_int8_scalar(const int8_t* a, const int8_t* b,
                                                                              int64_t k) {
    int64_t acc = 0, kk = 0, limit = k - 31;
    while (kk < limit) {
        for (int l = 0; l < 32; l++) acc += (int64_t)a[kk + l] * (int64_t)b[kk + l];
        kk += 32;
    }
    while (kk < k) { acc += (int64_t)a[kk] * (int64_t)b[kk]; kk++; }
    return acc;
}

__attribute__((optimize("no-tree-vectorize"))) TVO_API int tvo_matmul_int8_per_channel_scalar(
    const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias, float* Y, int64_t m, int64_t n, int64_t k,
    float scale_a, const float* scales_w, int64_t n_scales) {
    if (n_scales < n) return -1;
    for (int64_t mm = 0; mm < m; mm++)
        for (int64_t nn = 0; nn < n; nn++) {
            int64_t acc = dot_int8_scalar(A + mm * k, W + nn * k, k);
            double b = (n_bias > 0) ? (double)bias[nn] : 0.0;
            Y[mm * n + nn] = (float)((double)acc * (double)scale_a * (double)scales_w[nn] + b);
        }
    return 0;
}

/* matmul_int8_symmetric, tv/quantization/matmul.tkv:4-15: s = scale_a*scale_w
 * is an untyped local (f64, exact product of two f32). */
TVO_API int tvo_matmul_int8_symmetric(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias,
                                      float* Y, int64_t m, int64_t n, int64_t k, float scale_a, float scale_w) {
    double s = (double)scale_a * (double)scale_w;
#pragma omp parallel for schedule(static)
    for (int64_t mm = 0; mm < m; mm++)
        for (int64_t nn = 0; nn < n; nn++) {
            int64_t acc = tvo_dot_int8(A + mm * k, W + nn * k, k);
            double b = (n_bias > 0) ? (double)bias[nn] : 0.0;
            Y[mm * n + nn] = (float)((double)acc * s + b);
        }
    return 0;
}

/* matmul_int8_asymmetric, tv/quantization/matmul.tkv:31-44 */
TVO_API int tvo_matmul_int8_asymmetric(const int8_t* A, const int8_t* W, const float* bias, int64_t n_bias,
                                       float* Y, int64_t m, int64_t n, int64_t k, float scale_a, int64_t zp_a,
                                       float scale_w, int64_t zp_w) {
    double s = (double)scale_a * (double)scale_w;
#pragma omp parallel for schedule(static)
    for (int64_t mm = 0; mm < m; mm++)
        for (int64_t nn = 0; nn < n; nn++) {
            int64_t acc = 0;
            for (int64_t kk = 0; kk < k; kk++)
                acc += ((int64_t)A[mm * k + kk] - zp_a) * ((int64_t)W[nn * k + kk] - zp_w);
            double b = (n_bias > 0) ? (double)bias[nn] : 0.0;
            Y[mm * n + nn] = (float)((double)acc * s + b);
        }
    return 0;
}

/* quantize_fp16, tv/quantization/matmul.tkv:106-114 (the fp16 pattern of
 * each element; the reference splits it into two signed bytes) */
TVO_API int tvo_quantize_fp16(const float* src, int64_t n, uint16_t* dst) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) dst[i] = (uint16_t)tvo_f16_encode(src[i]);
    return 0;
}

/* matmul_fp16, tv/quantization/matmul.tkv:79-96: A [m,k], W [n,k] fp16
 * patterns decoded by FP16.to_float (native_f16_decode), acc an untyped
 * (binary64) sum in k order, y = fl32(acc + bias). */
TVO_API int tvo_matmul_fp16(const uint16_t* A, const uint16_t* W, const float* bias, int64_t n_bias, float* Y,
                            int64_t m, int64_t n, int64_t k) {
    static double tab[65536];
    static int ready = 0;
    if (!ready) {
        for (int v = 0; v < 65536; v++) tab[v] = (double)tvo_f16_decode(v);
        ready = 1;
    }
#pragma omp parallel for schedule(static)
    for (int64_t mm = 0; mm < m; mm++)
        for (int64_t nn = 0; nn < n; nn++) {
            double acc = 0.0;
            for (int64_t kk = 0; kk < k; kk++) acc = acc + tab[A[mm * k + kk]] * tab[W[nn * k + kk]];
            double b = (n_bias > 0) ? (double)bias[nn] : 0.0;
            Y[mm * n + nn] = (float)(acc + b);
        }
    return 0;
}

/* Decode table for E4M3 bytes through the restated decoder. */
static void e4m3_table(double* t) {
    for (int v = 0; v < 256; v++) t[v] = (double)tvo_e4m3_decode(v);
}

/* quantize_fp8_e4m3, tv/quantization/matmul.tkv:60-66, storing the encoded
 * byte itself (the reference stores byte - 128 in a list[i32]; the byte form
 * is what the tensor cores read, the offset is applied at the boundary). */
TVO_API int tvo_quantize_fp8_e4m3(const float* src, int64_t n, uint8_t* dst) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) dst[i] = (uint8_t)tvo_e4m3_encode(src[i]);
    return 0;
}

/* Scaled FP8 quantize used by BASELINE config 3 (scale = amax/448): the
 * reference has no scaled FP8 quantizer, so it is composed the way the INT8
 * quantizer is (engine.tkv:219-224): inv = 1.0/scale in f64, the product is
 * rounded to f32 at the encoder's 'f32' parameter, then encoded. */
TVO_API int tvo_quantize_fp8_e4m3_scaled(const float* src, int64_t rows, int64_t cols, uint8_t* dst,
                                         const float* scales, int per_row) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        double sc = per_row ? (double)scales[r] : (double)scales[0];
        double inv = (sc > 0.00000001) ? 1.0 / sc : 1.0 / 0.00000001;
        for (int64_t c = 0; c < cols; c++) {
            float v = (float)((double)src[r * cols + c] * inv);
            dst[r * cols + c] = (uint8_t)tvo_e4m3_encode(v);
        }
    }
    return 0;
}

/* dequantize_fp8_e4m3, tv/quantization/matmul.tkv:68-73 (byte form) */
TVO_API int tvo_dequantize_fp8_e4m3(const uint8_t* src, int64_t n, float* dst) {
    for (int64_t i = 0; i < n; i++) dst[i] = tvo_e4m3_decode(src[i]);
    return 0;
}

/* matmul_fp8_e4m3, tv/quantization/matmul.tkv:46-58: two decodes per MAC, f64
 * accumulator (acc = 0.0), py = acc + bias.  The reference has no scales; the
 * optional scale_a * scales_w[n] factor multiplies the
 * accumulator before the bias, mirroring the INT8 epilogue (matmul.tkv:28).
 * With scale_a == 1 and scales_w == NULL the expression is the reference's. */
TVO_API int tvo_matmul_fp8_e4m3(const uint8_t* A, const uint8_t* W, const float* bias, int64_t n_bias,
                                float* Y, int64_t m, int64_t n, int64_t k, float scale_a, const float* scales_w) {
    double tab[256];
    e4m3_table(tab);
    const int scaled = (scales_w != NULL) || scale_a != 1.0f;
#pragma omp parallel for schedule(static)
    for (int64_t mm = 0; mm < m; mm++)
        for (int64_t nn = 0; nn < n; nn++) {
            double acc = 0.0;
            for (int64_t kk = 0; kk < k; kk++) acc = acc + tab[A[mm * k + kk]] * tab[W[nn * k + kk]];
            double b = (n_bias > 0) ? (double)bias[nn] : 0.0;
            if (scaled) {
                double sw = scales_w ? (double)scales_w[nn] : 1.0;
                Y[mm * n + nn] = (float)(acc * (double)scale_a * sw + b);
            } else {
                Y[mm * n + nn] = (float)(acc + b);
            }
        }
    return 0;
}

/* ---------------------------------------------------------------------- */
/* Activations: tv/optimization/kernels.tkv:14-38, tv/training/tensor.tkv  */
/* ---------------------------------------------------------------------- */

/* _tanh(x: f32) -> f32, tv/optimization/kernels.tkv:32-38 */
static float ref_tanh(float x) {
    if ((double)x > 10.0) return 1.0f;
    if ((double)x < -10.0) return -1.0f;
    double e = exp(2.0 * (double)x);
    return (float)((e - 1.0) / (e + 1.0));
}

/* apply_activation GELU (tanh form), tv/optimization/kernels.tkv:22-24 */
TVO_API float tvo_gelu_tanh(float x) {
    double xd = x;
    double x3 = xd * xd * xd;
    float targ = (float)(0.79788456 * (xd + 0.044715 * x3));
    return (float)(0.5 * xd * (1.0 + (double)ref_tanh(targ)));
}

/* erf(x: f32) -> f32, Abramowitz-Stegun 7.1.26, tv/training/tensor.tkv:165-187 */
TVO_API float tvo_erf_as(float x) {
    double sg = 1.0;
    if (x < 0.0f) sg = -1.0;
    double ax = fabs((double)x);
    double t = 1.0 / (1.0 + 0.3275911 * ax);
    double poly = 1.061405429;
    poly = poly * t + -1.453152027;
    poly = poly * t + 1.421413741;
    poly = poly * t + -0.284496736;
    poly = poly * t + 0.254829592;
    poly = poly * t;
    return (float)(sg * (1.0 - exp(-ax * ax) * poly));
}

/* gelu_erf(v: f32) -> f32, tv/training/tensor.tkv:189-190: the argument of
 * erf rounds to f32 at erf's parameter. */
TVO_API float tvo_gelu_erf(float v) {
    float arg = (float)((double)v / 1.4142135623730951);
    return (float)(0.5 * (double)v * (1.0 + (double)tvo_erf_as(arg)));
}

TVO_API void tvo_gelu_erf_inplace(float* x, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) x[i] = tvo_gelu_erf(x[i]);
}

/* ---------------------------------------------------------------------- */
/* GPT-2 composition pieces, tv/training/gpt2_ref.tkv                      */
/* ---------------------------------------------------------------------- */

/* gpt2_layernorm interpreted path, tv/training/gpt2_ref.tkv:61-78 (f64
 * statistics, one rounding to f32 on store). */
TVO_API void tvo_layernorm(const float* x, const float* g, const float* b, float* out, int64_t n, int64_t h,
                           double eps) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) {
        const float* xr = x + i * h;
        double mu = 0.0;
        for (int64_t j = 0; j < h; j++) mu = mu + (double)xr[j];
        mu = mu / (double)h;
        double v = 0.0;
        for (int64_t j = 0; j < h; j++) { double d = (double)xr[j] - mu; v = v + d * d; }
        v = v / (double)h;
        double rstd = 1.0 / sqrt(v + eps);
        for (int64_t j = 0; j < h; j++)
            out[i * h + j] = (float)(((double)xr[j] - mu) * rstd * (double)g[j] + (double)b[j]);
    }
}

/* gpt2_embed, tv/training/gpt2_ref.tkv:80-88 */
TVO_API void tvo_embed(const int64_t* ids, const int64_t* pos, const float* wte, const float* wpe, float* out,
                       int64_t n, int64_t h) {
    for (int64_t i = 0; i < n; i++)
        for (int64_t j = 0; j < h; j++)
            out[i * h + j] = (float)((double)wte[ids[i] * h + j] + (double)wpe[pos[i] * h + j]);
}

/* gpt2_attention scalar path, tv/training/gpt2_ref.tkv:360-395 (without the
 * projection, which is a QuantizedGemm here): qkv rows are [Q | K | V] with
 * heads contiguous (head_dim = h / nheads); causal within each packed
 * sequence [seg[s], seg[s+1]).  f64 throughout, ctx rounds to f32. */
TVO_API void tvo_attention_causal(const float* qkv, float* ctx, int64_t n, int64_t h, int64_t nheads,
                                  const int64_t* seg, int64_t nseg) {
    int64_t hd = h / nheads;
    double inv = 1.0 / sqrt((double)hd);
    for (int64_t s = 0; s < nseg; s++) {
        int64_t lo = seg[s], hi = seg[s + 1];
#pragma omp parallel for schedule(dynamic, 4)
        for (int64_t t = lo; t < hi; t++) {
            double* sc = (double*)malloc(sizeof(double) * (size_t)(hi - lo + hd));
            double* pv = sc + (hi - lo);
            for (int64_t head = 0; head < nheads; head++) {
                int64_t ho = head * hd;
                const float* q = qkv + t * 3 * h + ho;
                for (int64_t u = lo; u <= t; u++) {
                    const float* kv = qkv + u * 3 * h + h + ho;
                    double acc = 0.0;
                    for (int64_t d = 0; d < hd; d++) acc = acc + (double)q[d] * (double)kv[d];
                    sc[u - lo] = acc * inv;
                }
                double mx = sc[0];
                for (int64_t u = 1; u <= t - lo; u++) if (sc[u] > mx) mx = sc[u];
                double tot = 0.0;
                for (int64_t u = 0; u <= t - lo; u++) { double e = exp(sc[u] - mx); sc[u] = e; tot = tot + e; }
                double inv_tot = 1.0 / tot;
                /* every output d sums over u in order; the d outputs advance
                 * together so that each V row is read once, contiguously */
                for (int64_t d = 0; d < hd; d++) pv[d] = 0.0;
                for (int64_t u = lo; u <= t; u++) {
                    const double p = sc[u - lo];
                    const float* vr = qkv + u * 3 * h + 2 * h + ho;
                    for (int64_t d = 0; d < hd; d++) pv[d] = pv[d] + p * (double)vr[d];
                }
                for (int64_t d = 0; d < hd; d++) ctx[t * h + ho + d] = (float)(pv[d] * inv_tot);
            }
            free(sc);
        }
    }
}

/* residual: out = a + b (f32 store) */
TVO_API void tvo_add(const float* a, const float* b, float* out, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; i++) out[i] = (float)((double)a[i] + (double)b[i]);
}

/* LM head with the tied embedding, tv/training/gpt2_ref.tkv:603-610:
 * logits[i,o] = sum_k x[i,k] * wte[o,k], f64 accumulator, k in order.
 * Tiled for the cache (64 wte rows x 64 rows of x per tile, both held as
 * f64, x transposed in groups of eight rows) and for the adder (four wte
 * rows x eight x rows side by side): every output still keeps its own
 * sequential k-order sum, so the bits equal the plain loop
 * (tvo_lm_head_plain); only the order in which outputs are formed changes. */
#define TVO_LMX 8   /* x rows per vector group */
#define TVO_LMO 64  /* wte rows per tile */
#define TVO_LMT 64  /* x rows per tile */
TVO_API void tvo_lm_head(const float* x, const float* wte, float* logits, int64_t n, int64_t vocab, int64_t h) {
    const int64_t nb = (n + TVO_LMX - 1) / TVO_LMX;
    double* xt = (double*)malloc(sizeof(double) * (size_t)(nb * h * TVO_LMX));
    if (!xt) return;
    for (int64_t b = 0; b < nb; b++)
        for (int64_t k = 0; k < h; k++)
            for (int j = 0; j < TVO_LMX; j++) {
                const int64_t i = b * TVO_LMX + j;
                xt[(b * h + k) * TVO_LMX + j] = i < n ? (double)x[i * h + k] : 0.0;
            }
    const int64_t ntiles = (vocab + TVO_LMO - 1) / TVO_LMO;
#pragma omp parallel
    {
        double* wd = (double*)malloc(sizeof(double) * (size_t)(TVO_LMO * h));
#pragma omp for schedule(dynamic, 4)
        for (int64_t t = 0; t < ntiles; t++) {
            const int64_t o0 = t * TVO_LMO;
            const int64_t no = (vocab - o0 < TVO_LMO) ? vocab - o0 : TVO_LMO;
            if (!wd) continue;
            for (int64_t r = 0; r < TVO_LMO; r++)
                for (int64_t k = 0; k < h; k++) wd[r * h + k] = r < no ? (double)wte[(o0 + r) * h + k] : 0.0;
            for (int64_t b0 = 0; b0 < nb; b0 += TVO_LMT / TVO_LMX)
                for (int64_t r = 0; r < no; r += 4)
                    for (int64_t b = b0; b < nb && b < b0 + TVO_LMT / TVO_LMX; b++) {
                        const double* xb = xt + b * h * TVO_LMX;
                        const double *w0 = wd + r * h, *w1 = w0 + h, *w2 = w1 + h, *w3 = w2 + h;
                        /* eight lanes per wte row as two 4-wide vectors: a separate
                         * multiply and add per lane, exactly the scalar sum */
                        __m256d a0l = _mm256_setzero_pd(), a0h = a0l, a1l = a0l, a1h = a0l;
                        __m256d a2l = a0l, a2h = a0l, a3l = a0l, a3h = a0l;
                        for (int64_t k = 0; k < h; k++) {
                            const __m256d xl = _mm256_loadu_pd(xb + k * TVO_LMX);
                            const __m256d xh = _mm256_loadu_pd(xb + k * TVO_LMX + 4);
                            const __m256d c0 = _mm256_broadcast_sd(w0 + k), c1 = _mm256_broadcast_sd(w1 + k);
                            const __m256d c2 = _mm256_broadcast_sd(w2 + k), c3 = _mm256_broadcast_sd(w3 + k);
                            a0l = _mm256_add_pd(a0l, _mm256_mul_pd(xl, c0));
                            a0h = _mm256_add_pd(a0h, _mm256_mul_pd(xh, c0));
                            a1l = _mm256_add_pd(a1l, _mm256_mul_pd(xl, c1));
                            a1h = _mm256_add_pd(a1h, _mm256_mul_pd(xh, c1));
                            a2l = _mm256_add_pd(a2l, _mm256_mul_pd(xl, c2));
                            a2h = _mm256_add_pd(a2h, _mm256_mul_pd(xh, c2));
                            a3l = _mm256_add_pd(a3l, _mm256_mul_pd(xl, c3));
                            a3h = _mm256_add_pd(a3h, _mm256_mul_pd(xh, c3));
                        }
                        double a0[TVO_LMX], a1[TVO_LMX], a2[TVO_LMX], a3[TVO_LMX];
                        _mm256_storeu_pd(a0, a0l); _mm256_storeu_pd(a0 + 4, a0h);
                        _mm256_storeu_pd(a1, a1l); _mm256_storeu_pd(a1 + 4, a1h);
                        _mm256_storeu_pd(a2, a2l); _mm256_storeu_pd(a2 + 4, a2h);
                        _mm256_storeu_pd(a3, a3l); _mm256_storeu_pd(a3 + 4, a3h);
                        for (int j = 0; j < TVO_LMX; j++) {
                            const int64_t i = b * TVO_LMX + j;
                            if (i >= n) break;
                            float* row = logits + i * vocab + o0 + r;
                            row[0] = (float)a0[j];
                            if (r + 1 < no) row[1] = (float)a1[j];
                            if (r + 2 < no) row[2] = (float)a2[j];
                            if (r + 3 < no) row[3] = (float)a3[j];
                        }
                    }
        }
        free(wd);
    }
    free(xt);
}

/* The same LM head as the plain loop of the reference (one output at a time);
 * kept to check that the interleaved form above gives the same bits. */
TVO_API void tvo_lm_head_plain(const float* x, const float* wte, float* logits, int64_t n, int64_t vocab, int64_t h) {
#pragma omp parallel for schedule(static)
    for (int64_t o = 0; o < vocab; o++)
        for (int64_t i = 0; i < n; i++) {
            double acc = 0.0;
            for (int64_t k = 0; k < h; k++) acc = acc + (double)x[i * h + k] * (double)wte[o * h + k];
            logits[i * vocab + o] = (float)acc;
        }
}

/* _gi_noise, tv/training/gpt2_ref.tkv:1977-1991: LCG + Box-Muller, x0.02 */
TVO_API void tvo_gi_noise(float* out, int64_t n, int64_t seed, double mult) {
    int64_t s = seed % 2147483648LL;
    for (int64_t i = 0; i < n; i++) {
        s = (s * 1103515245LL + 12345LL) % 2147483648LL;
        double u1 = ((double)s + 0.5) / 2147483648.0;
        s = (s * 1103515245LL + 12345LL) % 2147483648LL;
        double u2 = (double)s / 2147483648.0;
        out[i] = (float)(sqrt(0.0 - 2.0 * log(u1)) * cos(6.283185307179586 * u2) * mult);
    }
}

TVO_API int tvo_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

TVO_API void tvo_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ---------------------------------------------------------------------- */
/* tv/runtime/session.tkv: the ONNX QDQ operator family                   */
/* ---------------------------------------------------------------------- */

/* Channel of flat index i for the (outer, dim, inner) split of a tensor at
 * its quantization axis (session.tkv:1925-1940); 0 when per-tensor. */
static inline int64_t qdq_channel(int64_t i, int64_t dim, int64_t inner, int64_t nsc) {
    return nsc == 1 ? 0 : (i / inner) % dim;
}

/* _exec_quantize_linear, session.tkv:1896-1953.  s = sc > 1e-12 ? sc : 1e-12
 * (the floor is the double 1e-12), q = int(round(x / s)) + zp in f64,
 * clamped to [-128, 127].  nsc == 1: per tensor; else one scale per channel
 * of the axis split (outer, dim, inner), nsc == dim. */
TVO_API int tvo_quantize_linear(const float* x, int8_t* y, int64_t outer, int64_t dim, int64_t inner,
                                const float* sc, int64_t nsc, int64_t zp) {
    const int64_t n = outer * dim * inner;
    if (nsc != 1 && nsc != dim) return -1;
    for (int64_t i = 0; i < n; i++) {
        const float sf = sc[qdq_channel(i, dim, inner, nsc)];
        const double s = ((double)sf > 0.000000000001) ? (double)sf : 0.000000000001;
        int64_t q = net_round_to_i64((double)x[i] / s);
        q = (q > INT64_MAX - 256 || q < INT64_MIN + 256) ? q : q + zp;
        y[i] = (int8_t)clamp_i64(q, -128, 127);
    }
    return 0;
}

/* _exec_dequantize_linear, session.tkv:1955-1990: y = float(int(x) - zp) * sc
 * in f64, stored to f32. */
TVO_API int tvo_dequantize_linear(const int8_t* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                                  const float* sc, int64_t nsc, int64_t zp) {
    const int64_t n = outer * dim * inner;
    if (nsc != 1 && nsc != dim) return -1;
    for (int64_t i = 0; i < n; i++) {
        const double v = (double)((int64_t)x[i] - zp) * (double)sc[qdq_channel(i, dim, inner, nsc)];
        y[i] = (float)v;
    }
    return 0;
}

/* _exec_matmul_integer, session.tkv:2789-2851: Y int32 [m, n] = A int8
 * [m, k] x B int8 [k, n] (B row-major [K, N]); zero points are not read. */
TVO_API int tvo_matmul_integer(const int8_t* a, const int8_t* b, int32_t* y, int64_t m, int64_t k, int64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            int64_t acc = 0;
            for (int64_t p = 0; p < k; p++) acc += (int64_t)a[i * k + p] * (int64_t)b[p * n + j];
            y[i * n + j] = (int32_t)acc;
        }
    return 0;
}

/* _exec_qlinear_matmul, session.tkv:1992-2071: acc = sum (a - zpa)(b - zpw)
 * over k (B row-major [K, N]), mult = sa * sw / sy in f64 (sy == 0 -> 1),
 * y = clamp(int(round(acc * mult)) + zpy, -128, 127). */
TVO_API int tvo_qlinear_matmul(const int8_t* a, float sa, int64_t zpa, const int8_t* b, float sw, int64_t zpw,
                               float sy, int64_t zpy, int8_t* y, int64_t m, int64_t k, int64_t n) {
    const double syd = ((double)sy == 0.0) ? 1.0 : (double)sy;
    const double mult = (double)sa * (double)sw / syd;
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            int64_t acc = 0;
            for (int64_t p = 0; p < k; p++)
                acc += ((int64_t)a[i * k + p] - zpa) * ((int64_t)b[p * n + j] - zpw);
            int64_t v = net_round_to_i64((double)acc * mult);
            v = (v > INT64_MAX - 256 || v < INT64_MIN + 256) ? v : v + zpy;
            y[i * n + j] = (int8_t)clamp_i64(v, -128, 127);
        }
    return 0;
}

/* _exec_dyn_quant, session.tkv:2853-2905: uint8 asymmetric quantization over
 * the whole tensor, stored shifted to int8.  mn / mx start at x[0] and take
 * strict comparisons (a NaN never replaces them), then include 0; the range
 * is at least 1e-8; sc = (mx - mn) / 255 in f64 (stored to f32 as the scale
 * output), zp = clamp(int(round(-mn / sc)), 0, 255), q = clamp(int(round(x /
 * sc)) + zp, 0, 255) - 128 with the unrounded f64 sc. */
TVO_API int tvo_dynamic_quantize_linear(const float* x, int64_t n, int8_t* y, float* y_scale, float* y_zp) {
    if (n < 1) return -1;
    float mn = x[0], mx = x[0];
    for (int64_t i = 1; i < n; i++) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
    }
    double mnd = mn, mxd = mx;
    if (mnd > 0.0) mnd = 0.0;
    if (mxd < 0.0) mxd = 0.0;
    if (mxd - mnd < 0.00000001) mxd = mnd + 0.00000001;
    const double sc = (mxd - mnd) / 255.0;
    const int64_t zp = clamp_i64(net_round_to_i64(-mnd / sc), 0, 255);
    *y_scale = (float)sc;
    *y_zp = (float)zp;
    for (int64_t i = 0; i < n; i++) {
        int64_t q = net_round_to_i64((double)x[i] / sc);
        q = (q > INT64_MAX - 256 || q < INT64_MIN + 256) ? q : q + zp;
        q = clamp_i64(q, 0, 255) - 128;
        y[i] = (int8_t)clamp_i64(q, -128, 127);
    }
    return 0;
}

/* ---------------------------------------------------------------------- */
/* tv/quantization/engine.tkv -- calibration methods (KL, percentile, MSE) */
/* ---------------------------------------------------------------------- */

/* int() of a non-negative f64 (truncation, saturating, NaN -> 0). */
static inline int64_t net_trunc_to_i64(double v) {
    if (isnan(v)) return 0;
    if (v >= 9.2233720368547758e18) return INT64_MAX;
    if (v <= -9.2233720368547758e18) return INT64_MIN;
    return (int64_t)v;
}

/* max |data[i]| with `a > am` from am = 0 (NaN never wins), f64. */
static double abs_max(const float* data, int64_t n) {
    double am = 0.0;
    for (int64_t i = 0; i < n; i++) {
        double a = fabs((double)data[i]);
        if (a > am) am = a;
    }
    return am;
}

/* calibrate_kl, tv/quantization/engine.tkv:42-122: histogram of |x| over
 * [0, am) in num_bins bins (bin = int(|x| / bw), NaN -> bin 0, the top clamps
 * to the last bin); for th = target_bins, +16, ..., num_bins the tail is
 * merged into bin th-1, the truncated distribution normalised, quantized to
 * target_bins equal-width groups and expanded back, KL(P||Q) summed in bin
 * order over the bins where both exceed 1e-12; the first strict minimum
 * wins; threshold = best_th * bw.  All sums in f64, in the reference's order. */
TVO_API tvo_qparams tvo_calibrate_kl(const float* data, int64_t n, int64_t num_bins, int64_t target_bins) {
    if (n == 0) return quant_identity();
    const double am = abs_max(data, n);
    if (am < 0.00000001) return tvo_calibrate_minmax(data, n, 1);
    int64_t* hist = (int64_t*)calloc((size_t)num_bins, sizeof(int64_t));
    double* p = (double*)calloc((size_t)num_bins, sizeof(double));
    double* q = (double*)calloc((size_t)num_bins, sizeof(double));
    const double bw = am / (double)num_bins;
    for (int64_t i = 0; i < n; i++) {
        int64_t b = net_trunc_to_i64(fabs((double)data[i]) / bw);
        if (b >= num_bins) b = num_bins - 1;
        hist[b] += 1;
    }
    double total = 0.0;
    for (int64_t i = 0; i < num_bins; i++) total = total + (double)hist[i];
    if (total == 0) {
        free(hist); free(p); free(q);
        return tvo_calibrate_minmax(data, n, 1);
    }
    int64_t best_bin = num_bins;
    double best_kl = 1e45;
    for (int64_t th = target_bins; th <= num_bins; th += 16) {
        double s = 0.0;
        for (int64_t i = 0; i < th; i++) {
            p[i] = (double)hist[i];
            s = s + (double)hist[i];
        }
        for (int64_t i = th; i < num_bins; i++) {
            p[th - 1] = p[th - 1] + (double)hist[i];
            s = s + (double)hist[i];
        }
        if (s != 0) {
            for (int64_t i = 0; i < th; i++) p[i] = p[i] / s;
            const int64_t per = th / target_bins;
            if (per >= 1) {
                for (int64_t i = 0; i < th; i++) q[i] = 0.0;
                for (int64_t b = 0; b < target_bins; b++) {
                    const int64_t start = b * per;
                    const int64_t end = (b == target_bins - 1) ? th : start + per;
                    double mass = 0.0;
                    for (int64_t i = start; i < end; i++) mass = mass + p[i];
                    int64_t span = end - start;
                    if (span < 1) span = 1;
                    const double share = mass / (double)span;
                    for (int64_t i = start; i < end; i++) q[i] = share;
                }
                double kl = 0.0;
                for (int64_t i = 0; i < th; i++)
                    if (p[i] > 0.000000000001 && q[i] > 0.000000000001) kl = kl + p[i] * log(p[i] / q[i]);
                if (kl < best_kl) {
                    best_kl = kl;
                    best_bin = th;
                }
            }
        }
    }
    free(hist); free(p); free(q);
    const double thr = (double)best_bin * bw;
    tvo_qparams r = {(float)(thr / 127.0), 0, (float)(-thr), (float)thr};
    return r;
}

static int cmp_f32_asc(const void* a, const void* b) {
    const float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

/* calibrate_percentile, tv/quantization/engine.tkv:125-162: clip = the
 * int(min(n-1, percentile/100 * n))-th smallest |x| (ascending; inputs
 * without NaN -- the reference's heap sort leaves NaN placement undefined),
 * floored at 1e-8.  Symmetric: scale clip/127.  Asymmetric: mn / mx start at
 * data[0] unclamped, then take data[1..] clamped to [-clip, clip].
 * *err = 1 for percentile outside (0, 100] (the reference's ValueError). */
TVO_API tvo_qparams tvo_calibrate_percentile(const float* data, int64_t n, float percentile, int symmetric,
                                             int* err) {
    *err = 0;
    if (n == 0) return quant_identity();
    if (percentile <= 0.0f || percentile > 100.0f) {
        *err = 1;
        return quant_identity();
    }
    float* ab = (float*)malloc((size_t)n * sizeof(float));
    for (int64_t i = 0; i < n; i++) ab[i] = fabsf(data[i]);
    qsort(ab, (size_t)n, sizeof(float), cmp_f32_asc);
    const double nab = (double)(n - 1 < 0 ? 0 : n - 1);
    const double want = (double)percentile / 100.0 * (double)n;
    const int64_t idx = net_trunc_to_i64(nab < want ? nab : want);
    double clip = ab[idx];
    free(ab);
    if (clip <= 0.00000001) clip = 0.00000001;
    tvo_qparams r;
    if (symmetric) {
        r.scale = (float)(clip / 127.0);
        r.zero_point = 0;
        r.min_val = (float)(-clip);
        r.max_val = (float)clip;
        return r;
    }
    double mn = data[0], mx = data[0];
    for (int64_t i = 1; i < n; i++) {
        double v = data[i];
        if (v < -clip) v = -clip;
        if (v > clip) v = clip;
        if (v < mn) mn = v;
        if (v > mx) mx = v;
    }
    if (fabs(mx - mn) < 0.00000001) mx = mn + 0.00000001;
    const double scale = (mx - mn) / 255.0;
    int64_t zp = net_round_to_i64(-mn / scale) - 128;
    r.scale = (float)scale;
    r.zero_point = clamp_i64(zp, -128, 127);
    r.min_val = (float)mn;
    r.max_val = (float)mx;
    return r;
}

/* calibrate_mse, tv/quantization/engine.tkv:165-197: thresholds am*c/num for
 * c = 1..num (num >= 4); per threshold the mean of (x - dq)^2 with
 * dq = clamp(int(round(clamp(x, +-thr) * (1/scale))), -127, 127) * scale,
 * scale = thr/127; the first strict minimum wins.  Each candidate's sum runs
 * in element order (candidates in parallel). */
TVO_API tvo_qparams tvo_calibrate_mse(const float* data, int64_t n, int64_t num_candidates) {
    if (n == 0) return quant_identity();
    if (num_candidates < 4) num_candidates = 4;
    const double am = abs_max(data, n);
    if (am < 0.00000001) return tvo_calibrate_minmax(data, n, 1);
    double* mses = (double*)malloc((size_t)num_candidates * sizeof(double));
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t c = 1; c <= num_candidates; c++) {
        const double thr = am * (double)c / (double)num_candidates;
        const double scale = thr / 127.0;
        const double inv = 1.0 / scale;
        double mse = 0.0;
        for (int64_t i = 0; i < n; i++) {
            double cl = data[i];
            if (cl < -thr) cl = -thr;
            if (cl > thr) cl = thr;
            const double dq = (double)clamp_i64(net_round_to_i64(cl * inv), -127, 127) * scale;
            const double d = (double)data[i] - dq;
            mse = mse + d * d;
        }
        mses[c - 1] = mse / (double)n;
    }
    double best_thr = am, best_mse = 1e45;
    for (int64_t c = 1; c <= num_candidates; c++) {
        if (mses[c - 1] < best_mse) {
            best_mse = mses[c - 1];
            best_thr = am * (double)c / (double)num_candidates;
        }
    }
    free(mses);
    tvo_qparams r = {(float)(best_thr / 127.0), 0, (float)(-best_thr), (float)best_thr};
    return r;
}

/* The per-candidate mean squared errors of calibrate_mse (test support). */
TVO_API void tvo_calibrate_mse_curve(const float* data, int64_t n, int64_t num_candidates, double* out) {
    const double am = abs_max(data, n);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t c = 1; c <= num_candidates; c++) {
        const double thr = am * (double)c / (double)num_candidates;
        const double scale = thr / 127.0;
        const double inv = 1.0 / scale;
        double mse = 0.0;
        for (int64_t i = 0; i < n; i++) {
            double cl = data[i];
            if (cl < -thr) cl = -thr;
            if (cl > thr) cl = thr;
            const double dq = (double)clamp_i64(net_round_to_i64(cl * inv), -127, 127) * scale;
            const double d = (double)data[i] - dq;
            mse = mse + d * d;
        }
        out[c - 1] = mse / (double)n;
    }
}

/* ---------------------------------------------------------------------- */
/* tv/quantization/int4.tkv: group-wise INT4 (GPTQ / AWQ layout)           */
/* ---------------------------------------------------------------------- */
/* Packing: two nibbles per byte, low nibble first; the reference keeps the
 * bytes in list[i32] (values 0..255), here uint8.  Locals are f64, list
 * stores round to f32, int(round()) is half-to-even (net_round_to_i64). */

/* quantize_int4_grouped, int4.tkv:27-48 (+ _int4_scales_sym :18-29):
 * scale[r, g] = fl32(max(max|x|, 1e-8) / 7); q = clamp(round(x * (1/s)),
 * -8, 7) + 8.  Returns -1 when cols is not a multiple of group_size or odd
 * (the reference's ValueError). */
TVO_API int tvo_quantize_int4_grouped(const float* src, int64_t rows, int64_t cols, int64_t group_size,
                                      uint8_t* packed, float* scales) {
    if (group_size <= 0 || cols % group_size != 0 || cols % 2 != 0) return -1;
    const int64_t ng = cols / group_size;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t g = 0; g < ng; g++) {
            double am = 0.0;
            for (int64_t c = 0; c < group_size; c++) {
                const double a = fabs((double)src[r * cols + g * group_size + c]);
                if (a > am) am = a;
            }
            if (am < 0.00000001) am = 0.00000001;
            scales[r * ng + g] = (float)(am / 7.0);
        }
        for (int64_t c = 0; c < cols; c += 2) {
            const double sc = scales[r * ng + c / group_size];
            const double inv = 1.0 / sc;
            const int64_t q0 = clamp_i64(net_round_to_i64((double)src[r * cols + c] * inv), -8, 7) + 8;
            const int64_t q1 = clamp_i64(net_round_to_i64((double)src[r * cols + c + 1] * inv), -8, 7) + 8;
            packed[r * (cols / 2) + c / 2] = (uint8_t)((q1 << 4) | q0);
        }
    }
    return 0;
}

/* dequantize_int4_grouped, int4.tkv:51-64: fl32((nib - 8) * s). */
TVO_API int tvo_dequantize_int4_grouped(const uint8_t* packed, float* dst, int64_t rows, int64_t cols,
                                        int64_t group_size, const float* scales) {
    if (group_size <= 0 || cols % group_size != 0 || cols % 2 != 0) return -1;
    const int64_t ng = cols / group_size;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c += 2) {
            const double sc = scales[r * ng + c / group_size];
            const int b = packed[r * (cols / 2) + c / 2];
            dst[r * cols + c] = (float)((double)((b & 0xF) - 8) * sc);
            dst[r * cols + c + 1] = (float)((double)(((b >> 4) & 0xF) - 8) * sc);
        }
    return 0;
}

/* quantize_int4_grouped_asym, int4.tkv:68-150: per group (scale, zero
 * point) with the reference's corrections for all-positive groups (zp 0,
 * scale max/15) and zp clamped to 15 (scale -min/15), floors 1e-8. */
TVO_API int tvo_quantize_int4_grouped_asym(const float* src, int64_t rows, int64_t cols, int64_t group_size,
                                           uint8_t* packed, float* scales, int64_t* zps) {
    if (group_size <= 0 || cols % group_size != 0 || cols % 2 != 0) return -1;
    const int64_t ng = cols / group_size;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        for (int64_t gg = 0; gg < ng; gg++) {
            double mn = src[r * cols + gg * group_size];
            double mx = mn;
            for (int64_t c = 1; c < group_size; c++) {
                const double v = src[r * cols + gg * group_size + c];
                if (v < mn) mn = v;
                if (v > mx) mx = v;
            }
            if (mx - mn < 0.00000001) mx = mn + 0.00000001;
            double sc = (mx - mn) / 15.0;
            int64_t zp = net_round_to_i64(-mn / sc);
            if (zp < 0) zp = 0;
            if (zp > 15) zp = 15;
            if (zp == 0) {
                if (mn > 0) {
                    sc = mx / 15.0;
                    if (sc < 0.00000001) sc = 0.00000001;
                    zp = 0;
                }
            } else if (zp == 15) {
                sc = -mn / 15.0;
            }
            if (sc < 0.00000001) sc = 0.00000001;
            scales[r * ng + gg] = (float)sc;
            zps[r * ng + gg] = zp;
        }
        for (int64_t c = 0; c < cols; c += 2) {
            const int64_t gg = c / group_size;
            const double sc = scales[r * ng + gg];
            const int64_t zp = zps[r * ng + gg];
            const double mn = (double)(-zp) * sc;
            const int64_t q0 = clamp_i64(net_round_to_i64(((double)src[r * cols + c] - mn) / sc), 0, 15);
            const int64_t q1 = clamp_i64(net_round_to_i64(((double)src[r * cols + c + 1] - mn) / sc), 0, 15);
            packed[r * (cols / 2) + c / 2] = (uint8_t)((q1 << 4) | q0);
        }
    }
    return 0;
}

/* dequantize_int4_grouped_asym, int4.tkv:153-164: fl32((nib - zp) * s). */
TVO_API int tvo_dequantize_int4_grouped_asym(const uint8_t* packed, float* dst, int64_t rows, int64_t cols,
                                             int64_t group_size, const float* scales, const int64_t* zps) {
    if (group_size <= 0 || cols % group_size != 0 || cols % 2 != 0) return -1;
    const int64_t ng = cols / group_size;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c += 2) {
            const double sc = scales[r * ng + c / group_size];
            const int64_t zp = zps[r * ng + c / group_size];
            const int b = packed[r * (cols / 2) + c / 2];
            dst[r * cols + c] = (float)((double)((b & 0xF) - zp) * sc);
            dst[r * cols + c + 1] = (float)((double)(((b >> 4) & 0xF) - zp) * sc);
        }
    return 0;
}

/* permute_cols / inv_permute_cols, int4.tkv:169-184: out[r, c] = src[r,
 * perm[c]] / out[r, perm[c]] = src[r, c].  -1 for an index out of range. */
TVO_API int tvo_permute_cols(const float* src, float* out, int64_t rows, int64_t cols, const int64_t* perm,
                             int inverse) {
    for (int64_t c = 0; c < cols; c++)
        if (perm[c] < 0 || perm[c] >= cols) return -1;
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++)
        for (int64_t c = 0; c < cols; c++) {
            if (inverse) out[r * cols + perm[c]] = src[r * cols + c];
            else out[r * cols + c] = src[r * cols + perm[c]];
        }
    return 0;
}

/* matmul_int4_grouped (int4.tkv:213-239) and, with perm, the act-order
 * matmul_int4_grouped_ordered (:187-208): y[m, n] = fl32(sum_k a[m, perm[k]]
 * * fl64((nib - 8) * s[n, k / gs]) + bias[n]) with a sequential f64 sum (the
 * products are exact in f64: 24 + 28 significant bits). */
TVO_API int tvo_matmul_int4_grouped(const float* A, const uint8_t* packed, const float* bias, int64_t n_bias,
                                    float* Y, int64_t m, int64_t n, int64_t k, int64_t group_size,
                                    const float* scales, const int64_t* perm) {
    if (group_size <= 0 || k % group_size != 0 || k % 2 != 0) return -1;
    const int64_t ng = k / group_size;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) {
            double acc = 0.0;
            for (int64_t kk = 0; kk < k; kk++) {
                const int b = packed[j * (k / 2) + kk / 2];
                const int nib = (kk % 2 == 0) ? (b & 0xF) : ((b >> 4) & 0xF);
                const double w = (double)(nib - 8) * (double)scales[j * ng + kk / group_size];
                const double a = A[i * k + (perm ? perm[kk] : kk)];
                acc = acc + a * w;
            }
            const double bb = n_bias > 0 ? (double)bias[j] : 0.0;
            Y[i * n + j] = (float)(acc + bb);
        }
    return 0;
}
