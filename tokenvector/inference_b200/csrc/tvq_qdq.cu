// tvq_qdq.cu -- the ONNX QDQ operator family of the reference runtime on the
// GPU: QuantizeLinear, DequantizeLinear, MatMulInteger, QLinearMatMul and
// DynamicQuantizeLinear (tv/runtime/session.tkv:1896-2071, 2789-2905).
//
// Same numeric model as the rest of libtvq: the reference evaluates in
// binary64 and rounds to binary32 only at typed stores; round is half to even
// and int() saturates with NaN -> 0.  Quotients x / s are decided in binary32
// with a proof that the binary64 quotient rounds to the same integer (its
// distance to the nearest half-integer exceeds both rounding errors), and fall
// back to binary64 otherwise; products acc * mult are evaluated as float
// expansions with the same kind of proof.  MatMulInteger and the integer part
// of QLinearMatMul run on the tcgen05 INT8 GEMM (exact int32 accumulators):
// B [K, N] is transposed to the K-major [N, K] operand first; QLinearMatMul's
// zero points enter through row sums of A and column sums of B.
#include <algorithm>
#include <cmath>

#include "tvq_common.cuh"
#include "tvq_exact.cuh"
#include "tvq_kernels.h"

namespace tvq {

namespace {

// int(round(v)) of the reference (half to even, saturating, NaN -> 0), int64.
__device__ __forceinline__ long long net_round_i64(double v) {
    if (v != v) return 0;
    const double r = rint(v);
    if (r >= 9.2233720368547758e18) return 0x7FFFFFFFFFFFFFFFll;
    if (r <= -9.2233720368547758e18) return static_cast<long long>(0x8000000000000000ull);
    return static_cast<long long>(r);
}

static __device__ __noinline__ long long qdiv_slow(float x, double s) { return net_round_i64(static_cast<double>(x) / s); }

// int(round(fl64(x / s))) for s > 0.  Fast path: r = fl32(x / sf) with sf =
// fl32(s) (|sf / s - 1| <= 2^-24): |r - x/s| <= 2^-22.9 |r|, and fl64(x/s) is
// within 2^-53 of x/s, so both round to rint(r) whenever r is farther than
// 2^-21 |r| from a half-integer (and |r| < 2^21, below which such a distance
// exists).  NaN, Inf and the rest go through binary64.
__device__ __forceinline__ long long qdiv(float x, double s, float sf) {
    const float r = __fdiv_rn(x, sf);
    const float ar = fabsf(r);
    if (ar < 2097152.0f) {
        const float k = rintf(r);
        const float h = fabsf(fabsf(r - k) - 0.5f);  // distance to the nearest half-integer
        if (h > ar * 4.76837158203125e-07f + 1e-30f) return static_cast<long long>(k);
    }
    return qdiv_slow(x, s);
}

__device__ __forceinline__ int8_t sat_i8(long long q, long long zp) {
    // q + zp without overflowing at the saturated ends, then [-128, 127]
    if (q > 0x7FFFFFFFFFFFFF00ll || q < -0x7FFFFFFFFFFFFF00ll) return q > 0 ? 127 : -128;
    const long long v = q + zp;
    return static_cast<int8_t>(v < -128 ? -128 : (v > 127 ? 127 : v));
}

// _exec_quantize_linear, session.tkv:1896-1953.  nsc == 1: per tensor, else
// channel (i / inner) % dim.  s = sc > 1e-12 ? sc : 1e-12 (a double).
__global__ void quantize_linear_kernel(const float* __restrict__ x, int8_t* __restrict__ y, int64_t n, int64_t dim,
                                       int64_t inner, const float* __restrict__ sc, int nsc, long long zp) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float sf0 = __ldg(sc + (nsc == 1 ? 0 : (i / inner) % dim));
        const bool floor = !(static_cast<double>(sf0) > 0.000000000001);
        const double s = floor ? 0.000000000001 : static_cast<double>(sf0);
        const long long q = floor ? qdiv_slow(x[i], s) : qdiv(x[i], s, sf0);
        y[i] = sat_i8(q, zp);
    }
}

// _exec_dequantize_linear, session.tkv:1955-1990: y = fl32((x - zp) * sc).
// For |x - zp| < 2^24 both factors are exact binary32 values and the binary64
// product is exact, so its rounding to f32 is the correctly rounded f32
// product.
__global__ void dequantize_linear_kernel(const int8_t* __restrict__ x, float* __restrict__ y, int64_t n, int64_t dim,
                                         int64_t inner, const float* __restrict__ sc, int nsc, long long zp) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float s = __ldg(sc + (nsc == 1 ? 0 : (i / inner) % dim));
        const long long v = static_cast<long long>(x[i]) - zp;
        y[i] = (v > -16777216ll && v < 16777216ll)
                   ? __fmul_rn(static_cast<float>(v), s)
                   : __double2float_rn(static_cast<double>(v) * static_cast<double>(s));
    }
}

// [rows, cols] int8 -> [cols, ld] int8 (transposed, rows padded with zeros
// up to ld), 32 x 32 tiles.
__global__ void transpose_i8_kernel(const int8_t* __restrict__ a, int8_t* __restrict__ b, int rows, int cols,
                                    int ld) {
    griddep_wait();
    __shared__ int8_t tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        tile[i][threadIdx.x] = (r < rows && c < cols) ? a[static_cast<int64_t>(r) * cols + c] : 0;
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int oc = c0 + i;           // output row = input column
        const int orr = r0 + threadIdx.x; // output column = input row
        if (oc < cols && orr < ld) b[static_cast<int64_t>(oc) * ld + orr] = tile[threadIdx.x][i];
    }
}

// [rows, cols] int8 -> [rows, ld] int8 (zero-padded columns)
__global__ void pad_i8_kernel(const int8_t* __restrict__ a, int8_t* __restrict__ b, int64_t rows, int cols, int ld) {
    griddep_wait();
    const int64_t n = rows * ld;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / ld;
        const int c = static_cast<int>(i - r * ld);
        b[i] = c < cols ? a[r * cols + c] : 0;
    }
}

// sum over k of A[i, k] (one warp per row) and of B[k, j] (one thread per column)
__global__ void row_sums_i8_kernel(const int8_t* __restrict__ a, int64_t rows, int k, int* __restrict__ out) {
    griddep_wait();
    const int64_t r = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    int s = 0;
    for (int c = lane; c < k; c += 32) s += a[r * k + c];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) out[r] = s;
}

__global__ void col_sums_i8_kernel(const int8_t* __restrict__ b, int k, int64_t n, int* __restrict__ out) {
    griddep_wait();
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= n) return;
    int s = 0;
    for (int p = 0; p < k; p++) s += b[static_cast<int64_t>(p) * n + j];
    out[j] = s;
}

static __device__ __noinline__ long long qmul_slow(long long acc, double mult) {
    return net_round_i64(static_cast<double>(acc) * mult);
}

// _exec_qlinear_matmul's requantization, session.tkv:2050-2071:
// acc' = sum (a - zpa)(b - zpw) = acc - zpw rowA[i] - zpa colB[j] + k zpa zpw,
// y = clamp(int(round(acc' * mult)) + zpy, -128, 127) with mult = sa sw / sy
// in binary64 (passed as a float pair mh + ml, |mh + ml - mult| <= 2^-48 mult).
__global__ void qlinear_requant_kernel(const int32_t* __restrict__ acc, const int* __restrict__ rowA,
                                       const int* __restrict__ colB, int64_t m, int64_t n, int k, long long zpa,
                                       long long zpw, long long zpy, double mult, float mh, float ml,
                                       int8_t* __restrict__ y) {
    griddep_wait();
    const int64_t total = m * n;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / n, c = i - r * n;
        const long long a = static_cast<long long>(acc[i]) - zpw * rowA[r] - zpa * colB[c] +
                            static_cast<long long>(k) * zpa * zpw;
        long long q;
        const long long absa = a < 0 ? -a : a;
        if (absa < (1ll << 48)) {
            // a = ah + ar exactly (ah has 24 bits, |ar| < 2^25), then
            // a * (mh + ml) as p1 + (e1 + cross terms): relative error ~2^-44
            const float ah = static_cast<float>(a);
            const float ar = static_cast<float>(a - static_cast<long long>(ah));
            const float p1 = __fmul_rn(ah, mh);
            float pl = fmaf(ah, mh, -p1);
            pl = fmaf(ah, ml, pl);
            pl = fmaf(ar, mh, pl);
            pl = fmaf(ar, ml, pl);
            const float v = __fadd_rn(p1, pl);
            const float av = fabsf(v);
            q = 0;
            bool ok = false;
            if (av < 2097152.0f) {
                const float kf = rintf(v);
                // distance of p1 + pl to the half-integer nearest kf, in two parts
                const float hb = (v >= kf) ? kf + 0.5f : kf - 0.5f;
                const float d = fabsf(__fadd_rn(__fsub_rn(p1, hb), pl));
                if (d > av * 9.094947017729282e-13f * 64.0f + 1e-30f) {
                    q = static_cast<long long>(kf);
                    ok = true;
                }
            }
            if (!ok) q = qmul_slow(a, mult);
        } else {
            q = qmul_slow(a, mult);
        }
        y[i] = sat_i8(q, zpy);
    }
}

// DynamicQuantizeLinear finalize: from the running min / max (ordinal
// encoded) and x[0]: mn, mx include 0, range >= 1e-8, sc = (mx - mn) / 255
// (f64, kept for the quantize pass), zp = clamp(int(round(-mn / sc)), 0, 255).
__device__ __forceinline__ float ord2f_q(uint32_t u) {
    const uint32_t b = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    return __uint_as_float(b);
}

__global__ void dynq_finalize_kernel(const uint32_t* mm, const float* first, double* sc_out, long long* zp_out,
                                     float* y_scale, float* y_zp) {
    griddep_wait();
    double mn, mx;
    if (*first != *first) {  // x[0] NaN: no comparison ever replaces it
        mn = mx = __longlong_as_double(0x7FF8000000000000ll);
    } else {
        mn = ord2f_q(mm[0]);
        mx = ord2f_q(mm[1]);
    }
    if (mn > 0.0) mn = 0.0;
    if (mx < 0.0) mx = 0.0;
    if (mx - mn < 0.00000001) mx = mn + 0.00000001;
    const double sc = (mx - mn) / 255.0;
    long long zp = net_round_i64(-mn / sc);
    zp = zp < 0 ? 0 : (zp > 255 ? 255 : zp);
    *sc_out = sc;
    *zp_out = zp;
    *y_scale = __double2float_rn(sc);
    *y_zp = static_cast<float>(zp);
}

__global__ void dynq_quantize_kernel(const float* __restrict__ x, int64_t n, const double* __restrict__ sc_p,
                                     const long long* __restrict__ zp_p, int8_t* __restrict__ y) {
    griddep_wait();
    const double sc = *sc_p;
    const long long zp = *zp_p;
    const float sf = __double2float_rn(sc);
    const bool fast = sf > 0.0f && sf < 3.0e38f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const long long q0 = fast ? qdiv(x[i], sc, sf) : qdiv_slow(x[i], sc);
        long long q;
        if (q0 > 0x7FFFFFFFFFFFFF00ll || q0 < -0x7FFFFFFFFFFFFF00ll) q = q0 > 0 ? 255 : 0;
        else q = q0 + zp;
        q = q < 0 ? 0 : (q > 255 ? 255 : q);
        y[i] = static_cast<int8_t>(q - 128);
    }
}

int grid_1d(int64_t n, int threads) {
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    const int64_t cap = static_cast<int64_t>(ds ? ds->sm_count : 148) * 8;
    const int64_t want = (n + threads - 1) / threads;
    return static_cast<int>(std::max<int64_t>(1, std::min(want, cap)));
}

}  // namespace

int launch_row_sums_i8(const int8_t* a, int64_t rows, int64_t k, int* out, cudaStream_t st) {
    TVQ_CHECK(rows >= 0 && k >= 0 && k < (1ll << 31), TVQ_ERR_INVALID, "bad row-sum size");
    if (rows == 0) return TVQ_OK;
    if (k == 0) {
        TVQ_CUDA(cudaMemsetAsync(out, 0, sizeof(int) * rows, st));
        return TVQ_OK;
    }
    return launch_pdl(row_sums_i8_kernel, dim3(static_cast<unsigned>((rows * 32 + 255) / 256)), dim3(256), 0, st, a,
                      rows, static_cast<int>(k), out);
}

int launch_quantize_linear(const float* x, int8_t* y, int64_t outer, int64_t dim, int64_t inner, const float* scales,
                           int64_t nsc, int64_t zp, cudaStream_t st) {
    const int64_t n = outer * dim * inner;
    TVQ_CHECK(outer >= 0 && dim >= 0 && inner >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(nsc == 1 || nsc == dim, TVQ_ERR_SIZE, "need one scale or one per channel of the axis");
    if (n == 0) return TVQ_OK;
    return launch_pdl(quantize_linear_kernel, dim3(grid_1d(n, 256)), dim3(256), 0, st, x, y, n, dim, inner, scales,
                      static_cast<int>(nsc), static_cast<long long>(zp));
}

int launch_dequantize_linear(const int8_t* x, float* y, int64_t outer, int64_t dim, int64_t inner,
                             const float* scales, int64_t nsc, int64_t zp, cudaStream_t st) {
    const int64_t n = outer * dim * inner;
    TVQ_CHECK(outer >= 0 && dim >= 0 && inner >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(nsc == 1 || nsc == dim, TVQ_ERR_SIZE, "need one scale or one per channel of the axis");
    if (n == 0) return TVQ_OK;
    return launch_pdl(dequantize_linear_kernel, dim3(grid_1d(n, 256)), dim3(256), 0, st, x, y, n, dim, inner, scales,
                      static_cast<int>(nsc), static_cast<long long>(zp));
}

// Scratch of one MatMulInteger: A padded [m, kp] (when k % 16 != 0) and
// B^T [n, kp], stream-ordered, freed by the caller with cudaFreeAsync.
static int gemm_operands(const int8_t* a, const int8_t* b, int64_t m, int64_t k, int64_t n, cudaStream_t st,
                         int8_t** base, const int8_t** ap, const int8_t** btp, int64_t* kp_out) {
    const int64_t kp = (k + 15) / 16 * 16;
    const bool pad_a = kp != k;
    const size_t bytes = static_cast<size_t>(n) * kp + (pad_a ? static_cast<size_t>(m) * kp : 0) + 256;
    int8_t* buf = nullptr;
    TVQ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&buf), bytes, st));
    int8_t* bt = buf;
    int8_t* apad = buf + ((static_cast<size_t>(n) * kp + 255) / 256 * 256);
    int rc = launch_pdl(transpose_i8_kernel, dim3(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>((kp + 31) / 32)),
                        dim3(32, 8), 0, st, b, bt, static_cast<int>(k), static_cast<int>(n), static_cast<int>(kp));
    if (!rc && pad_a)
        rc = launch_pdl(pad_i8_kernel, dim3(grid_1d(m * kp, 256)), dim3(256), 0, st, a, apad, m, static_cast<int>(k),
                        static_cast<int>(kp));
    *base = buf;
    *ap = pad_a ? apad : a;
    *btp = bt;
    *kp_out = kp;
    return rc;
}

int launch_matmul_integer(const int8_t* a, const int8_t* b, int32_t* y, int64_t m, int64_t k, int64_t n,
                          cudaStream_t st) {
    TVQ_CHECK(m >= 0 && k >= 0 && n >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(m < (1ll << 31) && n < (1ll << 31) && k < 133143, TVQ_ERR_UNSUPPORTED, "size out of range");
    if (m == 0 || n == 0) return TVQ_OK;
    if (k == 0) {
        TVQ_CUDA(cudaMemsetAsync(y, 0, sizeof(int32_t) * m * n, st));
        return TVQ_OK;
    }
    int8_t* buf = nullptr;
    const int8_t *ap = nullptr, *bt = nullptr;
    int64_t kp = 0;
    int rc = gemm_operands(a, b, m, k, n, st, &buf, &ap, &bt, &kp);
    if (!rc) {
        GemmArgs g;
        g.kind = GEMM_I8;
        g.A = ap;
        g.W = bt;
        g.acc_out = y;
        g.m = m;
        g.n = n;
        g.k = kp;
        rc = launch_gemm(g, st);
    }
    cudaError_t e = cudaFreeAsync(buf, st);
    if (!rc && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return rc;
}

int launch_qlinear_matmul(const int8_t* a, float sa, int64_t zpa, const int8_t* b, float sw, int64_t zpw, float sy,
                          int64_t zpy, int8_t* y, int64_t m, int64_t k, int64_t n, cudaStream_t st) {
    TVQ_CHECK(m >= 0 && k >= 0 && n >= 0, TVQ_ERR_INVALID, "negative size");
    TVQ_CHECK(m < (1ll << 31) && n < (1ll << 31) && k < 133143, TVQ_ERR_UNSUPPORTED, "size out of range");
    if (m == 0 || n == 0) return TVQ_OK;
    // int32 accumulators + row / column sums, stream-ordered scratch
    const size_t acc_bytes = (static_cast<size_t>(m) * n * 4 + 255) / 256 * 256;
    const size_t sums_bytes = (static_cast<size_t>(m + n) * 4 + 255) / 256 * 256;
    char* scratch = nullptr;
    TVQ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&scratch), acc_bytes + sums_bytes, st));
    int32_t* acc = reinterpret_cast<int32_t*>(scratch);
    int* rowA = reinterpret_cast<int*>(scratch + acc_bytes);
    int* colB = rowA + m;
    int rc = launch_matmul_integer(a, b, acc, m, k, n, st);
    if (!rc && k > 0)
        rc = launch_pdl(row_sums_i8_kernel, dim3(static_cast<unsigned>((m * 32 + 255) / 256)), dim3(256), 0, st, a, m,
                        static_cast<int>(k), rowA);
    if (!rc && k > 0)
        rc = launch_pdl(col_sums_i8_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, st, b,
                        static_cast<int>(k), n, colB);
    if (!rc && k == 0) {
        cudaError_t e2 = cudaMemsetAsync(rowA, 0, sizeof(int) * (m + n), st);
        if (e2 != cudaSuccess) rc = cuda_fail(e2, "cudaMemsetAsync");
    }
    if (!rc) {
        const double syd = (static_cast<double>(sy) == 0.0) ? 1.0 : static_cast<double>(sy);
        const double mult = static_cast<double>(sa) * static_cast<double>(sw) / syd;
        const float mh = static_cast<float>(mult);
        const float ml = static_cast<float>(mult - static_cast<double>(mh));
        rc = launch_pdl(qlinear_requant_kernel, dim3(grid_1d(m * n, 256)), dim3(256), 0, st,
                        static_cast<const int32_t*>(acc), static_cast<const int*>(rowA), static_cast<const int*>(colB),
                        m, n, static_cast<int>(k), static_cast<long long>(zpa), static_cast<long long>(zpw),
                        static_cast<long long>(zpy), mult, mh, ml, y);
    }
    cudaError_t e = cudaFreeAsync(scratch, st);
    if (!rc && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return rc;
}

int launch_dynamic_quantize_linear(const float* x, int64_t n, int8_t* y, float* y_scale, float* y_zp,
                                   cudaStream_t st) {
    TVQ_CHECK(n >= 1, TVQ_ERR_SIZE, "DynamicQuantizeLinear needs at least one element");
    // scratch: min/max ordinals, x[0], the f64 scale and the zero point
    char* s = nullptr;
    TVQ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&s), 64, st));
    uint32_t* mm = reinterpret_cast<uint32_t*>(s);
    float* first = reinterpret_cast<float*>(s + 8);
    double* sc = reinterpret_cast<double*>(s + 16);
    long long* zp = reinterpret_cast<long long*>(s + 24);
    int rc = launch_minmax_reset(mm, st);
    if (!rc) rc = launch_minmax_accumulate(x, n, mm, first, st);
    if (!rc) rc = launch_pdl(dynq_finalize_kernel, dim3(1), dim3(1), 0, st, static_cast<const uint32_t*>(mm),
                             static_cast<const float*>(first), sc, zp, y_scale, y_zp);
    if (!rc) rc = launch_pdl(dynq_quantize_kernel, dim3(grid_1d(n, 256)), dim3(256), 0, st, x, n,
                             static_cast<const double*>(sc), static_cast<const long long*>(zp), y);
    cudaError_t e = cudaFreeAsync(s, st);
    if (!rc && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return rc;
}

}  // namespace tvq
