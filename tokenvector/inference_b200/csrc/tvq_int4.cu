// tvq_int4.cu -- group-wise INT4 weights (tv/quantization/int4.tkv) on the GPU.
//
// Layout as in the reference: weights [rows, cols] -> packed bytes [rows,
// cols / 2] (two nibbles per byte, low nibble first) + scales [rows, cols /
// group_size] (+ zero points for the AWQ-style asymmetric form).  The codecs
// below reproduce the reference's f64 arithmetic exactly (the symmetric
// quantize through the exact x * (1 / s) rounding of tvq_exact.cuh, the
// per-group statistics and the asymmetric quotient in f64, once per group or
// element); the grouped GEMM runs on the tensor cores as GEMM_W4 (tvq_gemm.cu)
// on the weights unpacked to their integer values in fp16 and the
// activations split into fp16 hi / lo under power-of-two row scales
// (launch_split_f16_rows), optionally gathered by the act-order permutation.
#include <cuda_fp16.h>

#include <algorithm>

#include "tvq_common.cuh"
#include "tvq_exact.cuh"
#include "tvq_kernels.h"

namespace tvq {

namespace {

// quantize_int4_grouped, int4.tkv:27-48 with _int4_scales_sym :18-29: thread
// per (row, group).  scale = fl32(max(max|x|, 1e-8) / 7) (f64 quotient);
// q = clamp(round(x * (1.0 / scale)), -8, 7) + 8, exactly as the f64 product.
__global__ void int4_quantize_sym_kernel(const float* __restrict__ src, int64_t rows, int64_t cols, int64_t gs,
                                         uint8_t* __restrict__ packed, float* __restrict__ scales) {
    griddep_wait();
    const int64_t ng = cols / gs;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < rows * ng;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / ng, g = t - r * ng;
        const float* x = src + r * cols + g * gs;
        float am = 0.0f;  // max |x| is exact in f32
        for (int64_t c = 0; c < gs; c++) am = fmaxf(am, fabsf(x[c]));
        double a = am;
        if (a < 0.00000001) a = 0.00000001;
        const float sc = __double2float_rn(a / 7.0);
        scales[t] = sc;
        const InvScale qs = make_inv_scale(static_cast<double>(sc));
        uint8_t* out = packed + r * (cols / 2) + g * gs / 2;
        for (int64_t c = 0; c < gs; c += 2) {
            const int q0 = min(max(static_cast<int>(quant_exact(x[c], qs)), -8), 7) + 8;
            const int q1 = min(max(static_cast<int>(quant_exact(x[c + 1], qs)), -8), 7) + 8;
            out[c / 2] = static_cast<uint8_t>((q1 << 4) | q0);
        }
    }
}

// dequantize_int4_grouped, int4.tkv:51-64: fl32((nib - 8) * s), one rounding
// of an exact product.
__global__ void int4_dequantize_kernel(const uint8_t* __restrict__ packed, float* __restrict__ dst, int64_t rows,
                                       int64_t cols, int64_t gs, const float* __restrict__ scales,
                                       const int64_t* __restrict__ zps) {
    griddep_wait();
    const int64_t ng = cols / gs, half = cols / 2;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * half;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / half, c = 2 * (i - r * half);
        const int64_t gi = r * ng + c / gs;
        const float sc = __ldg(scales + gi);
        const int zp = zps ? static_cast<int>(__ldg(zps + gi)) : 8;
        const int b = packed[i];
        float2 v;
        v.x = __fmul_rn(static_cast<float>((b & 0xF) - zp), sc);
        v.y = __fmul_rn(static_cast<float>(((b >> 4) & 0xF) - zp), sc);
        *reinterpret_cast<float2*>(dst + r * cols + c) = v;
    }
}

// quantize_int4_grouped_asym, int4.tkv:68-150: thread per (row, group), the
// reference's f64 statistics and corrections, then q = clamp(round((x -
// mn) / s), 0, 15) with mn = -zp * s in f64 (the stored f32 scale).
__global__ void int4_quantize_asym_kernel(const float* __restrict__ src, int64_t rows, int64_t cols, int64_t gs,
                                          uint8_t* __restrict__ packed, float* __restrict__ scales,
                                          int64_t* __restrict__ zps) {
    griddep_wait();
    const int64_t ng = cols / gs;
    for (int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; t < rows * ng;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / ng, g = t - r * ng;
        const float* x = src + r * cols + g * gs;
        float fmn = x[0], fmx = x[0];
        for (int64_t c = 1; c < gs; c++) {  // the comparison chain of the reference (NaN compares false)
            if (x[c] < fmn) fmn = x[c];
            if (x[c] > fmx) fmx = x[c];
        }
        double mn = fmn, mx = fmx;
        if (mx - mn < 0.00000001) mx = mn + 0.00000001;
        double sc = (mx - mn) / 15.0;
        double zr = rint(-mn / sc);
        int64_t zp = (zr != zr) ? 0 : static_cast<int64_t>(fmin(fmax(zr, -1.0), 16.0));
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
        const float scf = __double2float_rn(sc);
        scales[t] = scf;
        zps[t] = zp;
        const double sd = scf;
        const double mnq = static_cast<double>(-zp) * sd;
        uint8_t* out = packed + r * (cols / 2) + g * gs / 2;
        for (int64_t c = 0; c < gs; c += 2) {
            int q[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const double v = rint((static_cast<double>(x[c + h]) - mnq) / sd);
                q[h] = (v != v) ? 0 : static_cast<int>(fmin(fmax(v, 0.0), 15.0));
            }
            out[c / 2] = static_cast<uint8_t>((q[1] << 4) | q[0]);
        }
    }
}

// permute_cols / inv_permute_cols, int4.tkv:169-184.  An index out of range
// (the reference's IndexError) records an error and is skipped.
__global__ void permute_cols_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t rows,
                                    int64_t cols, const int64_t* __restrict__ perm, int inverse, int* err) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * cols;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / cols, c = i - r * cols;
        const int64_t pc = __ldg(perm + c);
        if (pc < 0 || pc >= cols) {
            record_error(err, DEVERR_BAD_INDEX);
            continue;
        }
        if (inverse) dst[r * cols + pc] = src[i];
        else dst[i] = src[r * cols + pc];
    }
}

// packed [n, k / 2] -> the signed integer values nib - 8 in fp16 [n, k]
// (exact): GEMM_W4's B operand.
__global__ void int4_unpack_f16_kernel(const uint8_t* __restrict__ packed, __half2* __restrict__ q, int64_t count) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
        const int b = packed[i];
        q[i] = __halves2half2(__int2half_rn((b & 0xF) - 8), __int2half_rn(((b >> 4) & 0xF) - 8));
    }
}

int grid1d(int64_t work, int threads, DeviceState* ds) {
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((work + threads - 1) / threads, ds->sm_count * 8)));
}

}  // namespace

int launch_int4_quantize(const float* src, int64_t rows, int64_t cols, int64_t gs, uint8_t* packed, float* scales,
                         int64_t* zps, cudaStream_t st) {
    TVQ_CHECK(gs > 0 && cols % gs == 0 && cols % 2 == 0, TVQ_ERR_SIZE,
              "cols must be a multiple of group_size and even");  // int4.tkv:28-31
    if (rows <= 0 || cols <= 0) return TVQ_OK;
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    const int64_t work = rows * (cols / gs);
    if (zps)
        return launch_pdl(int4_quantize_asym_kernel, dim3(grid1d(work, 128, ds)), dim3(128), 0, st, src, rows, cols, gs,
                          packed, scales, zps);
    return launch_pdl(int4_quantize_sym_kernel, dim3(grid1d(work, 128, ds)), dim3(128), 0, st, src, rows, cols, gs,
                      packed, scales);
}

int launch_int4_dequantize(const uint8_t* packed, float* dst, int64_t rows, int64_t cols, int64_t gs,
                           const float* scales, const int64_t* zps, cudaStream_t st) {
    TVQ_CHECK(gs > 0 && cols % gs == 0 && cols % 2 == 0, TVQ_ERR_SIZE,
              "cols must be a multiple of group_size and even");
    if (rows <= 0 || cols <= 0) return TVQ_OK;
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    TVQ_CHECK((reinterpret_cast<uintptr_t>(dst) & 7) == 0, TVQ_ERR_UNSUPPORTED, "dst must be 8-byte aligned");
    return launch_pdl(int4_dequantize_kernel, dim3(grid1d(rows * cols / 2, 256, ds)), dim3(256), 0, st, packed, dst,
                      rows, cols, gs, scales, zps);
}

int launch_permute_cols(const float* src, float* dst, int64_t rows, int64_t cols, const int64_t* perm, int inverse,
                        cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return TVQ_OK;
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    return launch_pdl(permute_cols_kernel, dim3(grid1d(rows * cols, 256, ds)), dim3(256), 0, st, src, dst, rows, cols,
                      perm, inverse, ds->d_error);
}

int launch_int4_unpack_f16(const uint8_t* packed, void* q, int64_t n, int64_t k, cudaStream_t st) {
    if (n <= 0 || k <= 0) return TVQ_OK;
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    TVQ_CHECK((reinterpret_cast<uintptr_t>(q) & 3) == 0 && k % 2 == 0, TVQ_ERR_UNSUPPORTED,
              "unpacked weights must be 4-byte aligned, k even");
    const int64_t count = n * k / 2;
    return launch_pdl(int4_unpack_f16_kernel, dim3(grid1d(count, 256, ds)), dim3(256), 0, st, packed,
                      static_cast<__half2*>(q), count);
}

}  // namespace tvq
