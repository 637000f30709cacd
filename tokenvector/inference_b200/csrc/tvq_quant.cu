// tvq_quant.cu -- HBM-bound PTQ kernels: min/max calibration, INT8
// quantize/dequantize, FP8-E4M3 encode/decode.
//
// Each kernel restates one function of tv/quantization (paths relative to the
// TokenVector.Inference repository) with the reference compiler's numeric
// model: scale arithmetic in binary64, round half to even (Math.Round), int()
// saturating with NaN -> 0, rounding to binary32 only at typed stores.  The
// per-element binary64 expressions are evaluated exactly with binary32
// arithmetic and a rare binary64 slow path (tvq_exact.cuh): FP64 on the CUDA
// cores is far too slow on B200 to keep up with HBM.
//
// Layout: 16-byte vector loads/stores where the pointers allow it, grid-
// stride loops over grids sized to a multiple of the SM count, warp-shuffle +
// shared-memory reductions, one atomic per block.
#include <cuda_fp8.h>

#include <algorithm>
#include <cstring>

#include "tvq_common.cuh"
#include "tvq_e4m3.h"
#include "tvq_f16.h"
#include "tvq_exact.cuh"
#include "tvq_kernels.h"

namespace tvq {

// ------------------------------------------------------------ helpers

// Order-preserving map float -> uint32 (for atomicMin/atomicMax of floats).
__device__ __forceinline__ uint32_t f2ord(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t u) {
    uint32_t b = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    return __uint_as_float(b);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

static int grid_for(int64_t work_items, int threads, int per_sm) {
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    int sms = ds ? ds->sm_count : 148;
    int64_t want = (work_items + threads - 1) / threads;
    int64_t cap = static_cast<int64_t>(sms) * per_sm;
    if (want < 1) want = 1;
    return static_cast<int>(want < cap ? want : cap);
}

// ------------------------------------------------------------ K1: min / max
// calibrate_minmax, tv/quantization/engine.tkv:13-36: the running min and max
// with `<` / `>` comparisons, so NaN elements never win; NaN in data[0] is
// handled in the finalize step (it poisons the comparison chain there).
__global__ void minmax_kernel(const float* __restrict__ x, int64_t n, uint32_t* __restrict__ mm) {
    float lo = INFINITY, hi = -INFINITY;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    int64_t n4 = vec ? n / 4 : 0;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int64_t i = tid; i < n4; i += stride) {
        float4 v = __ldcs(x4 + i);
        lo = fminf(lo, fminf(fminf(v.x, v.y), fminf(v.z, v.w)));
        hi = fmaxf(hi, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
    for (int64_t i = n4 * 4 + tid; i < n; i += stride) {
        float v = x[i];
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
    }
    lo = warp_min(lo);
    hi = warp_max(hi);
    __shared__ float slo[32], shi[32];
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) { slo[w] = lo; shi[w] = hi; }
    __syncthreads();
    if (w == 0) {
        const int nw = blockDim.x >> 5;
        lo = (l < nw) ? slo[l] : INFINITY;
        hi = (l < nw) ? shi[l] : -INFINITY;
        lo = warp_min(lo);
        hi = warp_max(hi);
        if (l == 0) {
            if (lo == lo && lo != INFINITY) atomicMin(mm + 0, f2ord(lo));
            if (hi == hi && hi != -INFINITY) atomicMax(mm + 1, f2ord(hi));
            // +/-Inf elements are values, not "nothing seen": record them.
            if (lo == INFINITY && hi == INFINITY) { atomicMin(mm + 0, f2ord(lo)); atomicMax(mm + 1, f2ord(hi)); }
            if (lo == -INFINITY && hi == -INFINITY) { atomicMin(mm + 0, f2ord(lo)); atomicMax(mm + 1, f2ord(hi)); }
        }
    }
}

__global__ void minmax_reset_kernel(uint32_t* mm) {
    mm[0] = 0xFFFFFFFFu;  // above every non-NaN ordinal
    mm[1] = 0u;
}

__global__ void copy_first_kernel(const float* x, float* first) { *first = x[0]; }

// QuantParams from a min and max, exactly as engine.tkv:24-36 in f64 with f32
// field stores.  params = {scale, zero_point, min, max}.
__device__ __forceinline__ void params_from_minmax(double mn, double mx, int symmetric, float* params) {
    if (symmetric) {
        double am = fabs(mx);
        if (fabs(mn) > am) am = fabs(mn);
        if (am < 0.00000001) am = 0.00000001;
        params[0] = __double2float_rn(am / 127.0);
        params[1] = 0.0f;
        params[2] = __double2float_rn(-am);
        params[3] = __double2float_rn(am);
        return;
    }
    if (fabs(mx - mn) < 0.00000001) mx = mn + 0.00000001;
    double scale = (mx - mn) / 255.0;
    double z = -mn / scale;
    long long zp = (z != z) ? 0 : static_cast<long long>(rint(fmin(fmax(z, -1e18), 1e18)));
    zp -= 128;
    zp = zp < -128 ? -128 : (zp > 127 ? 127 : zp);
    params[0] = __double2float_rn(scale);
    params[1] = static_cast<float>(zp);
    params[2] = __double2float_rn(mn);
    params[3] = __double2float_rn(mx);
}

// QuantParams from the accumulated min/max (engine.tkv:13-36).
__global__ void minmax_finalize_kernel(const uint32_t* mm, const float* first, int symmetric, float* params) {
    double mn, mx;
    const bool poisoned = first && (*first != *first);
    if (poisoned) {
        mn = mx = __longlong_as_double(0x7FF8000000000000ll);
    } else if (mm[0] == 0xFFFFFFFFu && mm[1] == 0u) {
        // nothing but NaNs after data[0]: cannot happen with data[0] finite
        mn = mx = 0.0;
    } else {
        mn = ord2f(mm[0]);
        mx = ord2f(mm[1]);
    }
    params_from_minmax(mn, mx, symmetric, params);
}

// The reference's running extreme of one row: `v < mn` / `v > mx` from
// data[0] on keeps the FIRST element (in index order) of the extreme value
// (which decides the sign of a zero extreme), never takes a NaN, and stays
// NaN when data[0] is NaN.  A candidate is (value, index); idx < 0 = none.
struct Extreme {
    float v;
    int64_t i;
};
template <bool MIN>
__device__ __forceinline__ Extreme better(Extreme a, Extreme b) {
    if (b.i < 0) return a;
    if (a.i < 0) return b;
    const bool take = MIN ? (b.v < a.v || (b.v == a.v && b.i < a.i)) : (b.v > a.v || (b.v == a.v && b.i < a.i));
    return take ? b : a;
}
template <bool MIN>
__device__ __forceinline__ Extreme warp_extreme(Extreme e) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        Extreme t;
        t.v = __shfl_xor_sync(0xffffffffu, e.v, o);
        t.i = __shfl_xor_sync(0xffffffffu, e.i, o);
        e = better<MIN>(e, t);
    }
    return e;
}

// calibrate_per_channel_minmax(data, rows, cols, symmetric), engine.tkv:
// 202-213: calibrate_minmax of every row, one warp per row, all four
// QuantParams fields (the true row extremes, not rebuilt from the scale).
__global__ void rowwise_params_kernel(const float* __restrict__ x, int64_t rows, int64_t cols, int symmetric,
                                      float* __restrict__ scale, int64_t* __restrict__ zp, float* __restrict__ mnv,
                                      float* __restrict__ mxv) {
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float* xr = x + r * cols;
        Extreme lo{0.0f, -1}, hi{0.0f, -1};
        for (int64_t c = lane; c < cols; c += 32) {
            const float v = xr[c];
            if (v != v) continue;  // a NaN never wins a comparison
            if (lo.i < 0 || v < lo.v) lo = Extreme{v, c};
            if (hi.i < 0 || v > hi.v) hi = Extreme{v, c};
        }
        lo = warp_extreme<true>(lo);
        hi = warp_extreme<false>(hi);
        if (lane == 0) {
            double mn, mx;
            if (xr[0] != xr[0]) {
                mn = mx = __longlong_as_double(0x7FF8000000000000ll);
            } else {
                mn = lo.v;
                mx = hi.v;
            }
            float p[4];
            params_from_minmax(mn, mx, symmetric, p);
            scale[r] = p[0];
            zp[r] = static_cast<int64_t>(p[1]);
            mnv[r] = p[2];
            mxv[r] = p[3];
        }
    }
}

int launch_rowwise_params(const float* x, int64_t rows, int64_t cols, int symmetric, float* scale, int64_t* zp,
                          float* mn, float* mx, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return TVQ_OK;
    const int threads = 256;
    rowwise_params_kernel<<<grid_for(rows * 32, threads, 8), threads, 0, st>>>(x, rows, cols, symmetric, scale, zp, mn,
                                                                              mx);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

int launch_minmax_reset(uint32_t* mm, cudaStream_t st) {
    minmax_reset_kernel<<<1, 1, 0, st>>>(mm);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

int launch_minmax_accumulate(const float* x, int64_t n, uint32_t* mm, float* first, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    if (first) copy_first_kernel<<<1, 1, 0, st>>>(x, first);
    const int threads = 512;
    minmax_kernel<<<grid_for((n + 3) / 4, threads, 4), threads, 0, st>>>(x, n, mm);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

int launch_minmax_finalize(const uint32_t* mm, const float* first, int symmetric, float* params, cudaStream_t st) {
    minmax_finalize_kernel<<<1, 1, 0, st>>>(mm, first, symmetric, params);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// ------------------------------------------------------------ K2: quantize
// quantize_int8_symmetric, tv/quantization/engine.tkv:216-226:
// q = clamp(int(round(x * (1.0/scale))), -127, 127).  16 elements per thread
// step: four 16-byte loads, one 16-byte store.  With amax set, the scale is
// first calibrated from the recorded max|x| (calibrate_minmax, engine.tkv:
// 13-36) by every block and block 0 stores it to scale_out.
__global__ void quantize_i8_kernel(const float* __restrict__ x, int8_t* __restrict__ q, int64_t n,
                                   const float* __restrict__ scale, const uint32_t* __restrict__ amax,
                                   float* __restrict__ scale_out) {
    griddep_wait();
    float sc;
    if (amax) {
        sc = scale_from_amax_bits(*amax);
        if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = sc;
    } else {
        sc = __ldg(scale);
    }
    const InvScale qs = make_inv_scale(static_cast<double>(sc));
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(q)) & 15) == 0;
    const int64_t n16 = vec ? n / 16 : 0;
    for (int64_t i = tid; i < n16; i += stride) {
        const float4* src = reinterpret_cast<const float4*>(x) + i * 4;
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = __ldcs(src + j);
        uint32_t w[4];
        bool ok = true;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            float t0, t1, t2, t3;
            ok &= quant_fast_t(v[j].x, qs.hi, t0) & quant_fast_t(v[j].y, qs.hi, t1) &
                  quant_fast_t(v[j].z, qs.hi, t2) & quant_fast_t(v[j].w, qs.hi, t3);
            w[j] = pack_q4(t0, t1, t2, t3);
        }
        if (!ok) {  // rare: the binary64 expression decides
#pragma unroll
            for (int j = 0; j < 4; j++) {
                char4 c;
                c.x = quant_exact(v[j].x, qs);
                c.y = quant_exact(v[j].y, qs);
                c.z = quant_exact(v[j].z, qs);
                c.w = quant_exact(v[j].w, qs);
                w[j] = *reinterpret_cast<const uint32_t*>(&c);
            }
        }
        reinterpret_cast<uint4*>(q)[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    for (int64_t i = n16 * 16 + tid; i < n; i += stride) q[i] = quant_exact(x[i], qs);
}

int launch_quantize_i8(const float* x, int8_t* q, int64_t n, const float* scale_dev, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    const int threads = 256;
    return launch_pdl(quantize_i8_kernel, dim3(grid_for((n + 15) / 16, threads, 8)), dim3(threads), 0, st, x, q, n,
                      scale_dev, static_cast<const uint32_t*>(nullptr), static_cast<float*>(nullptr));
}

int launch_quantize_i8_amax(const float* x, int8_t* q, int64_t n, const uint32_t* amax, float* scale_out,
                            cudaStream_t st) {
    const int threads = 256;
    const int64_t work = std::max<int64_t>((n + 15) / 16, 1);  // n = 0 still stores the scale
    return launch_pdl(quantize_i8_kernel, dim3(grid_for(work, threads, 8)), dim3(threads), 0, st, x, q, n,
                      static_cast<const float*>(nullptr), amax, scale_out);
}

// dequantize_int8_symmetric / _per_channel, engine.tkv:229-234, 253-262:
// fl32(q * scale) is one correctly rounded f32 multiply.
__global__ void dequantize_i8_kernel(const int8_t* __restrict__ q, float* __restrict__ y, int64_t rows,
                                     int64_t cols, const float* __restrict__ scales, int per_row) {
    const int64_t n = rows * cols;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = tid; i < n; i += stride) {
        const float s = per_row ? __ldg(scales + i / cols) : __ldg(scales);
        y[i] = __fmul_rn(static_cast<float>(q[i]), s);
    }
}

int launch_dequantize_i8(const int8_t* q, float* y, int64_t rows, int64_t cols, const float* scales_dev,
                         int per_row, cudaStream_t st) {
    if (rows * cols <= 0) return TVQ_OK;
    const int threads = 256;
    dequantize_i8_kernel<<<grid_for(rows * cols, threads, 8), threads, 0, st>>>(q, y, rows, cols, scales_dev,
                                                                                per_row);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// One warp per row.  mode 0: calibrate_per_channel_minmax (engine.tkv:202-213)
// fused with quantize_int8_per_channel (engine.tkv:237-250) -- scale[r] =
// fl32(max(amax,1e-8)/127), then q with inv = 1/max(scale[r],1e-8).
// mode 1: quantize with given scales.  mode 2: quantize_dynamic_int8_rowwise
// (engine.tkv:266-285) -- the f64 scale quantizes, its f32 copy is stored.
template <int MODE>
__global__ void rowwise_kernel(const float* __restrict__ x, int8_t* __restrict__ q, float* __restrict__ scales,
                               int64_t rows, int64_t cols) {
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(q) & 3) == 0);
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float* xr = x + r * cols;
        int8_t* qr = q + r * cols;
        InvScale qs;
        if (MODE == 1) {
            qs = make_inv_scale(static_cast<double>(__ldg(scales + r)));
        } else {
            float am = 0.0f;
            if (vec) {
                for (int64_t c = lane * 4; c < cols; c += 128) {
                    float4 v = *reinterpret_cast<const float4*>(xr + c);
                    am = fmaxf(am, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                }
            } else {
                for (int64_t c = lane; c < cols; c += 32) am = fmaxf(am, fabsf(xr[c]));
            }
            am = warp_max(am);
            double amd = am;
            bool poisoned = false;
            if (MODE == 0) poisoned = (xr[0] != xr[0]);   // NaN first element poisons min/max
            if (amd < 0.00000001) amd = 0.00000001;
            if (MODE == 0) {
                float sc = poisoned ? __int_as_float(0x7FC00000) : __double2float_rn(amd / 127.0);
                if (lane == 0) scales[r] = sc;
                qs = make_inv_scale(static_cast<double>(sc));  // NaN scale -> NaN inverse -> q = 0
            } else {
                double sc = amd / 127.0;
                if (lane == 0) scales[r] = __double2float_rn(sc);
                qs = make_inv_from_inv(1.0 / sc);  // the unrounded f64 scale quantizes
            }
        }
        if (vec) {
            for (int64_t c = lane * 4; c < cols; c += 128) {
                float4 v = *reinterpret_cast<const float4*>(xr + c);
                char4 o;
                o.x = quant_exact(v.x, qs);
                o.y = quant_exact(v.y, qs);
                o.z = quant_exact(v.z, qs);
                o.w = quant_exact(v.w, qs);
                *reinterpret_cast<char4*>(qr + c) = o;
            }
        } else {
            for (int64_t c = lane; c < cols; c += 32) qr[c] = quant_exact(xr[c], qs);
        }
    }
}

// Modes 0 and 2 for rows of 1025 .. 8192 floats (cols % 4 == 0, 16-byte
// aligned rows): a 256-thread block takes its rows one at a time, and the
// rows stream into a ring of ROW_SLOTS shared-memory slots by 1-D bulk
// copies (the TMA engine; warp 0 issues up to 8 KB per lane, completion on
// the slot's mbarrier), so HBM never waits for the arithmetic and each
// element is read once.  Per row: max |x| (one block reduction), the scale,
// the quantize.  Mode 0 (calibrate_per_channel_minmax + quantize) forms the
// scale in every thread without binary64: fl32(fl64(amax / 127)) is the
// correctly rounded f32 quotient (an f64 quotient by 127 repeats a 7-bit
// pattern, so it never lands on an f32 rounding midpoint), and the fast
// quantize needs only fl32(1 / scale) (quant_fast_t); the binary64 1/scale
// is formed in the rare near-tie path.  Mode 2 (dynamic, scale kept in
// binary64) takes its scale from warp 0.  Every wait is bounded
// (DEVERR_TIMEOUT_ROWS).
constexpr int ROW_THREADS = 256;      // four blocks per SM (rows up to 6400 floats): 32 warps
constexpr uint32_t ROW_CHUNK = 8192;  // bytes per bulk copy
constexpr int ROW_SLOTS = 2;

template <int MODE>
__global__ void __launch_bounds__(ROW_THREADS, 4) rowwise_pipe_kernel(const float* __restrict__ x, int8_t* __restrict__ q,
                                                                      float* __restrict__ scales, int64_t rows,
                                                                      int64_t cols, int* err) {
    extern __shared__ __align__(128) float4 rbuf[];  // [ROW_SLOTS][cols / 4]
    __shared__ float red[ROW_THREADS / 32];
    __shared__ InvScale row_qs;
    __shared__ __align__(8) uint64_t full[ROW_SLOTS];
    const int tid = threadIdx.x;
    const int n4 = static_cast<int>(cols / 4);
    const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
    const int64_t step = gridDim.x;
    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < ROW_SLOTS; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    // row r into ring slot `slot` (every thread is done reading the slot's
    // previous row: a block barrier separates those reads from this call)
    auto issue = [&](int64_t r, int slot) {
        if (r >= rows || tid >= 32) return;
        if (tid == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&full[slot], row_bytes);
        }
        __syncwarp();
        const uint32_t off = static_cast<uint32_t>(tid) * ROW_CHUNK;
        if (off < row_bytes)
            bulk_load(reinterpret_cast<char*>(rbuf + static_cast<int64_t>(slot) * n4) + off,
                      reinterpret_cast<const char*>(x + r * cols) + off, min(ROW_CHUNK, row_bytes - off), &full[slot]);
    };
    int64_t r = blockIdx.x;
#pragma unroll
    for (int s = 0; s < ROW_SLOTS - 1; s++) issue(r + s * step, s);
    for (int i = 0; r < rows; i++, r += step) {
        const int slot = i % ROW_SLOTS;
        const uint32_t par = static_cast<uint32_t>(i / ROW_SLOTS) & 1u;
        const bool ok = mbar_wait(&full[slot], par, err, DEVERR_TIMEOUT_ROWS);
        // every thread is past the previous row (its slot is free, red[] too)
        if (!__syncthreads_and(ok)) {  // the error word holds the cause
            // the only copy in flight is this slot's (the next row is issued
            // after this barrier): give it a bounded time to land, then leave
            if (tid == 0) {
                const uint64_t t0 = globaltimer_ns();
                while (!mbar_try_wait(&full[slot], par) && globaltimer_ns() - t0 < 100000000ull) __nanosleep(1000);
            }
            return;
        }
        issue(r + (ROW_SLOTS - 1) * step, (i + ROW_SLOTS - 1) % ROW_SLOTS);
        const float4* row = rbuf + static_cast<int64_t>(slot) * n4;
        float am = 0.0f;
        for (int c = tid; c < n4; c += ROW_THREADS) {
            const float4 v = row[c];
            am = fmaxf(am, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
        am = warp_max(am);
        if ((tid & 31) == 0) red[tid >> 5] = am;
        __syncthreads();
#pragma unroll
        for (int w = 0; w < ROW_THREADS / 32; w++) am = fmaxf(am, red[w]);
        float sc, hi;
        if (MODE == 0) {
            const float x0 = reinterpret_cast<const float*>(row)[0];
            if (x0 != x0) {  // NaN first element poisons min/max
                sc = __int_as_float(0x7FC00000);
            } else if (static_cast<double>(am) < 0.00000001) {
                sc = __double2float_rn(0.00000001 / 127.0);
            } else {
                sc = __fdiv_rn(am, 127.0f);  // = fl32(fl64(am / 127)), see above
            }
            hi = (static_cast<double>(sc) > 0.00000001) ? __frcp_rn(sc) : __double2float_rn(1.0 / 0.00000001);
            if (sc != sc) hi = sc;  // NaN scale: NaN products -> 0
            if (tid == 0) scales[r] = sc;
        } else {
            if (tid == 0) {
                double amd = am;
                if (amd < 0.00000001) amd = 0.00000001;
                const double scd = amd / 127.0;
                scales[r] = __double2float_rn(scd);
                row_qs = make_inv_from_inv(1.0 / scd);
            }
            __syncthreads();
            hi = row_qs.hi;
            sc = 0.0f;
        }
        uint32_t* qr = reinterpret_cast<uint32_t*>(q + r * cols);
        for (int c = tid; c < n4; c += ROW_THREADS) {
            const float4 v = row[c];
            float t0, t1, t2, t3;
            const bool fast = quant_fast_t(v.x, hi, t0) & quant_fast_t(v.y, hi, t1) & quant_fast_t(v.z, hi, t2) &
                              quant_fast_t(v.w, hi, t3);
            uint32_t w = pack_q4(t0, t1, t2, t3);
            if (!fast) {  // rare: the binary64 expression decides
                const InvScale qs = (MODE == 0) ? make_inv_scale(static_cast<double>(sc)) : row_qs;
                char4 o;
                o.x = quant_exact(v.x, qs);
                o.y = quant_exact(v.y, qs);
                o.z = quant_exact(v.z, qs);
                o.w = quant_exact(v.w, qs);
                w = *reinterpret_cast<const uint32_t*>(&o);
            }
            qr[c] = w;
        }
    }
}

int launch_rowwise(int mode, const float* x, int8_t* q, float* scales, int64_t rows, int64_t cols,
                   cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return TVQ_OK;
    const int threads = 256;
    const bool vec = (cols % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15) == 0) &&
                     ((reinterpret_cast<uintptr_t>(q) & 3) == 0);
    if (mode != 1 && vec && cols > 1024 && cols <= 8192) {
        const size_t smem = static_cast<size_t>(ROW_SLOTS) * static_cast<size_t>(cols) * 4;  // <= 96 KB
        static int attr_done[64] = {0};  // per device
        int dev = 0;
        TVQ_CUDA(cudaGetDevice(&dev));
        if (dev < 64 && !attr_done[dev]) {
            TVQ_CUDA(cudaFuncSetAttribute(rowwise_pipe_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          ROW_SLOTS * 8192 * 4));
            TVQ_CUDA(cudaFuncSetAttribute(rowwise_pipe_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          ROW_SLOTS * 8192 * 4));
            attr_done[dev] = 1;
        }
        int rc = 0;
        DeviceState* ds = device_state(&rc);
        if (!ds) return rc;
        const int per_sm = static_cast<int>(std::min<size_t>(4, (227 * 1024) / (smem + 1024)));
        const int g = grid_for(rows * ROW_THREADS, ROW_THREADS, per_sm);
        if (mode == 0) rowwise_pipe_kernel<0><<<g, ROW_THREADS, smem, st>>>(x, q, scales, rows, cols, ds->d_error);
        else rowwise_pipe_kernel<2><<<g, ROW_THREADS, smem, st>>>(x, q, scales, rows, cols, ds->d_error);
        TVQ_CUDA(cudaGetLastError());
        return TVQ_OK;
    }
    const int grid = grid_for(rows * 32, threads, 8);
    if (mode == 0) rowwise_kernel<0><<<grid, threads, 0, st>>>(x, q, scales, rows, cols);
    else if (mode == 1) rowwise_kernel<1><<<grid, threads, 0, st>>>(x, q, scales, rows, cols);
    else rowwise_kernel<2><<<grid, threads, 0, st>>>(x, q, scales, rows, cols);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// ------------------------------------------------------------ K3: FP8 E4M3

// The reference's E4M3 encoder: tvq_e4m3.h (e4m3_encode_fast in the kernels,
// e4m3_encode_ref beside it, equal on every binary32 input).

// native_fp8_e4m3_decode = _qt_fp8_decode(v, 7, 3, 15, 0), types.tkv:193-226,
// through f32_bits_to_f64 (f32_bits.tkv:60-74): 0x7F/0xFF give +/-Inf (the
// exponent-255 branch returns 2^129), -0 gives +0 (0.0 - 0.0), subnormal m
// gives m * 2^-10 (the decoder's exponent is 127 - bias - n).
__host__ __device__ __forceinline__ float e4m3_decode_ref(uint32_t v) {
    const uint32_t sign = (v >> 7) & 1;
    const uint32_t e8 = (v >> 3) & 15;
    const uint32_t m8 = v & 7;
    float mag;
    if (e8 == 15 && m8 == 7) {
        mag = INFINITY;
    } else if (e8 == 0) {
        if (m8 == 0) return 0.0f;
        mag = static_cast<float>(m8) * 0.0009765625f;  // 2^-10
    } else {
        mag = (1.0f + static_cast<float>(m8) * 0.125f) * ldexpf(1.0f, static_cast<int>(e8) - 7);
    }
    return sign ? -mag : mag;
}

__device__ __forceinline__ uint8_t e4m3_encode_hw(float x) {
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3));
}

// fl32(fl64(x) * inv): the scaled value as the reference forms it (binary64
// product, rounded once to binary32 at the typed store), evaluated directly
// -- one DMUL and two conversions, cheaper on B200 than the float-expansion
// proof of mul_round_exact (the FP8 kernels are compute-bound).
__device__ __forceinline__ float mul_round_f64(float x, const InvScale& s) {
    return __double2float_rn(__dmul_rn(static_cast<double>(x), s.d));
}

// The reference's E4M3 byte.  Away from its departures from OCP E4M3 the
// reference encoder rounds the exact value to nearest-even on the same grid
// as the hardware RN-satfinite conversion (one instruction), so that
// conversion serves every v with |v| < 240, outside (0.875, 1) 2^-6 and
// normal or larger; the rest goes to e4m3_encode_fast: |v| >= 240 (the
// reference saturates to 448 from 240 on; NaN and Inf), the subnormal codes
// that would carry into the normals (the reference stays at code 7), zeros
// and binary32 denormals (sign handling).  Checked on all 2^32 inputs.
__device__ __forceinline__ uint32_t e4m3_encode_ref_hw(float v) {
    const uint32_t a = __float_as_uint(v) & 0x7FFFFFFFu;
    const bool slow = a >= 0x43700000u || (a > 0x3C600000u && a < 0x3C800000u) || a < 0x00800000u;
    return slow ? e4m3_encode_fast(__float_as_uint(v)) : e4m3_encode_hw(v);
}

__device__ __forceinline__ uint32_t e4m3_byte(float v, bool hw) {
    return hw ? e4m3_encode_hw(v) : e4m3_encode_ref_hw(v);
}

// four scaled elements -> four E4M3 bytes, little-endian in a word
__device__ __forceinline__ uint32_t e4m3_word(const float4& v, const InvScale& s, bool hw) {
    return e4m3_byte(mul_round_f64(v.x, s), hw) | (e4m3_byte(mul_round_f64(v.y, s), hw) << 8) |
           (e4m3_byte(mul_round_f64(v.z, s), hw) << 16) | (e4m3_byte(mul_round_f64(v.w, s), hw) << 24);
}

// SCALE: 0 none (quantize_fp8_e4m3, matmul.tkv:60-66), 1 per tensor, 2 per
// row; the scaled value is fl32(x * (1/scale)) as the encoder's f32 argument.
// VEC: 16-byte loads and 4-byte stores (x 16-byte and q 4-byte aligned, n % 4
// == 0 for the flat form, cols % 4 == 0 for the per-row form).
template <int SCALE, int HW, int VEC>
__global__ void fp8_encode_kernel(const float* __restrict__ x, uint8_t* __restrict__ q, int64_t rows, int64_t cols,
                                  const float* __restrict__ scales) {
    const int64_t n = rows * cols;
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    InvScale s0{1.0, 1.0f, 0.0f};
    if (SCALE == 1) s0 = make_inv_scale(static_cast<double>(__ldg(scales)));
    if (VEC) {
        for (int64_t i = tid; i < n / 4; i += stride) {
            float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
            if (SCALE == 1) {
                v.x = mul_round_f64(v.x, s0);
                v.y = mul_round_f64(v.y, s0);
                v.z = mul_round_f64(v.z, s0);
                v.w = mul_round_f64(v.w, s0);
            }
            reinterpret_cast<uint32_t*>(q)[i] = e4m3_byte(v.x, HW) | (e4m3_byte(v.y, HW) << 8) |
                                                (e4m3_byte(v.z, HW) << 16) | (e4m3_byte(v.w, HW) << 24);
        }
        return;
    }
    for (int64_t i = tid; i < n; i += stride) {
        float v = x[i];
        if (SCALE == 1) v = mul_round_f64(v, s0);
        q[i] = static_cast<uint8_t>(e4m3_byte(v, HW));
    }
}

// Per-row scales: one warp per row, the row's 1/scale formed once.
template <int HW, int VEC>
__global__ void fp8_encode_rows_kernel(const float* __restrict__ x, uint8_t* __restrict__ q, int64_t rows,
                                       int64_t cols, const float* __restrict__ scales) {
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    const int lane = threadIdx.x & 31;
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const InvScale s = make_inv_scale(static_cast<double>(__ldg(scales + r)));
        if (VEC) {
            const float4* xr = reinterpret_cast<const float4*>(x + r * cols);
            uint32_t* qr = reinterpret_cast<uint32_t*>(q + r * cols);
            const int64_t n4 = cols / 4;
            int64_t c = lane;
            // four 16-byte loads in flight per lane before any is encoded
            for (; c + 96 < n4; c += 128) {
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) v[u] = __ldcs(xr + c + 32 * u);
#pragma unroll
                for (int u = 0; u < 4; u++) qr[c + 32 * u] = e4m3_word(v[u], s, HW);
            }
            for (; c < n4; c += 32) qr[c] = e4m3_word(__ldcs(xr + c), s, HW);
            continue;
        }
        for (int64_t c = lane; c < cols; c += 32) {
            const float v = mul_round_f64(x[r * cols + c], s);
            q[r * cols + c] = static_cast<uint8_t>(e4m3_byte(v, HW));
        }
    }
}

int launch_fp8_encode(const float* x, uint8_t* q, int64_t rows, int64_t cols, const float* scales, int scale_mode,
                      int hw, cudaStream_t st) {
    const int64_t n = rows * cols;
    if (n <= 0) return TVQ_OK;
    const int threads = 256;
    const bool aligned = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((reinterpret_cast<uintptr_t>(q) & 3) == 0);
    if (scale_mode == 2) {
        const int g = grid_for(rows * 32, threads, 8);
        const bool vec = aligned && cols % 4 == 0;
#define TVQ_FP8_ROWS(H, V) fp8_encode_rows_kernel<H, V><<<g, threads, 0, st>>>(x, q, rows, cols, scales)
        if (hw) { if (vec) TVQ_FP8_ROWS(1, 1); else TVQ_FP8_ROWS(1, 0); }
        else { if (vec) TVQ_FP8_ROWS(0, 1); else TVQ_FP8_ROWS(0, 0); }
#undef TVQ_FP8_ROWS
    } else {
        const bool vec = aligned && n % 4 == 0;
        const int grid = grid_for(vec ? n / 4 : n, threads, 8);
#define TVQ_FP8_LAUNCH(S, H, V) fp8_encode_kernel<S, H, V><<<grid, threads, 0, st>>>(x, q, rows, cols, scales)
#define TVQ_FP8_LAUNCH_V(S, H) do { if (vec) TVQ_FP8_LAUNCH(S, H, 1); else TVQ_FP8_LAUNCH(S, H, 0); } while (0)
        if (scale_mode == 0) { if (hw) TVQ_FP8_LAUNCH_V(0, 1); else TVQ_FP8_LAUNCH_V(0, 0); }
        else { if (hw) TVQ_FP8_LAUNCH_V(1, 1); else TVQ_FP8_LAUNCH_V(1, 0); }
#undef TVQ_FP8_LAUNCH_V
#undef TVQ_FP8_LAUNCH
    }
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

__global__ void fp8_decode_kernel(const uint8_t* __restrict__ q, float* __restrict__ y, int64_t n) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = tid; i < n; i += stride) y[i] = e4m3_decode_ref(q[i]);
}

int launch_fp8_decode(const uint8_t* q, float* y, int64_t n, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    const int threads = 256;
    fp8_decode_kernel<<<grid_for(n, threads, 8), threads, 0, st>>>(q, y, n);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// quantize_fp16 (matmul.tkv:106-114): the reference's FP16 encoder
// (tvq_f16.h) per element.  VEC: 16-byte loads, 8-byte stores.
template <int VEC>
__global__ void f16_encode_kernel(const float* __restrict__ x, uint16_t* __restrict__ q, int64_t n) {
    griddep_wait();
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    if (VEC) {
        for (int64_t i = tid; i < n / 4; i += stride) {
            const float4 v = __ldcs(reinterpret_cast<const float4*>(x) + i);
            const uint32_t lo = f16_encode_fast(__float_as_uint(v.x)) | (f16_encode_fast(__float_as_uint(v.y)) << 16);
            const uint32_t hi = f16_encode_fast(__float_as_uint(v.z)) | (f16_encode_fast(__float_as_uint(v.w)) << 16);
            __stcs(reinterpret_cast<uint2*>(q) + i, make_uint2(lo, hi));
        }
        return;
    }
    for (int64_t i = tid; i < n; i += stride) q[i] = f16_encode_fast(__float_as_uint(x[i]));
}

int launch_f16_encode(const float* x, uint16_t* q, int64_t n, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    const int threads = 256;
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0) && ((reinterpret_cast<uintptr_t>(q) & 7) == 0) &&
                     n % 4 == 0;
    if (vec) return launch_pdl(f16_encode_kernel<1>, dim3(grid_for(n / 4, threads, 8)), dim3(threads), 0, st, x, q, n);
    return launch_pdl(f16_encode_kernel<0>, dim3(grid_for(n, threads, 8)), dim3(threads), 0, st, x, q, n);
}

// ------------------------------------------------------------ list[i32] forms
__global__ void i8_to_i32_kernel(const int8_t* __restrict__ a, int32_t* __restrict__ b, int64_t n, int32_t off) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = tid; i < n; i += stride) b[i] = static_cast<int32_t>(a[i]) + off;
}
__global__ void u8_to_i32_kernel(const uint8_t* __restrict__ a, int32_t* __restrict__ b, int64_t n, int32_t off) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = tid; i < n; i += stride) b[i] = static_cast<int32_t>(a[i]) + off;
}
// list[i32] -> bytes: int8 values wrap as the reference's int() of an
// already-clamped value; FP8 values are byte - 128 (matmul.tkv:65, :76).
__global__ void i32_to_u8_kernel(const int32_t* __restrict__ a, uint8_t* __restrict__ b, int64_t n, int32_t off) {
    const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = tid; i < n; i += stride) b[i] = static_cast<uint8_t>((a[i] + off) & 0xFF);
}

int launch_widen(const void* src, int32_t* dst, int64_t n, int is_unsigned, int32_t off, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    const int threads = 256;
    const int grid = grid_for(n, threads, 8);
    if (is_unsigned) u8_to_i32_kernel<<<grid, threads, 0, st>>>(static_cast<const uint8_t*>(src), dst, n, off);
    else i8_to_i32_kernel<<<grid, threads, 0, st>>>(static_cast<const int8_t*>(src), dst, n, off);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

int launch_narrow(const int32_t* src, void* dst, int64_t n, int32_t off, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    const int threads = 256;
    i32_to_u8_kernel<<<grid_for(n, threads, 8), threads, 0, st>>>(src, static_cast<uint8_t*>(dst), n, off);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// Host copy of the reference decoder for the C ABI's scalar helpers.
float e4m3_decode_host(uint32_t v) { return e4m3_decode_ref(v); }
uint8_t e4m3_encode_host(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    return e4m3_encode_fast(b);
}

}  // namespace tvq
