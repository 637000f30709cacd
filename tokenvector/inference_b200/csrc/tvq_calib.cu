// tvq_calib.cu -- the calibration methods of tv/quantization/engine.tkv
// beyond min/max: KL (:42-122), percentile (:125-162) and MSE (:165-197), on
// the GPU with the reference's binary64 model.
//
// KL: one pass for max |x| (the min/max kernel of tvq_quant.cu), one pass of
// shared-memory histograms (bin = int(|x| / bw), decided in binary32 with a
// proof that the binary64 quotient truncates to the same integer, else
// binary64), then one block where each thread evaluates one candidate
// threshold with the reference's sequential binary64 loops over the bins
// (same operation order, so the divergence-free result equals a sequential
// evaluation up to the last bit of log()).
// Percentile: the int(min(n-1, percentile/100 n))-th smallest |x| by an exact
// 4-pass radix select on the binary32 bit patterns (|x| orders like its
// bits), no sort.
// MSE: per candidate threshold the binary64 squared-error sum, block partials
// in a fixed order (deterministic; the order differs from the reference's
// sequential sum, so two candidates within ~1e-15 relative of each other
// could swap -- a tie the reference breaks by index).
#include <algorithm>
#include <cmath>
#include <vector>

#include "tvq_common.cuh"
#include "tvq_kernels.h"

namespace tvq {

#define STEP_RC(expr)          \
    do {                       \
        int r__ = (expr);      \
        if (r__) return r__;   \
    } while (0)

namespace {

__device__ __forceinline__ float ord2f_c(uint32_t u) {
    const uint32_t b = (u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u;
    return __uint_as_float(b);
}

// QuantParams as four words: scale f32, zero point (as f32, exact in range),
// min f32, max f32 -- plus the binary64 threshold / clip kept for later passes.
struct CalibState {
    double am;        // max |x|
    double bw;        // KL bin width
    double clip;      // percentile clip
    uint32_t prefix;  // radix select: value bits found so far
    uint32_t pad;
    long long k;      // radix select: rank within the current prefix bucket
    float out[4];     // scale, zero point, min, max
    int use_minmax;   // am < 1e-8: the caller falls back to calibrate_minmax
    int pad2;
};

__global__ void calib_absmax_kernel(const uint32_t* mm, CalibState* cs) {
    griddep_wait();
    // the running min / max ignore NaN; max |x| = max(|min|, |max|), 0 when empty
    double am = 0.0;
    if (!(mm[0] == 0xFFFFFFFFu && mm[1] == 0u)) {
        am = fabs(static_cast<double>(ord2f_c(mm[0])));
        const double b = fabs(static_cast<double>(ord2f_c(mm[1])));
        if (b > am) am = b;
    }
    cs->am = am;
    cs->use_minmax = am < 0.00000001;
}

static __device__ __noinline__ long long trunc_slow(double v) {
    if (v != v) return 0;
    if (v >= 9.2233720368547758e18) return 0x7FFFFFFFFFFFFFFFll;
    return static_cast<long long>(v);
}

// int(|x| / bw) for bw > 0: fast in binary32 when the quotient is clearly
// between two integers (distance > 2^-21 |r|), else binary64.
__device__ __forceinline__ long long trunc_div(float ax, double bw, float bwf) {
    const float r = __fdiv_rn(ax, bwf);
    if (r < 2097152.0f) {  // false for NaN
        const float k = truncf(r);
        const float f = r - k;
        const float d = fminf(f, 1.0f - f);
        if (d > r * 4.76837158203125e-07f + 1e-30f) return static_cast<long long>(k);
    }
    return trunc_slow(static_cast<double>(ax) / bw);
}

// histogram of |x| into nb bins; shared-memory counts, one atomic per bin per block
__global__ void kl_hist_kernel(const float* __restrict__ x, int64_t n, const CalibState* __restrict__ cs, int nb,
                               unsigned long long* __restrict__ hist) {
    griddep_wait();
    extern __shared__ unsigned int sh[];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) sh[i] = 0;
    __syncthreads();
    if (!cs->use_minmax) {
        const double bw = cs->bw;
        const float bwf = __double2float_rn(bw);
        const bool fast = bwf > 0.0f && static_cast<double>(bwf) == bw;
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
            const float ax = fabsf(x[i]);
            long long b = fast ? trunc_div(ax, bw, bwf) : trunc_slow(static_cast<double>(ax) / bw);
            if (b >= nb) b = nb - 1;
            atomicAdd(&sh[b], 1u);
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nb; i += blockDim.x)
        if (sh[i]) atomicAdd(&hist[i], static_cast<unsigned long long>(sh[i]));
}

__global__ void kl_setup_kernel(CalibState* cs, int nb) {
    griddep_wait();
    cs->bw = cs->am / static_cast<double>(nb);
}

// One thread per candidate th = tb + 16 c: the reference's loops, in order.
__global__ void kl_search_kernel(const unsigned long long* __restrict__ hist, int nb, int tb, int ncand,
                                 CalibState* __restrict__ cs) {
    griddep_wait();
    extern __shared__ unsigned long long hs[];
    __shared__ double best_kl_s[1024];
    __shared__ int best_th_s[1024];
    for (int i = threadIdx.x; i < nb; i += blockDim.x) hs[i] = hist[i];
    __syncthreads();
    double best_kl = 1e45;
    int best_th = nb;
    if (!cs->use_minmax && threadIdx.x < ncand) {
        const int th = tb + 16 * threadIdx.x;
        double s = 0.0;
        for (int i = 0; i < th; i++) s = s + static_cast<double>(hs[i]);
        double p_last = static_cast<double>(hs[th - 1]);
        for (int i = th; i < nb; i++) {
            p_last = p_last + static_cast<double>(hs[i]);
            s = s + static_cast<double>(hs[i]);
        }
        if (s != 0.0) {
            const int per = th / tb;
            if (per >= 1) {
                double kl = 0.0;
                for (int b = 0; b < tb; b++) {
                    const int start = b * per;
                    const int end = (b == tb - 1) ? th : start + per;
                    double mass = 0.0;
                    for (int i = start; i < end; i++) {
                        const double pi = ((i == th - 1) ? p_last : static_cast<double>(hs[i])) / s;
                        mass = mass + pi;
                    }
                    int span = end - start;
                    if (span < 1) span = 1;
                    const double share = mass / static_cast<double>(span);
                    // q[i] = share for i in [start, end); the KL terms of those bins
                    // are added below in bin order (kl is a running sum over i)
                    for (int i = start; i < end; i++) {
                        const double pi = ((i == th - 1) ? p_last : static_cast<double>(hs[i])) / s;
                        if (pi > 0.000000000001 && share > 0.000000000001) kl = kl + pi * log(pi / share);
                    }
                }
                best_kl = kl;
                best_th = th;
            }
        }
    }
    best_kl_s[threadIdx.x] = best_kl;
    best_th_s[threadIdx.x] = best_th;
    __syncthreads();
    if (threadIdx.x == 0 && !cs->use_minmax) {
        double bk = 1e45;
        int bt = nb;
        for (int i = 0; i < ncand; i++)  // candidates in th order: the first strict minimum
            if (best_kl_s[i] < bk) {
                bk = best_kl_s[i];
                bt = best_th_s[i];
            }
        const double thr = static_cast<double>(bt) * cs->bw;
        cs->out[0] = __double2float_rn(thr / 127.0);
        cs->out[1] = 0.0f;
        cs->out[2] = __double2float_rn(-thr);
        cs->out[3] = __double2float_rn(thr);
    }
}

// radix select over |x| bit patterns: pass `shift` counts digit (bits >>
// shift) & 255 of the elements whose higher bits equal the prefix
__global__ void radix_hist_kernel(const float* __restrict__ x, int64_t n, const CalibState* __restrict__ cs,
                                  int shift, unsigned long long* __restrict__ hist) {
    griddep_wait();
    __shared__ unsigned int sh[256];
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sh[i] = 0;
    __syncthreads();
    const uint32_t prefix = cs->prefix;
    const uint32_t hmask = (shift >= 24) ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const uint32_t u = __float_as_uint(x[i]) & 0x7FFFFFFFu;
        if ((u & hmask) == (prefix & hmask)) atomicAdd(&sh[(u >> shift) & 255u], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 256; i += blockDim.x)
        if (sh[i]) atomicAdd(&hist[i], static_cast<unsigned long long>(sh[i]));
}

__global__ void radix_pick_kernel(unsigned long long* __restrict__ hist, int shift, CalibState* __restrict__ cs) {
    griddep_wait();
    long long k = cs->k;
    int d = 0;
    for (; d < 256; d++) {
        const long long c = static_cast<long long>(hist[d]);
        if (k < c) break;
        k -= c;
    }
    if (d > 255) d = 255;  // cannot happen for k < n
    cs->prefix |= static_cast<uint32_t>(d) << shift;
    cs->k = k;
    for (int i = 0; i < 256; i++) hist[i] = 0;  // ready for the next pass
}

__global__ void pct_finish_sym_kernel(CalibState* cs) {
    griddep_wait();
    double clip = static_cast<double>(__uint_as_float(cs->prefix));
    if (clip <= 0.00000001) clip = 0.00000001;
    cs->clip = clip;
    cs->out[0] = __double2float_rn(clip / 127.0);
    cs->out[1] = 0.0f;
    cs->out[2] = __double2float_rn(-clip);
    cs->out[3] = __double2float_rn(clip);
}

// min / max of clamp(x[i], -clip, clip) for i >= 1 (NaN ignored), ordinal encoded
__global__ void pct_clamped_minmax_kernel(const float* __restrict__ x, int64_t n, const CalibState* __restrict__ cs,
                                          uint32_t* __restrict__ mm) {
    griddep_wait();
    // clip is a binary32 value or 1e-8; clamping a binary32 x to +-clip and
    // comparing is the same in f32 when clip is an f32 value, so fold 1e-8
    // separately (values between fl32(1e-8) and 1e-8 cannot be data)
    const double clip = cs->clip;
    const float lo = __double2float_rn(-clip), hi = __double2float_rn(clip);
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t i = 1 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v = x[i];
        if (v != v) continue;
        if (static_cast<double>(v) < -clip) v = lo;
        if (static_cast<double>(v) > clip) v = hi;
        mn = fminf(mn, v);
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    if ((threadIdx.x & 31) == 0) {
        if (mn != INFINITY) {
            const uint32_t b = __float_as_uint(mn);
            atomicMin(mm + 0, (b & 0x80000000u) ? ~b : (b | 0x80000000u));
        }
        if (mx != -INFINITY) {
            const uint32_t b = __float_as_uint(mx);
            atomicMax(mm + 1, (b & 0x80000000u) ? ~b : (b | 0x80000000u));
        }
    }
}

static __device__ __noinline__ long long round_slow(double v) {
    if (v != v) return 0;
    const double r = rint(v);
    if (r >= 9.2233720368547758e18) return 0x7FFFFFFFFFFFFFFFll;
    if (r <= -9.2233720368547758e18) return static_cast<long long>(0x8000000000000000ull);
    return static_cast<long long>(r);
}

// asymmetric finish: mn / mx start at data[0] unclamped (engine.tkv:143-151),
// clip is exactly representable as used here (a binary32 value or 1e-8)
__global__ void pct_finish_asym_kernel(const float* __restrict__ x, int64_t n, const uint32_t* __restrict__ mm,
                                       CalibState* __restrict__ cs) {
    griddep_wait();
    const double clip = cs->clip;
    double mn = x[0], mx = x[0];
    if (n > 1 && !(mm[0] == 0xFFFFFFFFu && mm[1] == 0u)) {
        // clamped values that equal -clip / clip exactly stand for the double clip
        double cmn = ord2f_c(mm[0]), cmx = ord2f_c(mm[1]);
        if (cmn == static_cast<double>(__double2float_rn(-clip))) cmn = -clip;
        if (cmx == static_cast<double>(__double2float_rn(clip))) cmx = clip;
        if (cmn < mn) mn = cmn;
        if (cmx > mx) mx = cmx;
    }
    if (fabs(mx - mn) < 0.00000001) mx = mn + 0.00000001;
    const double scale = (mx - mn) / 255.0;
    long long zp = round_slow(-mn / scale);
    if (zp != 0x7FFFFFFFFFFFFFFFll && zp != static_cast<long long>(0x8000000000000000ull)) zp -= 128;
    zp = zp < -128 ? -128 : (zp > 127 ? 127 : zp);
    cs->out[0] = __double2float_rn(scale);
    cs->out[1] = static_cast<float>(zp);
    cs->out[2] = __double2float_rn(mn);
    cs->out[3] = __double2float_rn(mx);
}

// MSE: partial squared-error sums, block b of candidate c -> part[c * nblk + b]
__global__ void mse_partial_kernel(const float* __restrict__ x, int64_t n, const CalibState* __restrict__ cs, int ncand,
                                   double* __restrict__ part) {
    griddep_wait();
    __shared__ double red[32];
    const int c = blockIdx.y + 1;
    if (cs->use_minmax) return;
    const double am = cs->am;
    const double thr = am * static_cast<double>(c) / static_cast<double>(ncand);
    const double scale = thr / 127.0;
    const double inv = 1.0 / scale;
    double acc = 0.0;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const double xv = x[i];
        double cl = xv;
        if (cl < -thr) cl = -thr;
        if (cl > thr) cl = thr;
        const double t = cl * inv;  // |t| <= 127 (1 + 2^-52) unless x is NaN
        long long q = (t != t) ? 0 : static_cast<long long>(rint(t));
        q = q < -127 ? -127 : (q > 127 ? 127 : q);
        const double d = xv - static_cast<double>(q) * scale;
        acc = acc + d * d;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < (blockDim.x >> 5); w++) s += red[w];
        part[static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x] = s;
    }
}

__global__ void mse_pick_kernel(const double* __restrict__ part, int nblk, int ncand, int64_t n,
                                CalibState* __restrict__ cs, double* __restrict__ curve) {
    griddep_wait();
    if (cs->use_minmax) return;
    const double am = cs->am;
    double best_thr = am, best = 1e45;
    for (int c = 1; c <= ncand; c++) {
        double s = 0.0;
        for (int b = 0; b < nblk; b++) s += part[static_cast<int64_t>(c - 1) * nblk + b];
        const double mse = s / static_cast<double>(n);
        if (curve) curve[c - 1] = mse;
        if (mse < best) {
            best = mse;
            best_thr = am * static_cast<double>(c) / static_cast<double>(ncand);
        }
    }
    cs->out[0] = __double2float_rn(best_thr / 127.0);
    cs->out[1] = 0.0f;
    cs->out[2] = __double2float_rn(-best_thr);
    cs->out[3] = __double2float_rn(best_thr);
}

int grid_for_calib(int64_t n, int threads) {
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    const int64_t cap = static_cast<int64_t>(ds ? ds->sm_count : 148) * 8;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, cap)));
}

// scratch: CalibState, min/max ordinals, histogram / partials
struct CalibScratch {
    char* base = nullptr;
    CalibState* cs = nullptr;
    uint32_t* mm = nullptr;
    float* first = nullptr;
    unsigned long long* hist = nullptr;
    double* part = nullptr;
};

int calib_alloc(CalibScratch& s, size_t hist_words, size_t part_words, cudaStream_t st) {
    const size_t bytes = 256 + 256 + hist_words * 8 + part_words * 8 + 256;
    TVQ_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&s.base), bytes, st));
    TVQ_CUDA(cudaMemsetAsync(s.base, 0, bytes, st));
    s.cs = reinterpret_cast<CalibState*>(s.base);
    s.mm = reinterpret_cast<uint32_t*>(s.base + 256);
    s.first = reinterpret_cast<float*>(s.base + 264);
    s.hist = reinterpret_cast<unsigned long long*>(s.base + 512);
    s.part = reinterpret_cast<double*>(s.base + 512 + hist_words * 8);
    return TVQ_OK;
}

int absmax_pass(const float* x, int64_t n, CalibScratch& s, cudaStream_t st) {
    int rc = launch_minmax_reset(s.mm, st);
    if (!rc) rc = launch_minmax_accumulate(x, n, s.mm, s.first, st);
    if (!rc) rc = launch_pdl(calib_absmax_kernel, dim3(1), dim3(1), 0, st, static_cast<const uint32_t*>(s.mm), s.cs);
    return rc;
}

// the 4-word result (scale, zero point, min, max) to the caller's device buffer
int copy_out(CalibScratch& s, float* out4, cudaStream_t st) {
    TVQ_CUDA(cudaMemcpyAsync(out4, s.cs->out, 16, cudaMemcpyDeviceToDevice, st));
    return TVQ_OK;
}

}  // namespace

// Results are written to out4 (device): {scale, zero point, min, max}.  When
// max |x| < 1e-8 (KL, MSE) the reference returns calibrate_minmax(data, 1):
// *fallback (host) says so and the caller runs it.
int launch_calibrate_kl(const float* x, int64_t n, int num_bins, int target_bins, float* out4, int* fallback,
                        cudaStream_t st) {
    TVQ_CHECK(n >= 1, TVQ_ERR_SIZE, "no data");
    TVQ_CHECK(num_bins >= 1 && num_bins <= 4096 && target_bins >= 1, TVQ_ERR_UNSUPPORTED,
              "num_bins must be in [1, 4096] and target_bins >= 1");
    const int ncand = (target_bins <= num_bins) ? (num_bins - target_bins) / 16 + 1 : 0;
    TVQ_CHECK(ncand <= 1024, TVQ_ERR_UNSUPPORTED, "at most 1024 candidate thresholds");
    CalibScratch s;
    STEP_RC(calib_alloc(s, static_cast<size_t>(num_bins), 0, st));
    int rc = absmax_pass(x, n, s, st);
    if (!rc) rc = launch_pdl(kl_setup_kernel, dim3(1), dim3(1), 0, st, s.cs, num_bins);
    if (!rc)
        rc = launch_pdl(kl_hist_kernel, dim3(grid_for_calib(n, 256)), dim3(256), sizeof(unsigned int) * num_bins, st, x,
                        n, static_cast<const CalibState*>(s.cs), num_bins, s.hist);
    if (!rc) {
        // ncand == 0: no candidate, the threshold stays num_bins * bw
        const int threads = std::max(32, (std::max(ncand, 1) + 31) / 32 * 32);
        rc = launch_pdl(kl_search_kernel, dim3(1), dim3(threads), sizeof(unsigned long long) * num_bins, st,
                        static_cast<const unsigned long long*>(s.hist), num_bins, target_bins, ncand, s.cs);
    }
    int use_minmax = 0;
    if (!rc) {
        cudaError_t e = cudaMemcpyAsync(&use_minmax, &s.cs->use_minmax, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_fail(e, "calibrate_kl");
    }
    if (!rc && !use_minmax) rc = copy_out(s, out4, st);
    *fallback = use_minmax;
    cudaError_t e = cudaFreeAsync(s.base, st);
    if (!rc && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return rc;
}

int launch_calibrate_percentile(const float* x, int64_t n, float percentile, int symmetric, float* out4,
                                cudaStream_t st) {
    TVQ_CHECK(n >= 1, TVQ_ERR_SIZE, "no data");
    TVQ_CHECK(percentile > 0.0f && percentile <= 100.0f, TVQ_ERR_SIZE, "percentile must be in (0, 100]");
    // rank of the clip: int(min(n - 1, percentile / 100 * n)) in binary64 (engine.tkv:135)
    const double want = static_cast<double>(percentile) / 100.0 * static_cast<double>(n);
    const double nab = static_cast<double>(n - 1);
    const long long idx = static_cast<long long>(nab < want ? nab : want);
    CalibScratch s;
    STEP_RC(calib_alloc(s, 256, 0, st));
    CalibState init{};
    init.k = idx;
    TVQ_CUDA(cudaMemcpyAsync(s.cs, &init, sizeof(init), cudaMemcpyHostToDevice, st));
    int rc = TVQ_OK;
    for (int shift = 24; shift >= 0 && !rc; shift -= 8) {
        rc = launch_pdl(radix_hist_kernel, dim3(grid_for_calib(n, 256)), dim3(256), 0, st, x, n,
                        static_cast<const CalibState*>(s.cs), shift, s.hist);
        if (!rc) rc = launch_pdl(radix_pick_kernel, dim3(1), dim3(1), 0, st, s.hist, shift, s.cs);
    }
    if (!rc) rc = launch_pdl(pct_finish_sym_kernel, dim3(1), dim3(1), 0, st, s.cs);
    if (!rc && !symmetric) {
        rc = launch_minmax_reset(s.mm, st);
        if (!rc)
            rc = launch_pdl(pct_clamped_minmax_kernel, dim3(grid_for_calib(n, 256)), dim3(256), 0, st, x, n,
                            static_cast<const CalibState*>(s.cs), s.mm);
        if (!rc)
            rc = launch_pdl(pct_finish_asym_kernel, dim3(1), dim3(1), 0, st, x, n, static_cast<const uint32_t*>(s.mm),
                            s.cs);
    }
    if (!rc) rc = copy_out(s, out4, st);
    cudaError_t e = cudaFreeAsync(s.base, st);
    if (!rc && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return rc;
}

int launch_calibrate_mse(const float* x, int64_t n, int num_candidates, float* out4, double* curve, int* fallback,
                         cudaStream_t st) {
    TVQ_CHECK(n >= 1, TVQ_ERR_SIZE, "no data");
    if (num_candidates < 4) num_candidates = 4;
    TVQ_CHECK(num_candidates <= 65535, TVQ_ERR_UNSUPPORTED, "too many candidates");
    const int nblk = std::min(grid_for_calib(n, 256), 512);
    CalibScratch s;
    STEP_RC(calib_alloc(s, 0, static_cast<size_t>(nblk) * num_candidates, st));
    int rc = absmax_pass(x, n, s, st);
    if (!rc)
        rc = launch_pdl(mse_partial_kernel, dim3(nblk, num_candidates), dim3(256), 0, st, x, n,
                        static_cast<const CalibState*>(s.cs), num_candidates, s.part);
    if (!rc)
        rc = launch_pdl(mse_pick_kernel, dim3(1), dim3(1), 0, st, static_cast<const double*>(s.part), nblk,
                        num_candidates, n, s.cs, curve);
    int use_minmax = 0;
    if (!rc) {
        cudaError_t e = cudaMemcpyAsync(&use_minmax, &s.cs->use_minmax, sizeof(int), cudaMemcpyDeviceToHost, st);
        if (e == cudaSuccess) e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) rc = cuda_fail(e, "calibrate_mse");
    }
    if (!rc && !use_minmax) rc = copy_out(s, out4, st);
    *fallback = use_minmax;
    cudaError_t e = cudaFreeAsync(s.base, st);
    if (!rc && e != cudaSuccess) return cuda_fail(e, "cudaFreeAsync");
    return rc;
}

}  // namespace tvq
