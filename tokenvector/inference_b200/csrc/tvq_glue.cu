// tvq_glue.cu -- the fp32 parts of a GPT-2-shaped INT8 PTQ forward that sit
// between the quantized linears (tv/training/gpt2_ref.tkv is the model they
// follow): token + position embedding, LayerNorm (float-pair statistics, eps
// from the model), causal multi-head attention over packed ragged sequences, and
// the producers' fused static-scale INT8 quantize of the next linear's input.
//
// Every producer can also record max|y| of its f32 output into a device word
// (calibration), so calibrating a whole stack needs no host round trip.
#include <cuda_fp16.h>

#include "tvq_common.cuh"
#include "tvq_exact.cuh"
#include "tvq_glue.h"

namespace tvq {

namespace {

__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

int sm_count() {
    int rc = 0;
    DeviceState* d = device_state(&rc);
    return d ? d->sm_count : 148;
}

}  // namespace

// ------------------------------------------------------------------ embedding
// gpt2_embed, tv/training/gpt2_ref.tkv:80-88: x[t] = wte[ids[t]] + wpe[pos[t]];
// positions restart at 0 in every packed sequence (pos = t - seg start).
__global__ void embed_kernel(const int64_t* __restrict__ ids, const int* __restrict__ tok_seg_start,
                             const float* __restrict__ wte, const float* __restrict__ wpe, float* __restrict__ x,
                             int T, int d, int vocab, int max_pos, int* err) {
    griddep_wait();
    const int t = blockIdx.x;
    if (t >= T) return;
    int64_t id = ids[t];
    const int pos = t - tok_seg_start[t];
    if (id < 0 || id >= vocab || pos >= max_pos) {
        if (threadIdx.x == 0) atomicCAS(err, 0, 100);  // recorded, row zeroed
        for (int j = threadIdx.x; j < d; j += blockDim.x) x[static_cast<int64_t>(t) * d + j] = 0.0f;
        return;
    }
    const float* a = wte + id * d;
    const float* b = wpe + static_cast<int64_t>(pos) * d;
    float* o = x + static_cast<int64_t>(t) * d;
    for (int j = threadIdx.x; j < d; j += blockDim.x) o[j] = __fadd_rn(a[j], b[j]);
}

int launch_embed(const int64_t* ids, const int* tok_seg_start, const float* wte, const float* wpe, float* x, int T,
                 int d, int vocab, int max_pos, int* err, cudaStream_t st) {
    if (T <= 0) return TVQ_OK;
    return launch_pdl(embed_kernel, dim3(T), dim3(128), 0, st, ids, tok_seg_start, wte, wpe, x, T, d, vocab, max_pos,
                      err);
}

// ------------------------------------------------------------------ layernorm
// (h + l) / n for a small positive integer n, as a float pair (about 2^-46).
__device__ __forceinline__ void df_div_int(float h, float l, float n, float& qh, float& ql) {
    qh = __fdiv_rn(h, n);
    const float rem = fmaf(-qh, n, h);  // h - qh*n, exact
    ql = __fdiv_rn(__fadd_rn(rem, l), n);
}

// 1/sqrt(h + l) as a float pair: rsqrtf plus one Newton step evaluated with
// error-free products (about 2^-44 relative).
__device__ __forceinline__ void df_rsqrt(float h, float l, float& rh, float& rl) {
    const float y = rsqrtf(h);
    const float yy = __fmul_rn(y, y);
    const float yye = fmaf(y, y, -yy);
    const float a = __fmul_rn(h, yy);
    const float ae = fmaf(h, yy, -a);
    const float rest = __fadd_rn(ae, fmaf(h, yye, __fmul_rn(l, yy)));
    const float t = __fsub_rn(__fsub_rn(1.0f, a), rest);  // 1 - (h + l) y^2
    two_sum(y, __fmul_rn(__fmul_rn(0.5f, y), t), rh, rl);
}

// gpt2_layernorm, tv/training/gpt2_ref.tkv:61-78: mean and variance of the
// row, rstd = 1/sqrt(v + eps), out = fl32((x - mu) * rstd * g + b).  The
// reference sums in f64; here the sums are float pairs (error-free two-sum
// per element, pairwise across lanes, about 2^-45 relative), mu / var / rstd
// are float pairs too (no binary64 on the row path), and the output is a
// float pair rounded once.
// It agrees with the f64 oracle except, rarely, by one ulp where the value
// sits next to a rounding midpoint (the oracle's own sequential f64 sum has
// a rounding error of the same kind).  One warp per row.  Outputs: y (f32)
// and/or q (int8 with the static scale), amax of y when requested.
__global__ void layernorm_kernel(const float* __restrict__ x, const float* __restrict__ g,
                                 const float* __restrict__ b, float* __restrict__ y, int8_t* __restrict__ q,
                                 const float* __restrict__ qscale, uint32_t* __restrict__ amax, int T, int d,
                                 double eps) {
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x >> 5;
    InvScale qs{0.0, 0.0f, 0.0f};
    if (q) qs = make_inv_scale(static_cast<double>(__ldg(qscale)));
    const float eps_h = __double2float_rn(eps);
    const float eps_l = __double2float_rn(eps - static_cast<double>(eps_h));
    const float df = static_cast<float>(d);
    float am = 0.0f;
    for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
        const float* xr = x + static_cast<int64_t>(t) * d;
        float sh = 0.0f, sl = 0.0f;
        for (int j = lane; j < d; j += 32) {
            float s, e;
            two_sum(sh, xr[j], s, e);
            sh = s;
            sl = __fadd_rn(sl, e);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float oh = __shfl_xor_sync(0xffffffffu, sh, o), ol = __shfl_xor_sync(0xffffffffu, sl, o);
            df_add(sh, sl, oh, ol, sh, sl);
        }
        float mh, ml;
        df_div_int(sh, sl, df, mh, ml);  // mean as a float pair
        float vh = 0.0f, vl = 0.0f;
        for (int j = lane; j < d; j += 32) {
            float dh, de;
            two_sum(xr[j], -mh, dh, de);
            de = __fsub_rn(de, ml);
            const float p = __fmul_rn(dh, dh);
            float pe = fmaf(dh, dh, -p);
            pe = fmaf(2.0f * dh, de, pe);
            float s, e;
            two_sum(vh, p, s, e);
            vh = s;
            vl = __fadd_rn(vl, __fadd_rn(e, pe));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float oh = __shfl_xor_sync(0xffffffffu, vh, o), ol = __shfl_xor_sync(0xffffffffu, vl, o);
            df_add(vh, vl, oh, ol, vh, vl);
        }
        float wh, wl, rh, rl;
        df_div_int(vh, vl, df, wh, wl);        // variance
        df_add(wh, wl, eps_h, eps_l, wh, wl);  // + eps
        df_rsqrt(wh, wl, rh, rl);              // rstd = 1/sqrt(v + eps)
        for (int j = lane; j < d; j += 32) {
            float dh, de;
            two_sum(xr[j], -mh, dh, de);
            de = __fsub_rn(de, ml);
            const float tt = __fmul_rn(dh, rh);
            float te = fmaf(dh, rh, -tt);
            te = fmaf(dh, rl, te);
            te = fmaf(de, rh, te);
            const float gj = __ldg(g + j);
            const float u = __fmul_rn(tt, gj);
            float ue = fmaf(tt, gj, -u);
            ue = fmaf(te, gj, ue);
            float s, e;
            two_sum(u, __ldg(b + j), s, e);
            const float of = __fadd_rn(s, __fadd_rn(e, ue));
            const int64_t idx = static_cast<int64_t>(t) * d + j;
            if (y) y[idx] = of;
            if (q) {
                int8_t qq;
                if (!quant_fast(of, qs, qq)) qq = quant_slow(of, qs.d);
                q[idx] = qq;
            }
            am = fmaxf(am, fabsf(of));
        }
    }
    if (amax) {
        am = warp_max_f(am);
        if (lane == 0) atomicMax(amax, __float_as_uint(am));
    }
}

// Row-parallel variants for d % 4 == 0 (16-byte aligned rows): WPR warps
// share a row (WPR = LNW: a block per row, for few rows; WPR = 1: a warp
// per row, four rows per block, for many rows -- no block barrier between
// the rows of a warp), each thread holding NV float4 of it in registers; the
// float-pair partial sums are reduced over the warp by shuffles and, with
// WPR > 1, over the block through shared memory in a fixed order.  Same
// arithmetic as layernorm_kernel (only the summation order differs).
constexpr int LNW = 4;

__device__ __forceinline__ void ln_block_sum(float& h, float& l, float2* red, int lane, int warp) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oh = __shfl_xor_sync(0xffffffffu, h, o), ol = __shfl_xor_sync(0xffffffffu, l, o);
        df_add(h, l, oh, ol, h, l);
    }
    if (lane == 0) red[warp] = make_float2(h, l);
    __syncthreads();
    float2 t = red[0];
    h = t.x;
    l = t.y;
#pragma unroll
    for (int w = 1; w < LNW; w++) {
        t = red[w];
        df_add(h, l, t.x, t.y, h, l);
    }
}

__device__ __forceinline__ void ln_warp_sum(float& h, float& l) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float oh = __shfl_xor_sync(0xffffffffu, h, o), ol = __shfl_xor_sync(0xffffffffu, l, o);
        df_add(h, l, oh, ol, h, l);
    }
}

__device__ __forceinline__ double ln_warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over the LNW warps of a block (red: LNW slots, reused after the
// barrier that ends the row).
__device__ __forceinline__ double ln_block_sum_d(double v, double* red, int lane, int warp) {
    v = ln_warp_sum_d(v);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    double t = red[0];
#pragma unroll
    for (int w = 1; w < LNW; w++) t = __dadd_rn(t, red[w]);
    return t;
}

// SPLIT: the output goes out as the LM head's operand instead, the row-scaled
// fp16 split of launch_split_f16_rows (hi, lo [T, d], rscale [T]).
template <int NV, int WPR, bool SPLIT = false>
__global__ void __launch_bounds__(32 * LNW)
    layernorm_block_kernel(const float* __restrict__ x, const float* __restrict__ g, const float* __restrict__ b,
                           float* __restrict__ y, int8_t* __restrict__ q, const float* __restrict__ qscale,
                           uint32_t* __restrict__ amax, int T, int d, double eps, __half* __restrict__ shi = nullptr,
                           __half* __restrict__ slo = nullptr, float* __restrict__ srs = nullptr) {
    griddep_wait();
    __shared__ float2 red[2][LNW];
    __shared__ double redd[2][LNW];
    constexpr int RPB = LNW / WPR;  // rows per block per pass
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int tid = (WPR == 1) ? lane : static_cast<int>(threadIdx.x);  // thread index within its row
    const int d4 = d >> 2;
    InvScale qs{0.0, 0.0f, 0.0f};
    if (q) qs = make_inv_scale(static_cast<double>(__ldg(qscale)));
    const float4* g4 = reinterpret_cast<const float4*>(g);
    const float4* b4 = reinterpret_cast<const float4*>(b);
    float am = 0.0f;
    constexpr bool KEEP = 4 * NV <= 24;  // x in binary64 registers, else converted again
    // a warp per row with x kept in binary64: the next row's loads are issued
    // once this row's values have been copied out of v (a warp then has two
    // rows in flight, which its registers would not allow otherwise)
    constexpr bool PREFETCH = WPR == 1 && KEEP;
    const int tstep = static_cast<int>(gridDim.x) * RPB;
    float4 v[NV];
    auto load_row = [&](int tt) {
        const float4* xr = reinterpret_cast<const float4*>(x + static_cast<int64_t>(tt) * d);
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const int i = j * 32 * WPR + tid;
            v[j] = (i < d4) ? __ldcs(xr + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    };
    const int t0 = static_cast<int>(blockIdx.x) * RPB + (WPR == 1 ? warp : 0);
    if (PREFETCH && t0 < T) load_row(t0);
    for (int t = t0; t < T; t += tstep) {
        if (!PREFETCH) load_row(t);
        // statistics in binary64 as the reference (gpt2_ref.tkv:61-78):
        // mu = sum x / d, var = sum (x - mu)^2 / d, rstd = 1 / sqrt(var + eps),
        // y = fl32(((x - mu) * rstd) * g + b) (B200 runs FP64 at half the FP32
        // rate); the sums run as a tree instead of the reference's sequence.
        // Slots past the row hold 0 and add nothing to the sum.
        double xd[KEEP ? 4 * NV : 1];
        double sum = 0.0;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const double a0 = v[j].x, a1 = v[j].y, a2 = v[j].z, a3 = v[j].w;
            if constexpr (KEEP) {
                xd[4 * j] = a0;
                xd[4 * j + 1] = a1;
                xd[4 * j + 2] = a2;
                xd[4 * j + 3] = a3;
            }
            sum = __dadd_rn(sum, __dadd_rn(__dadd_rn(a0, a1), __dadd_rn(a2, a3)));
        }
        if (PREFETCH && t + tstep < T) load_row(t + tstep);  // v is not read again for this row
        if constexpr (WPR == 1) sum = ln_warp_sum_d(sum);
        else sum = ln_block_sum_d(sum, redd[0], lane, warp);
        // element k of float4 j in binary64 (kept, or converted again)
        auto x_at = [&](int j, int k) -> double {
            if constexpr (KEEP) {
                return xd[4 * j + k];
            } else {
                return static_cast<double>(k == 0 ? v[j].x : k == 1 ? v[j].y : k == 2 ? v[j].z : v[j].w);
            }
        };
        const double mu = sum / static_cast<double>(d);
        double ss = 0.0;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            if (j * 32 * WPR + tid >= d4) continue;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const double dd = __dsub_rn(x_at(j, k), mu);
                ss = __fma_rn(dd, dd, ss);
            }
        }
        if constexpr (WPR == 1) ss = ln_warp_sum_d(ss);
        else ss = ln_block_sum_d(ss, redd[1], lane, warp);
        const double rstd = 1.0 / sqrt(__dadd_rn(ss / static_cast<double>(d), eps));
        float4 ov[SPLIT ? NV : 1];
        float rmax = 0.0f;
        bool bad = false;
#pragma unroll
        for (int j = 0; j < NV; j++) {
            const int i = j * 32 * WPR + tid;
            if (i >= d4) continue;
            const float4 gg = __ldg(g4 + i), bb = __ldg(b4 + i);
            const float gk[4] = {gg.x, gg.y, gg.z, gg.w}, bk[4] = {bb.x, bb.y, bb.z, bb.w};
            float o4[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const double t = __dmul_rn(__dmul_rn(__dsub_rn(x_at(j, k), mu), rstd), static_cast<double>(gk[k]));
                o4[k] = __double2float_rn(__dadd_rn(t, static_cast<double>(bk[k])));
            }
#pragma unroll
            for (int k = 0; k < 4; k++) am = fmaxf(am, fabsf(o4[k]));
            if constexpr (SPLIT) {
                ov[j] = make_float4(o4[0], o4[1], o4[2], o4[3]);
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    rmax = fmaxf(rmax, fabsf(o4[k]));
                    bad |= !isfinite(o4[k]);
                }
                continue;
            }
            const int64_t idx = static_cast<int64_t>(t) * d + 4 * i;
            if (y) *reinterpret_cast<float4*>(y + idx) = make_float4(o4[0], o4[1], o4[2], o4[3]);
            if (q) {
                float t0, t1, t2, t3;
                const bool ok = quant_fast_t(o4[0], qs.hi, t0) & quant_fast_t(o4[1], qs.hi, t1) &
                                quant_fast_t(o4[2], qs.hi, t2) & quant_fast_t(o4[3], qs.hi, t3);
                if (ok) {
                    *reinterpret_cast<uint32_t*>(q + idx) = pack_q4(t0, t1, t2, t3);
                } else {
                    char4 qq;
                    qq.x = quant_exact(o4[0], qs);
                    qq.y = quant_exact(o4[1], qs);
                    qq.z = quant_exact(o4[2], qs);
                    qq.w = quant_exact(o4[3], qs);
                    *reinterpret_cast<char4*>(q + idx) = qq;
                }
            }
        }
        if constexpr (SPLIT) {
            // the row's largest |y| (red[0] is free: every thread has read the mean)
            rmax = warp_max_f(rmax);
            bad = __any_sync(0xffffffffu, bad);
            if constexpr (WPR > 1) {
                if (lane == 0) red[0][warp] = make_float2(rmax, bad ? 1.0f : 0.0f);
                __syncthreads();
#pragma unroll
                for (int w = 0; w < LNW; w++) {
                    rmax = fmaxf(rmax, red[0][w].x);
                    bad |= red[0][w].y != 0.0f;
                }
            }
            // as split_f16_rows_kernel: s with max|y| 2^s in [2^14, 2^15), 1 for a non-finite row
            int sh = 0;
            if (!bad && rmax > 0.0f) {
                int e;
                frexpf(rmax, &e);
                sh = min(15 - e, 126);
            }
            if (tid == 0) srs[t] = exp2i(-sh);
            const float f = exp2i(sh);
#pragma unroll
            for (int j = 0; j < NV; j++) {
                const int i = j * 32 * WPR + tid;
                if (i >= d4) continue;
                const float vv[4] = {ov[j].x * f, ov[j].y * f, ov[j].z * f, ov[j].w * f};
                __half h[4], l[4];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    h[k] = __float2half_rn(vv[k]);
                    l[k] = __float2half_rn(__fsub_rn(vv[k], __half2float(h[k])));
                }
                const int64_t idx = static_cast<int64_t>(t) * d + 4 * i;
                *reinterpret_cast<uint2*>(shi + idx) = make_uint2(
                    static_cast<uint32_t>(__half_as_ushort(h[0])) | (static_cast<uint32_t>(__half_as_ushort(h[1])) << 16),
                    static_cast<uint32_t>(__half_as_ushort(h[2])) | (static_cast<uint32_t>(__half_as_ushort(h[3])) << 16));
                *reinterpret_cast<uint2*>(slo + idx) = make_uint2(
                    static_cast<uint32_t>(__half_as_ushort(l[0])) | (static_cast<uint32_t>(__half_as_ushort(l[1])) << 16),
                    static_cast<uint32_t>(__half_as_ushort(l[2])) | (static_cast<uint32_t>(__half_as_ushort(l[3])) << 16));
            }
        }
        if constexpr (WPR > 1) __syncthreads();  // red is reused by the next row
    }
    if (amax) {
        am = warp_max_f(am);
        if (lane == 0) atomicMax(amax, __float_as_uint(am));
    }
}

int launch_layernorm_split(const float* x, const float* g, const float* b, void* hi, void* lo, float* rscale, int T,
                           int d, double eps, cudaStream_t st) {
    if (T <= 0) return TVQ_OK;
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(b) |
                         reinterpret_cast<uintptr_t>(hi) | reinterpret_cast<uintptr_t>(lo);
    const int nv = (d / 4 + 32 * LNW - 1) / (32 * LNW);
    TVQ_CHECK((d & 3) == 0 && (al & 15) == 0 && nv <= 4, TVQ_ERR_UNSUPPORTED,
              "the fused LayerNorm + split needs d % 4 == 0, d <= 2048 and 16-byte aligned buffers");
    const int bgrid = std::min(T, sm_count() * 16);
#define TVQ_LNS(NV)                                                                                                   \
    launch_pdl(layernorm_block_kernel<NV, LNW, true>, dim3(bgrid), dim3(32 * LNW), 0, st, x, g, b,                    \
               static_cast<float*>(nullptr), static_cast<int8_t*>(nullptr), static_cast<const float*>(nullptr),        \
               static_cast<uint32_t*>(nullptr), T, d, eps, static_cast<__half*>(hi), static_cast<__half*>(lo), rscale)
    if (nv <= 1) return TVQ_LNS(1);
    if (nv <= 2) return TVQ_LNS(2);
    return TVQ_LNS(4);
#undef TVQ_LNS
}

int launch_layernorm(const float* x, const float* g, const float* b, float* y, int8_t* q, const float* qscale,
                     uint32_t* amax, int T, int d, double eps, cudaStream_t st) {
    if (T <= 0) return TVQ_OK;
    const int threads = 128;
    const int rows_per_block = threads / 32;
    int grid = (T + rows_per_block - 1) / rows_per_block;
    grid = std::min(grid, sm_count() * 16);
    const uintptr_t al = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(g) |
                         reinterpret_cast<uintptr_t>(b) | (y ? reinterpret_cast<uintptr_t>(y) : 0) |
                         (q ? reinterpret_cast<uintptr_t>(q) & 3 : 0);
    // a warp per row once there are many more rows than a block-per-row grid
    // holds at once (TVQ_LN_WARP=0/1 forces the choice: tuning)
    static const int env_warp = [] {
        const char* e = getenv("TVQ_LN_WARP");
        return e ? atoi(e) : -1;
    }();
    const int nvw = (d / 4 + 31) / 32;
    const bool warp_rows = (env_warp >= 0) ? env_warp != 0 : (T >= 4 * sm_count() * 16 && nvw <= 16);
    const int nv = warp_rows ? nvw : (d / 4 + 32 * LNW - 1) / (32 * LNW);
    if ((d & 3) == 0 && (al & 15) == 0 && nv <= 16) {
        __half* nh = nullptr;  // no split output
        float* nf = nullptr;
        const int rpb = warp_rows ? LNW : 1;
        const int bgrid = std::min((T + rpb - 1) / rpb, sm_count() * 16);
#define TVQ_LN(NV)                                                                                                  \
    (warp_rows ? launch_pdl(layernorm_block_kernel<NV, 1>, dim3(bgrid), dim3(32 * LNW), 0, st, x, g, b, y, q, qscale, \
                            amax, T, d, eps, nh, nh, nf)                                                             \
               : launch_pdl(layernorm_block_kernel<NV, LNW>, dim3(bgrid), dim3(32 * LNW), 0, st, x, g, b, y, q,     \
                            qscale, amax, T, d, eps, nh, nh, nf))
        if (nv <= 1) return TVQ_LN(1);
        if (nv <= 2) return TVQ_LN(2);
        if (nv <= 4) return TVQ_LN(4);
        if (nv <= 6) return TVQ_LN(6);    // d 768, a warp per row
        if (nv <= 8) return TVQ_LN(8);
        if (nv <= 13) return TVQ_LN(13);  // d 1600, a warp per row
        return TVQ_LN(16);
#undef TVQ_LN
    } else {
        return launch_pdl(layernorm_kernel, dim3(grid), dim3(threads), 0, st, x, g, b, y, q, qscale, amax, T, d, eps);
    }
}

// ------------------------------------------------------------------ attention
// gpt2_attention, tv/training/gpt2_ref.tkv:360-395 (scores -> causal softmax
// -> context), per head, over packed sequences: token t of the sequence
// [s0, s1) attends to u in [s0, t].  qkv rows are [Q | K | V], heads
// contiguous.  fp32 flash-style tiling with an online softmax in base 2
// (log2(e) / sqrt(hd) folded into Q).  A block of 128 threads owns 64 query
// rows of one head and one chunk of keys; thread (ty, tx) holds rows
// 4ty..4ty+3, keys tx, tx+8, ..., tx+56 of each 64-key tile (strided, so the
// K reads are conflict-free) and output columns tx*HD/8...  Row-major Q, K, V
// and P tiles in shared memory, float4 loads throughout.
//
// Work items: tiles[i] = {q0, seq start, seq end, 0}; with split[i] =
// {key begin, key end, partial slot, 0} a block handles one key chunk and,
// when the slot is >= 0, writes an unnormalised partial (O, m, l) that
// attention_combine_kernel merges; without split the chunk is the whole
// causal range and the output is final.
namespace {
constexpr int AQ = 64;   // query rows per block
constexpr int AK = 64;   // keys per tile
constexpr int APAD = 4;  // row padding (floats) of the shared tiles
constexpr int ATHREADS = 128;
}  // namespace

template <int HD>
__global__ void __launch_bounds__(ATHREADS)
    attention_kernel(const float* __restrict__ qkv, const int4* __restrict__ tiles, const int4* __restrict__ split,
                     int d, int nheads, float q_scale, float* __restrict__ out, int8_t* __restrict__ outq,
                     const float* __restrict__ qscale, uint32_t* __restrict__ amax, float* __restrict__ part_o,
                     float2* __restrict__ part_ml) {
    griddep_wait();
    static_assert(HD % 16 == 0 && HD <= 64, "head dim");
    constexpr int LD = HD + APAD;   // row pitch of Q, K, V tiles
    constexpr int PLD = AK + APAD;  // row pitch of P
    constexpr int DPT = HD / 8;     // output columns per thread
    extern __shared__ float sm[];
    float* Qs = sm;             // [AQ][LD]
    float* Ks = Qs + AQ * LD;   // [AK][LD]
    float* Vs = Ks + AK * LD;   // [AK][LD]
    float* Ps = Vs + AK * LD;   // [AQ][PLD]

    const int item = blockIdx.x / nheads;
    const int head = blockIdx.x % nheads;
    const int4 tl = tiles[item];
    const int q0 = tl.x, s0 = tl.y, s1 = tl.z;
    int kb = s0, ke = min(q0 + AQ, s1), part = -1;
    if (split) {
        const int4 sp = split[item];
        kb = sp.x;
        ke = sp.y;
        part = sp.z;
    }
    const int tid = threadIdx.x;
    const int ty = tid >> 3, tx = tid & 7;
    const int64_t rs = 3LL * d;
    const int qoff = head * HD, koff = d + head * HD, voff = 2 * d + head * HD;
    constexpr int V4 = HD / 4;

    for (int i = tid; i < AQ * V4; i += ATHREADS) {
        const int r = i / V4, c = (i % V4) * 4;
        const int t = q0 + r;
        float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (t < s1) {
            v = *reinterpret_cast<const float4*>(qkv + t * rs + qoff + c);
            v.x *= q_scale; v.y *= q_scale; v.z *= q_scale; v.w *= q_scale;
        }
        *reinterpret_cast<float4*>(&Qs[r * LD + c]) = v;
    }

    float o[4][DPT];
    float mrow[4], lrow[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        mrow[i] = -INFINITY;
        lrow[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < DPT; j++) o[i][j] = 0.0f;
    }

    for (int k0 = kb; k0 < ke; k0 += AK) {
        __syncthreads();  // previous tile's K / V / P consumed
        for (int i = tid; i < AK * V4; i += ATHREADS) {
            const int r = i / V4, c = (i % V4) * 4;
            const int u = k0 + r;
            float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f), vv = kv;
            if (u < ke) {
                kv = *reinterpret_cast<const float4*>(qkv + u * rs + koff + c);
                vv = *reinterpret_cast<const float4*>(qkv + u * rs + voff + c);
            }
            *reinterpret_cast<float4*>(&Ks[r * LD + c]) = kv;
            *reinterpret_cast<float4*>(&Vs[r * LD + c]) = vv;
        }
        __syncthreads();

        float s[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) s[i][j] = 0.0f;
#pragma unroll 2
        for (int c = 0; c < HD; c += 4) {
            float4 qa[4], kf[8];
#pragma unroll
            for (int i = 0; i < 4; i++) qa[i] = *reinterpret_cast<const float4*>(&Qs[(4 * ty + i) * LD + c]);
#pragma unroll
            for (int j = 0; j < 8; j++) kf[j] = *reinterpret_cast<const float4*>(&Ks[(tx + 8 * j) * LD + c]);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    s[i][j] = fmaf(qa[i].x, kf[j].x, s[i][j]);
                    s[i][j] = fmaf(qa[i].y, kf[j].y, s[i][j]);
                    s[i][j] = fmaf(qa[i].z, kf[j].z, s[i][j]);
                    s[i][j] = fmaf(qa[i].w, kf[j].w, s[i][j]);
                }
        }

        // causal mask + online softmax; a row's 64 keys are spread over the
        // 8 consecutive lanes tx = 0..7
        float alpha[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = q0 + 4 * ty + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int u = k0 + tx + 8 * j;
                s[i][j] = (u <= t && u < ke) ? s[i][j] : -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            const float mnew = fmaxf(mrow[i], mx);
            const float mref = (mnew == -INFINITY) ? 0.0f : mnew;  // rows with no key yet stay empty
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const float pexp = exp2f(s[i][j] - mref);
                s[i][j] = pexp;
                sum += pexp;
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            alpha[i] = exp2f(mrow[i] - mref);  // 0 while mrow is -inf
            lrow[i] = lrow[i] * alpha[i] + sum;
            mrow[i] = mnew;
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) Ps[(4 * ty + i) * PLD + tx + 8 * j] = s[i][j];
        __syncthreads();

#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < DPT; j++) o[i][j] *= alpha[i];
        const int kmax = min(AK, ke - k0);
        for (int u = 0; u < kmax; u += 4) {
            float4 pa[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pa[i] = *reinterpret_cast<const float4*>(&Ps[(4 * ty + i) * PLD + u]);
#pragma unroll
            for (int uu = 0; uu < 4; uu++) {
                float vv[DPT];
#pragma unroll
                for (int j = 0; j < DPT; j += 2) {
                    const float2 t2 = *reinterpret_cast<const float2*>(&Vs[(u + uu) * LD + tx * DPT + j]);
                    vv[j] = t2.x;
                    vv[j + 1] = t2.y;
                }
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float pv = uu == 0 ? pa[i].x : uu == 1 ? pa[i].y : uu == 2 ? pa[i].z : pa[i].w;
#pragma unroll
                    for (int j = 0; j < DPT; j++) o[i][j] = fmaf(pv, vv[j], o[i][j]);
                }
            }
        }
    }

    if (part >= 0) {  // unnormalised partial for the combine step
        const int64_t slot = static_cast<int64_t>(part) * nheads + head;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = 4 * ty + i;
            float* dst = part_o + (slot * AQ + r) * HD + tx * DPT;
#pragma unroll
            for (int j = 0; j < DPT; j++) dst[j] = o[i][j];
            if (tx == 0) part_ml[slot * AQ + r] = make_float2(mrow[i], lrow[i]);
        }
        return;
    }
    InvScale qs{0.0, 0.0f, 0.0f};
    if (outq) qs = make_inv_scale(static_cast<double>(__ldg(qscale)));
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = q0 + 4 * ty + i;
        if (t >= s1) continue;
        const float il = 1.0f / lrow[i];
        const int64_t base = static_cast<int64_t>(t) * d + head * HD + tx * DPT;
#pragma unroll
        for (int j = 0; j < DPT; j++) {
            const float v = o[i][j] * il;
            if (out) out[base + j] = v;
            if (outq) outq[base + j] = quant_exact(v, qs);
            am = fmaxf(am, fabsf(v));
        }
    }
    if (amax) {
        am = warp_max_f(am);
        if ((tid & 31) == 0) atomicMax(amax, __float_as_uint(am));
    }
}

// Merge the key-chunk partials of one (query tile of QR rows, head):
// m = max m_c, l = sum l_c 2^(m_c - m), O = sum O_c 2^(m_c - m) / l.  Two
// threads per row, each owning HD/2 output columns.
template <int HD, int QR>
__global__ void __launch_bounds__(QR * 2)
    attention_combine_kernel(const int4* __restrict__ comb, int d, int nheads, const float* __restrict__ part_o,
                             const float2* __restrict__ part_ml, float* __restrict__ out, int8_t* __restrict__ outq,
                             const float* __restrict__ qscale, uint32_t* __restrict__ amax) {
    griddep_wait();
    constexpr int HC = HD / 2;
    const int e = blockIdx.x / nheads;
    const int head = blockIdx.x % nheads;
    const int4 c = comb[e];  // {q0, seq end, first partial slot, number of partials}
    const int q0 = c.x, s1 = c.y, first = c.z, np = c.w;
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    const int t = q0 + r;
    float am = 0.0f;
    if (t < s1) {
        float m = -INFINITY;
        for (int k = 0; k < np; k++)
            m = fmaxf(m, part_ml[(static_cast<int64_t>(first + k) * nheads + head) * QR + r].x);
        float l = 0.0f, acc[HC];
#pragma unroll
        for (int j = 0; j < HC; j++) acc[j] = 0.0f;
        for (int k = 0; k < np; k++) {
            const int64_t slot = static_cast<int64_t>(first + k) * nheads + head;
            const float2 ml = part_ml[slot * QR + r];
            const float w = (ml.x == -INFINITY) ? 0.0f : exp2f(ml.x - m);
            l = fmaf(ml.y, w, l);
            const float4* src = reinterpret_cast<const float4*>(part_o + (slot * QR + r) * HD + half * HC);
#pragma unroll
            for (int j = 0; j < HC / 4; j++) {
                const float4 v = src[j];
                acc[4 * j] = fmaf(v.x, w, acc[4 * j]);
                acc[4 * j + 1] = fmaf(v.y, w, acc[4 * j + 1]);
                acc[4 * j + 2] = fmaf(v.z, w, acc[4 * j + 2]);
                acc[4 * j + 3] = fmaf(v.w, w, acc[4 * j + 3]);
            }
        }
        InvScale qs{0.0, 0.0f, 0.0f};
        if (outq) qs = make_inv_scale(static_cast<double>(__ldg(qscale)));
        const int64_t o = static_cast<int64_t>(t) * d + head * HD + half * HC;
#pragma unroll
        for (int j = 0; j < HC; j++) {
            const float v = acc[j] / l;
            if (out) out[o + j] = v;
            if (outq) outq[o + j] = quant_exact(v, qs);
            am = fmaxf(am, fabsf(v));
        }
    }
    if (amax) {
        am = warp_max_f(am);
        if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(am));
    }
}

template <int HD>
static int launch_combine_hd(const int4* comb, int ncomb, int d, int nheads, int rows, const float* part_o,
                             const float2* part_ml, float* out, int8_t* outq, const float* qscale, uint32_t* amax,
                             cudaStream_t st) {
    if (rows == 64)
        return launch_pdl(attention_combine_kernel<HD, 64>, dim3(ncomb * nheads), dim3(128), 0, st, comb, d, nheads,
                          part_o, part_ml, out, outq, qscale, amax);
    return launch_pdl(attention_combine_kernel<HD, 128>, dim3(ncomb * nheads), dim3(256), 0, st, comb, d, nheads,
                      part_o, part_ml, out, outq, qscale, amax);
}

int launch_attention_combine(const int4* comb, int ncomb, int d, int nheads, int rows, const float* part_o,
                             const float2* part_ml, float* out, int8_t* outq, const float* qscale, uint32_t* amax,
                             cudaStream_t st) {
    if (ncomb <= 0) return TVQ_OK;
    TVQ_CHECK(rows == 64 || rows == 128, TVQ_ERR_INVALID, "query tiles are 64 or 128 rows");
    switch (d / nheads) {
        case 16: return launch_combine_hd<16>(comb, ncomb, d, nheads, rows, part_o, part_ml, out, outq, qscale, amax, st);
        case 32: return launch_combine_hd<32>(comb, ncomb, d, nheads, rows, part_o, part_ml, out, outq, qscale, amax, st);
        case 48: return launch_combine_hd<48>(comb, ncomb, d, nheads, rows, part_o, part_ml, out, outq, qscale, amax, st);
        case 64: return launch_combine_hd<64>(comb, ncomb, d, nheads, rows, part_o, part_ml, out, outq, qscale, amax, st);
        default:
            set_error(TVQ_ERR_UNSUPPORTED, "head dim must be 16, 32, 48 or 64");
            return TVQ_ERR_UNSUPPORTED;
    }
}

template <int HD>
static int launch_attention_hd(const float* qkv, const int4* tiles, const int4* split, int nitems, const int4* comb,
                               int ncomb, int d, int nheads, float* out, int8_t* outq, const float* qscale,
                               uint32_t* amax, float* part_o, float2* part_ml, cudaStream_t st) {
    constexpr size_t smem = sizeof(float) * (3 * AQ * (HD + APAD) + AQ * (AK + APAD));
    static bool attr[64] = {false};
    int dev = 0;
    TVQ_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !attr[dev]) {
        TVQ_CUDA(cudaFuncSetAttribute(attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
        attr[dev] = true;
    }
    // softmax in base 2: scores scaled by log2(e)/sqrt(hd) through Q
    const float q_scale = static_cast<float>(1.4426950408889634 / sqrt(static_cast<double>(HD)));
    const int lrc = launch_pdl(attention_kernel<HD>, dim3(nitems * nheads), dim3(ATHREADS), smem, st, qkv, tiles,
                               split, d, nheads, q_scale, out, outq, qscale, amax, part_o, part_ml);
    if (lrc) return lrc;
    if (ncomb > 0)
        return launch_combine_hd<HD>(comb, ncomb, d, nheads, AQ, part_o, part_ml, out, outq, qscale, amax, st);
    return TVQ_OK;
}

int launch_attention_split(const float* qkv, const int4* tiles, const int4* split, int nitems, const int4* comb,
                           int ncomb, int d, int nheads, float* out, int8_t* outq, const float* qscale,
                           uint32_t* amax, float* part_o, float2* part_ml, cudaStream_t st) {
    if (nitems <= 0) return TVQ_OK;
    TVQ_CHECK(nheads > 0 && d % nheads == 0, TVQ_ERR_INVALID, "d must be a multiple of the head count");
    const int hd = d / nheads;
    switch (hd) {
        case 16: return launch_attention_hd<16>(qkv, tiles, split, nitems, comb, ncomb, d, nheads, out, outq, qscale, amax, part_o, part_ml, st);
        case 32: return launch_attention_hd<32>(qkv, tiles, split, nitems, comb, ncomb, d, nheads, out, outq, qscale, amax, part_o, part_ml, st);
        case 48: return launch_attention_hd<48>(qkv, tiles, split, nitems, comb, ncomb, d, nheads, out, outq, qscale, amax, part_o, part_ml, st);
        case 64: return launch_attention_hd<64>(qkv, tiles, split, nitems, comb, ncomb, d, nheads, out, outq, qscale, amax, part_o, part_ml, st);
        default:
            set_error(TVQ_ERR_UNSUPPORTED, "head dim must be 16, 32, 48 or 64");
            return TVQ_ERR_UNSUPPORTED;
    }
}

int launch_attention(const float* qkv, const int4* tiles, int ntiles, int T, int d, int nheads, float* out,
                     int8_t* outq, const float* qscale, uint32_t* amax, cudaStream_t st) {
    (void)T;
    return launch_attention_split(qkv, tiles, nullptr, ntiles, nullptr, 0, d, nheads, out, outq, qscale, amax, nullptr,
                                  nullptr, st);
}

// ------------------------------------------------------------------ scales
// calibrate_minmax symmetric (tv/quantization/engine.tkv:24-30) from a
// recorded amax: scale = fl32(max(amax, 1e-8) / 127).
__global__ void scale_from_amax_kernel(const uint32_t* __restrict__ amax, float* __restrict__ scale, int n) {
    griddep_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    scale[i] = scale_from_amax_bits(amax[i]);
}

int launch_scale_from_amax(const uint32_t* amax, float* scale, int n, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    return launch_pdl(scale_from_amax_kernel, dim3((n + 127) / 128), dim3(128), 0, st, amax, scale, n);
}

// [k, n] (HF Conv1D layout) -> [n, k]
__global__ void transpose_kernel(const float* __restrict__ a, float* __restrict__ b, int rows, int cols) {
    __shared__ float tile[32][33];
    const int c = blockIdx.x * 32 + threadIdx.x;
    const int r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i;
        tile[i][threadIdx.x] = (r < rows && c < cols) ? a[static_cast<int64_t>(r) * cols + c] : 0.0f;
    }
    __syncthreads();
    const int oc = r0 + threadIdx.x;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int orow = blockIdx.x * 32 + i;
        if (orow < cols && oc < rows) b[static_cast<int64_t>(orow) * rows + oc] = tile[threadIdx.x][i];
    }
}

int launch_transpose(const float* a, float* b, int rows, int cols, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return TVQ_OK;
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    transpose_kernel<<<grid, block, 0, st>>>(a, b, rows, cols);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// per-token start of its packed sequence
__global__ void token_seg_kernel(const int* __restrict__ seg, int nseg, int* __restrict__ tok_start) {
    const int s = blockIdx.x;
    if (s >= nseg) return;
    for (int t = seg[s] + threadIdx.x; t < seg[s + 1]; t += blockDim.x) tok_start[t] = seg[s];
}

int launch_token_seg(const int* seg, int nseg, int* tok_start, cudaStream_t st) {
    if (nseg <= 0) return TVQ_OK;
    token_seg_kernel<<<nseg, 256, 0, st>>>(seg, nseg, tok_start);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// last token of every sequence: rows seg[s+1]-1 of a [T, n] matrix
__global__ void gather_last_kernel(const float* __restrict__ src, const int* __restrict__ seg, int nseg, int64_t n,
                                   float* __restrict__ dst) {
    griddep_wait();
    const int s = blockIdx.y;
    if (s >= nseg) return;
    const int64_t row = seg[s + 1] - 1;
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x)
        dst[s * n + j] = src[row * n + j];
}

int launch_gather_last(const float* src, const int* seg, int nseg, int64_t n, float* dst, cudaStream_t st) {
    if (nseg <= 0) return TVQ_OK;
    dim3 grid(static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 64)), nseg);
    return launch_pdl(gather_last_kernel, grid, dim3(256), 0, st, src, seg, nseg, n, dst);
}

}  // namespace tvq
