// tvq_glue.cu -- the fp32 parts of a GPT-2-shaped INT8 PTQ forward that sit
// between the quantized linears (tv/training/gpt2_ref.tkv is the model they
// follow): token + position embedding, LayerNorm (float-pair statistics, eps
// from the model), causal multi-head attention over packed ragged sequences, and
// the producers' fused static-scale INT8 quantize of the next linear's input.
//
// Every producer can also record max|y| of its f32 output into a device word
// (calibration), so calibrating a whole stack needs no host round trip.
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
    embed_kernel<<<T, 128, 0, st>>>(ids, tok_seg_start, wte, wpe, x, T, d, vocab, max_pos, err);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
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

int launch_layernorm(const float* x, const float* g, const float* b, float* y, int8_t* q, const float* qscale,
                     uint32_t* amax, int T, int d, double eps, cudaStream_t st) {
    if (T <= 0) return TVQ_OK;
    const int threads = 128;
    const int rows_per_block = threads / 32;
    int grid = (T + rows_per_block - 1) / rows_per_block;
    grid = std::min(grid, sm_count() * 16);
    layernorm_kernel<<<grid, threads, 0, st>>>(x, g, b, y, q, qscale, amax, T, d, eps);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

// ------------------------------------------------------------------ attention
// gpt2_attention, tv/training/gpt2_ref.tkv:360-395 (scores -> causal softmax
// -> context), per head, over packed sequences: token t of the sequence
// [s0, s1) attends to u in [s0, t].  qkv rows are [Q | K | V], heads
// contiguous.  fp32 flash-style tiling: a block owns BQ=64 query rows of one
// head, walks the key tiles up to the diagonal with an online softmax.
// 256 threads: thread (ty, tx) holds rows 4ty..4ty+3 and columns 4tx..4tx+3
// of the 64x64 score tile and of the 64 x HD output tile.
namespace {
constexpr int AQ = 64;   // query rows per block
constexpr int AK = 64;   // key rows per tile
constexpr int APAD = 4;
}

template <int HD>
__global__ void __launch_bounds__(256)
    attention_kernel(const float* __restrict__ qkv, const int4* __restrict__ tiles, int ntiles, int T, int d,
                     int nheads, float sm_scale, float* __restrict__ out, int8_t* __restrict__ outq,
                     const float* __restrict__ qscale, uint32_t* __restrict__ amax) {
    static_assert(HD % 16 == 0 && HD <= 64, "head dim");
    constexpr int CPT = HD / 16;  // output columns per thread
    extern __shared__ float sm[];
    float* Qt = sm;                         // [HD][AQ+APAD]   Q^T
    float* Kt = Qt + HD * (AQ + APAD);      // [HD][AK+APAD]   K^T
    float* Vs = Kt + HD * (AK + APAD);      // [AK][HD]
    float* Pt = Vs + AK * HD;               // [AK][AQ+APAD]   P^T

    const int tile_id = blockIdx.x / nheads;
    const int head = blockIdx.x % nheads;
    if (tile_id >= ntiles) return;
    const int4 tl = tiles[tile_id];  // {q0, seg start, seg end, unused}
    const int q0 = tl.x, s0 = tl.y, s1 = tl.z;
    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    const int64_t row_stride = 3LL * d;
    const int qoff = head * HD, koff = d + head * HD, voff = 2 * d + head * HD;

    // Q tile, transposed into shared memory (rows beyond the sequence are 0)
    for (int i = tid; i < AQ * HD; i += 256) {
        const int r = i / HD, c = i % HD;
        const int t = q0 + r;
        Qt[c * (AQ + APAD) + r] = (t < s1) ? qkv[t * row_stride + qoff + c] : 0.0f;
    }

    float o[4][CPT];
    float mrow[4], lrow[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        mrow[i] = -INFINITY;
        lrow[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < CPT; j++) o[i][j] = 0.0f;
    }

    const int last_key = min(q0 + AQ, s1) - 1;  // keys needed: [s0, last_key]
    for (int k0 = s0; k0 <= last_key; k0 += AK) {
        __syncthreads();  // previous tile's Kt/Vs/Pt fully consumed
        for (int i = tid; i < AK * HD; i += 256) {
            const int r = i / HD, c = i % HD;
            const int u = k0 + r;
            const bool ok = u < s1;
            Kt[c * (AK + APAD) + r] = ok ? qkv[u * row_stride + koff + c] : 0.0f;
            Vs[r * HD + c] = ok ? qkv[u * row_stride + voff + c] : 0.0f;
        }
        __syncthreads();

        // S = Q K^T for this thread's 4 x 4 block
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) s[i][j] = 0.0f;
#pragma unroll 8
        for (int c = 0; c < HD; c++) {
            const float4 qa = *reinterpret_cast<const float4*>(&Qt[c * (AQ + APAD) + ty * 4]);
            const float4 kb = *reinterpret_cast<const float4*>(&Kt[c * (AK + APAD) + tx * 4]);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w};
            const float kv[4] = {kb.x, kb.y, kb.z, kb.w};
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) s[i][j] = fmaf(qv[i], kv[j], s[i][j]);
        }

        // mask, online softmax (rows are shared by the 16 lanes of a half warp)
        float alpha[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int t = q0 + ty * 4 + i;
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int u = k0 + tx * 4 + j;
                const bool valid = (u <= t) && (u < s1);
                s[i][j] = valid ? s[i][j] * sm_scale : -INFINITY;
                mx = fmaxf(mx, s[i][j]);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mnew = fmaxf(mrow[i], mx);
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const float p = (s[i][j] == -INFINITY) ? 0.0f : expf(s[i][j] - mnew);
                s[i][j] = p;
                sum += p;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            alpha[i] = (mrow[i] == -INFINITY) ? 0.0f : expf(mrow[i] - mnew);
            lrow[i] = lrow[i] * alpha[i] + sum;
            mrow[i] = mnew;
        }
        // P^T into shared memory
#pragma unroll
        for (int j = 0; j < 4; j++)
            *reinterpret_cast<float4*>(&Pt[(tx * 4 + j) * (AQ + APAD) + ty * 4]) =
                make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
        __syncthreads();

        // O = alpha * O + P V
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < CPT; j++) o[i][j] *= alpha[i];
        const int kmax = min(AK, last_key - k0 + 1);
#pragma unroll 4
        for (int u = 0; u < kmax; u++) {
            const float4 pa = *reinterpret_cast<const float4*>(&Pt[u * (AQ + APAD) + ty * 4]);
            const float pv[4] = {pa.x, pa.y, pa.z, pa.w};
            float vv[CPT];
#pragma unroll
            for (int j = 0; j < CPT; j++) vv[j] = Vs[u * HD + tx * CPT + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < CPT; j++) o[i][j] = fmaf(pv[i], vv[j], o[i][j]);
        }
    }

    // normalise and store
    InvScale qs{0.0, 0.0f, 0.0f};
    if (outq) qs = make_inv_scale(static_cast<double>(__ldg(qscale)));
    float am = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = q0 + ty * 4 + i;
        if (t >= s1) continue;
        const float il = 1.0f / lrow[i];
#pragma unroll
        for (int j = 0; j < CPT; j++) {
            const float v = o[i][j] * il;
            const int64_t idx = static_cast<int64_t>(t) * d + head * HD + tx * CPT + j;
            if (out) out[idx] = v;
            if (outq) outq[idx] = quant_exact(v, qs);
            am = fmaxf(am, fabsf(v));
        }
    }
    if (amax) {
        am = warp_max_f(am);
        if ((tid & 31) == 0) atomicMax(amax, __float_as_uint(am));
    }
}

template <int HD>
static int launch_attention_hd(const float* qkv, const int4* tiles, int ntiles, int T, int d, int nheads,
                               float* out, int8_t* outq, const float* qscale, uint32_t* amax, cudaStream_t st) {
    const size_t smem = sizeof(float) * (HD * (AQ + APAD) + HD * (AK + APAD) + AK * HD + AK * (AQ + APAD));
    static bool attr[64] = {false};
    int dev = 0;
    TVQ_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !attr[dev]) {
        TVQ_CUDA(cudaFuncSetAttribute(attention_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
        attr[dev] = true;
    }
    const float sm_scale = static_cast<float>(1.0 / sqrt(static_cast<double>(HD)));
    attention_kernel<HD><<<ntiles * nheads, 256, smem, st>>>(qkv, tiles, ntiles, T, d, nheads, sm_scale, out, outq,
                                                             qscale, amax);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

int launch_attention(const float* qkv, const int4* tiles, int ntiles, int T, int d, int nheads, float* out,
                     int8_t* outq, const float* qscale, uint32_t* amax, cudaStream_t st) {
    if (ntiles <= 0) return TVQ_OK;
    TVQ_CHECK(nheads > 0 && d % nheads == 0, TVQ_ERR_INVALID, "d must be a multiple of the head count");
    const int hd = d / nheads;
    switch (hd) {
        case 16: return launch_attention_hd<16>(qkv, tiles, ntiles, T, d, nheads, out, outq, qscale, amax, st);
        case 32: return launch_attention_hd<32>(qkv, tiles, ntiles, T, d, nheads, out, outq, qscale, amax, st);
        case 48: return launch_attention_hd<48>(qkv, tiles, ntiles, T, d, nheads, out, outq, qscale, amax, st);
        case 64: return launch_attention_hd<64>(qkv, tiles, ntiles, T, d, nheads, out, outq, qscale, amax, st);
        default:
            set_error(TVQ_ERR_UNSUPPORTED, "head dim must be 16, 32, 48 or 64");
            return TVQ_ERR_UNSUPPORTED;
    }
}

// ------------------------------------------------------------------ scales
// calibrate_minmax symmetric (tv/quantization/engine.tkv:24-30) from a
// recorded amax: scale = fl32(max(amax, 1e-8) / 127).
__global__ void scale_from_amax_kernel(const uint32_t* __restrict__ amax, float* __restrict__ scale, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    double am = static_cast<double>(__uint_as_float(amax[i]));
    if (am < 0.00000001) am = 0.00000001;
    scale[i] = __double2float_rn(am / 127.0);
}

int launch_scale_from_amax(const uint32_t* amax, float* scale, int n, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    scale_from_amax_kernel<<<(n + 127) / 128, 128, 0, st>>>(amax, scale, n);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
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
    const int s = blockIdx.y;
    if (s >= nseg) return;
    const int64_t row = seg[s + 1] - 1;
    for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n; j += (int64_t)gridDim.x * blockDim.x)
        dst[s * n + j] = src[row * n + j];
}

int launch_gather_last(const float* src, const int* seg, int nseg, int64_t n, float* dst, cudaStream_t st) {
    if (nseg <= 0) return TVQ_OK;
    dim3 grid(static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 64)), nseg);
    gather_last_kernel<<<grid, 256, 0, st>>>(src, seg, nseg, n, dst);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

}  // namespace tvq
