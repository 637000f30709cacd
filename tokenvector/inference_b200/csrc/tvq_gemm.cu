// tvq_gemm.cu -- quantized GEMM on the 5th-generation tensor cores.
//
// Replaces matmul_int8_per_channel / matmul_int8_symmetric / matmul_fp8_e4m3
// (tv/quantization/matmul.tkv:4-58, inner loop _dot_int8 :116-127) reached
// from the QuantizedGemm node (tv/runtime/session.tkv:678-697).
//
//   Y[m,n] = epilogue( sum_k A[m,k] * W[n,k] )     A [M,K], W [N,K], K-major
//
// One persistent CTA per SM (384 threads, 12 warps), warp-specialised:
//   warp 0      TMA producer: A and W tiles (128 B of K per row, 128-byte
//               swizzle) into a STAGES-deep shared-memory ring
//   warp 1      MMA issuer: tcgen05.mma kind::i8 (int32 accumulate) or
//               kind::f8f6f4 (E4M3, f32 accumulate), 128 x BN x 32 per
//               instruction, accumulator in tensor memory
//   warp 2      tensor-memory allocator
//   warps 4-11  epilogue, two warps per TMEM lane group (warp w reads lanes
//               32*(w%4)..+31, alternate 16-column chunks): tcgen05.ld, the
//               reference's f64 dequant + bias evaluated exactly in f32
//               (tvq_exact.cuh), optional activation, a swizzled shared-
//               memory transpose, then residual add and coalesced f32 / int8
//               stores
// The accumulator is double-buffered in TMEM (2 x BN columns) so the
// epilogue of tile i overlaps the MMAs of tile i+1 (GEMM_TF32X3: four
// buffers of short K runs, summed in the epilogue's registers).  Every mbarrier wait is
// bounded (tvq_common.cuh); on a timeout the kernel records an error code,
// drains its own TMA loads and MMAs, frees TMEM and returns.
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include <cstdlib>
#include <mutex>

#include "tvq_common.cuh"
#include "tvq_exact.cuh"
#include "tvq_kernels.h"

namespace tvq {

namespace {

constexpr int BM = 128;        // rows of A per tile (= TMEM lanes)
constexpr int BK = 128;        // bytes of K per stage (one 128-byte swizzle row)
constexpr int UMMA_K = 32;     // K per tcgen05.mma for 8-bit operands
// Epilogue geometry for EW epilogue warps (EPW per TMEM lane group, each
// taking CH-column chunks): 16 warps / 8 columns for the INT8 and FP8
// epilogues (their exact dequant is latency-bound: more warps hide it), 8
// warps / 16 columns for the split-TF32 GEMM (register promotion of short K
// runs, fewer arrivals per run).
template <int EW>
struct Epi {
    static_assert(EW == 8 || EW == 16, "8 or 16 epilogue warps");
    static constexpr int EPI_WARPS = EW;
    static constexpr int EPW = EW / 4;
    static constexpr int THREADS = 128 + 32 * EW;  // warps 0-3: TMA, MMA, TMEM alloc, spare; then the epilogue
    static constexpr int CH = 128 / EW;            // accumulator columns per epilogue chunk
    static constexpr int LPR = CH / 4;             // store phase: lanes per 4*CH-byte row segment
    static constexpr int RPI = 32 / LPR;           // rows per store iteration
    static constexpr int SWS = (CH == 16) ? 1 : 2; // staging swizzle: slot j of row r at j ^ ((r >> SWS) & (LPR - 1))
};
// the split-precision fp32 GEMMs: hi / lo operand parts, three products
__host__ __device__ constexpr bool split_kind(int kind) { return kind == GEMM_TF32X3 || kind == GEMM_F16X3; }
// kinds whose partial sums are promoted to registers in short K runs
__host__ __device__ constexpr bool promoted_kind(int kind) { return split_kind(kind) || kind == GEMM_W4; }
template <int KIND>
using EpiOf = Epi<promoted_kind(KIND) ? 8 : 16>;
// GEMM_TF32X3 sums its products in TMEM over this many k-blocks (32 f32
// each) only; the epilogue adds the partial sums in registers with IEEE
// round-to-nearest.  The tensor core's own f32 accumulation is less exact
// than IEEE addition, and over a long K its error grows to ~2^-18 of
// sum|a*w|; promoting every few k-blocks keeps the result at fp32 SGEMM
// accuracy.  TVQ_TF32_PROMOTE_KB overrides it (tuning).
constexpr int TF32_PROMOTE_KB = 2;  // max error ~3x cuBLAS SGEMM, ~15% slower than no promotion
// GEMM_F16X3 (64 fp16 per k-block): every 3 k-blocks (K 192).  Measured at
// the GPT-2 LM head (M 1024, N 50257, K 768) against a float64 reference,
// max |error| / sum|a*w| per promotion interval 1 / 2 / 3 / 4 / 6 / 12:
// 0.30 / 0.47 / 0.66 / 0.93 / 1.41 / 3.28 x that of torch's true-fp32
// matmul, at 423 / 352 / 304 / 296 / 290 / 278 us.
constexpr int F16_PROMOTE_KB = 3;

struct KParams {
    int m, n, k;
    int num_m_blocks, num_n_blocks, num_k_blocks;
    int group_m;     // tile order: groups of group_m m-blocks, m fastest inside a group
    int single;      // GEMM_F16X3 without low parts: y = A W^T + bias on fp16 operands (matmul_fp16)
    // INT8, per-tensor scales, zero points (matmul_int8_asymmetric):
    // acc' = acc - zpw zrow[m] - zpa zcol[n] + zconst, exact in binary64
    const int* zrow;
    const int* zcol;
    double zpa, zpw, zconst;
    int promote_kb;  // k-blocks per TMEM accumulation unit (split kinds)
    int group_ks;    // GEMM_W4: k-steps (16 elements) per weight group = per accumulation unit
    int ngroups;     // GEMM_W4: k / group_size
    int acc_only;    // only the raw int32 accumulators (acc_out) are written
    const float* bias;
    const float* residual;
    float* Y;
    int8_t* Yq;
    int32_t* acc_out;
    const float* scale_a;
    const float* scales_w;
    int per_channel;
    int act;
    const float* scale_out;
    uint32_t* amax;
    int* err;
    // Optional attention operands of a c_attn GEMM (Y = qkv [m, 3 kvd]): the Q
    // and K columns [0, 2 kvd) also as fp16 hi / lo [m, kvd] (qh, ql, kh, kl)
    // and the V columns [2 kvd, 3 kvd) transposed as hi / lo [kvd, vt_pitch]
    // (vth, vtl), each 64-column head scaled by 2^kv_exp (kv_head_exp, from
    // the bounds kv_bound) and the exponents stored to kv_exp [3 kvd / 64].
    __half *qh, *ql, *kh, *kl, *vth, *vtl;
    int kvd, vt_pitch;
    int* kv_exp;
    const float* kv_bound;
    uint32_t* kv_vmax;  // per V column max |V| (float bits) or null
};

// hi / lo fp16 pair of two scaled values, packed two per 32-bit word
// (element a in the low half): hi = fp16(a), lo = fp16(a - hi)
__device__ __forceinline__ void split_h2_pair(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

__device__ __forceinline__ float gelu_tanh_f32(float x) {
    // apply_activation GELU, tv/optimization/kernels.tkv:22-24 + _tanh
    // :32-38, in the reference's numeric model: untyped locals and literals
    // in binary64, binary32 only where a value passes an f32 parameter or
    // return (_tanh's argument and result, apply_activation's result).  The
    // exponential is CUDA's binary64 exp: the f32 results agree with a host
    // libm's except where the binary64 quotient lies within an ulp of an f32
    // rounding boundary.
    const double xd = x;
    const double x3 = xd * xd * xd;
    const float targ = __double2float_rn(0.79788456 * (xd + 0.044715 * x3));
    float th;
    if (static_cast<double>(targ) > 10.0) {
        th = 1.0f;
    } else if (static_cast<double>(targ) < -10.0) {
        th = -1.0f;
    } else {
        const double e = exp(2.0 * static_cast<double>(targ));
        th = __double2float_rn((e - 1.0) / (e + 1.0));
    }
    return __double2float_rn(0.5 * xd * (1.0 + static_cast<double>(th)));
}

__device__ __forceinline__ float gelu_erf_f32(float v) {
    // gelu_erf with the Abramowitz-Stegun 7.1.26 erf, tv/training/tensor.tkv:165-190
    // (every operation spelled out, so that gelu_erf_x2 matches it bit for bit)
    const float x = __fmul_rn(v, 0.70710678118654752f);
    const float ax = fabsf(x);
    const float t = __fdividef(1.0f, fmaf(0.3275911f, ax, 1.0f));
    float poly = fmaf(1.061405429f, t, -1.453152027f);
    poly = fmaf(poly, t, 1.421413741f);
    poly = fmaf(poly, t, -0.284496736f);
    poly = fmaf(poly, t, 0.254829592f);
    poly = __fmul_rn(poly, t);
    float e = fmaf(-__expf(__fmul_rn(-ax, ax)), poly, 1.0f);
    e = __uint_as_float(__float_as_uint(e) ^ (__float_as_uint(x) & 0x80000000u));  // erf is odd
    return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, e));
}

// gelu_erf_f32 of two values with the f32x2 instructions (the reciprocal and
// exponential stay scalar): the same operations, the same results.
__device__ __forceinline__ void gelu_erf_x2(float& v0, float& v1) {
    const uint64_t V = f2_pack(v0, v1);
    const uint64_t X = f2_mul(V, f2_pack(0.70710678118654752f, 0.70710678118654752f));
    const uint64_t AX = f2_abs(X);
    float d0, d1;
    f2_unpack(f2_fma(f2_pack(0.3275911f, 0.3275911f), AX, f2_pack(1.0f, 1.0f)), d0, d1);
    const uint64_t T = f2_pack(__fdividef(1.0f, d0), __fdividef(1.0f, d1));
    uint64_t P = f2_fma(f2_pack(1.061405429f, 1.061405429f), T, f2_pack(-1.453152027f, -1.453152027f));
    P = f2_fma(P, T, f2_pack(1.421413741f, 1.421413741f));
    P = f2_fma(P, T, f2_pack(-0.284496736f, -0.284496736f));
    P = f2_fma(P, T, f2_pack(0.254829592f, 0.254829592f));
    P = f2_mul(P, T);
    float m0, m1;
    f2_unpack(f2_mul(AX, AX), m0, m1);  // -(ax ax) below: the same bits as (-ax) ax
    const uint64_t NEX = f2_pack(-__expf(-m0), -__expf(-m1));
    uint64_t E = f2_fma(NEX, P, f2_pack(1.0f, 1.0f));
    E ^= X & 0x8000000080000000ull;  // erf is odd
    f2_unpack(f2_mul(f2_mul(f2_pack(0.5f, 0.5f), V), f2_add(f2_pack(1.0f, 1.0f), E)), v0, v1);
}

// The reference's gelu_erf (tv/training/tensor.tkv:165-190) as the reference
// evaluates it: binary64 arithmetic, binary32 stores of erf's argument, of
// erf's result and of the GELU (the oracle's tvo_gelu_erf, operation for
// operation; exp is the CUDA binary64 exp, within 1 ulp).
__device__ __noinline__ float gelu_erf_ref(float v) {
    const float arg = __double2float_rn(__ddiv_rn(static_cast<double>(v), 1.4142135623730951));
    const double sg = arg < 0.0f ? -1.0 : 1.0;
    const double ax = fabs(static_cast<double>(arg));
    const double t = __ddiv_rn(1.0, __dadd_rn(1.0, __dmul_rn(0.3275911, ax)));
    double poly = 1.061405429;
    poly = __dadd_rn(__dmul_rn(poly, t), -1.453152027);
    poly = __dadd_rn(__dmul_rn(poly, t), 1.421413741);
    poly = __dadd_rn(__dmul_rn(poly, t), -0.284496736);
    poly = __dadd_rn(__dmul_rn(poly, t), 0.254829592);
    poly = __dmul_rn(poly, t);
    const double e = exp(__dmul_rn(-ax, ax));
    const float erf = __double2float_rn(__dmul_rn(sg, __dadd_rn(1.0, -__dmul_rn(e, poly))));
    return __double2float_rn(__dmul_rn(__dmul_rn(0.5, static_cast<double>(v)), __dadd_rn(1.0, static_cast<double>(erf))));
}

// GELU outputs g (from gelu_erf_x2) that an int8 quantize with hi = fl32(1 /
// scale) could round differently from the reference's own GELU value are
// re-evaluated with gelu_erf_ref.  The fast GELU lies within 2^-19 (1 + |g|)
// of the reference's (measured on B200 over 4M inputs in [-12, 12] and N(0,
// 9): at most 2^-21 + 2^-21.8 |g|), so the int8 value can differ only when
// g * hi lies within 2^-19 (1 + |g|) hi (+ 2^-16 for the product's own
// rounding) of a half-integer; about 1e-4 of the elements at GPT-2 scales.
template <int N>
__device__ __forceinline__ void gelu_fix_near_boundary(float (&g)[N], const float (&v)[N], float hi) {
    uint32_t near = 0;
#pragma unroll
    for (int j = 0; j < N; j++) {
        const float t = __fmul_rn(g[j], hi);
        const float r = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);  // rint for |t| < 2^22
        const float m = fmaf(fabsf(g[j]) + 1.0f, hi * 1.9073486328125e-06f, 1.52587890625e-05f);
        near |= (fabsf(fabsf(__fsub_rn(t, r)) - 0.5f) < m) ? (1u << j) : 0u;
    }
    if (near) {
#pragma unroll
        for (int j = 0; j < N; j++)
            if (near & (1u << j)) g[j] = gelu_erf_ref(v[j]);
    }
}

__device__ __forceinline__ float apply_act(float y, int act) {
    switch (act) {
        case TVQ_ACT_RELU: return y > 0.0f ? y : 0.0f;
        case TVQ_ACT_GELU_TANH: return gelu_tanh_f32(y);
        case TVQ_ACT_GELU_ERF: return gelu_erf_f32(y);
        default: return y;
    }
}

__device__ __forceinline__ int8_t q8_out(double v) {
    if (v != v) return 0;
    double r = rint(v);
    r = fmin(fmax(r, -127.0), 127.0);
    return static_cast<int8_t>(static_cast<int>(r));
}

struct EpiCtx {
    bool vec_ok;     // n % 4 == 0: 16-byte row segments
    InvScale qs;     // 1 / scale_out for the int8 output
    float sa;        // activation scale (attention operand bounds)
};

// Exponent of the power-of-two scale of one head (part 0 Q, 1 K, 2 V) of a
// c_attn output: every |Y| of the head is at most sa * A + B (A = max over its
// columns of sw[n] * 127 * sum_k |W[n,k]|, B = max |bias[n]|, both rounded
// up; 127 * sum_k |W[n,k]| bounds the accumulator), widened by 2^-20 for
// the rounding of Y itself.
__device__ __forceinline__ int kv_head_exp(const float* bound, int heads, int part, int h, float sa) {
    const float A = __ldg(bound + (2 * part) * heads + h), B = __ldg(bound + (2 * part + 1) * heads + h);
    return pow2_exp_below_2p15(__fmul_ru(__fadd_ru(__fmul_ru(sa, A), B), 1.00000095367431640625f));
}

template <int N>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 16) {
        tmem_ld16(taddr, r);
    } else {
        tmem_ld8(taddr, r);
    }
}

// The residual segments (row0 + RPI it + lane / LPR, n0 + 4 (lane % LPR))
// that stage_and_store adds, loaded ahead so their latency overlaps the TMEM
// read and the epilogue arithmetic (the residual may alias Y; each segment is
// read here, before the same thread stores it).
template <class E>
__device__ __forceinline__ void load_residual(const KParams& p, const EpiCtx& e, int lane, int row0, int n0,
                                              float4 (&res)[E::LPR]) {
#pragma unroll
    for (int it = 0; it < E::LPR; it++) {
        const int row = row0 + it * E::RPI + lane / E::LPR;
        const int col = n0 + 4 * (lane % E::LPR);
        res[it] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (p.residual && e.vec_ok && row < p.m && col + 3 < p.n)
            res[it] = *reinterpret_cast<const float4*>(p.residual + static_cast<int64_t>(row) * p.n + col);
    }
}

// Second half of the epilogue for one 32-row x CH-column chunk, y = row
// `lane`: swizzled shared-memory transpose (float4 slot j of row r sits at
// slot j ^ ((r >> SWS) & (LPR - 1)), conflict-free both ways), then LPR lanes
// per 4*CH-byte row segment: residual add, f32 / int8 stores, running amax.
// QOUT compiles the int8 output in (the promoted fp32 forms never write int8;
// leaving it out keeps their kernels small).
template <class E, bool QOUT>
__device__ __forceinline__ void stage_and_store(const KParams& p, const EpiCtx& e, float* stage, const float (&y)[E::CH],
                                                int lane, int row0, int n0, float& amax, const float4 (&res)[E::LPR],
                                                float kvf = 1.0f) {
#pragma unroll
    for (int j = 0; j < E::LPR; j++)
        *reinterpret_cast<float4*>(&stage[lane * E::CH + 4 * (j ^ ((lane >> E::SWS) & (E::LPR - 1)))]) =
            make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
    __syncwarp();
    if (!e.vec_ok) {
        // rows not 16-byte aligned (n % 4 != 0, e.g. the 50257-wide LM
        // head): CH consecutive lanes write CH consecutive columns of one
        // row, 32 / CH rows per store instruction (staging reads stay
        // conflict-free: the 32 / CH rows cover the 32 banks once)
#pragma unroll
        for (int it = 0; it < E::CH; it++) {
            const int rr = it * (32 / E::CH) + lane / E::CH;
            const int c = lane % E::CH;
            const int row = row0 + rr;
            const int col = n0 + c;
            float x = stage[rr * E::CH + 4 * ((c >> 2) ^ ((rr >> E::SWS) & (E::LPR - 1))) + (c & 3)];
            if (row >= p.m || col >= p.n) continue;
            const int64_t off = static_cast<int64_t>(row) * p.n + col;
            if (p.residual) x = __fadd_rn(x, p.residual[off]);
            if (p.amax) amax = fmaxf(amax, fabsf(x));
            if (p.Y) p.Y[off] = x;
            if (QOUT && p.Yq) p.Yq[off] = quant_exact(x, e.qs);
        }
        return;
    }
#pragma unroll
    for (int it = 0; it < E::LPR; it++) {
        const int rr = it * E::RPI + lane / E::LPR;
        const int c4 = lane % E::LPR;
        const int row = row0 + rr;
        const int col = n0 + 4 * c4;
        float4 v = *reinterpret_cast<const float4*>(&stage[rr * E::CH + 4 * (c4 ^ ((rr >> E::SWS) & (E::LPR - 1)))]);
        if (row >= p.m || col >= p.n) continue;
        const int64_t off = static_cast<int64_t>(row) * p.n + col;
        if (p.kh && col < 2 * p.kvd) {  // Q / K part: fp16 hi / lo split, row-major [m, kvd]
            const int part = col >= p.kvd ? 1 : 0;
            const int c = col - part * p.kvd;
            const int64_t ko = static_cast<int64_t>(row) * p.kvd + c;
            uint2 h, l;  // kvf: 2^kv_exp of the chunk's head (a chunk lies inside one head)
            split_h2_pair(v.x * kvf, v.y * kvf, h.x, l.x);
            split_h2_pair(v.z * kvf, v.w * kvf, h.y, l.y);
            *reinterpret_cast<uint2*>((part ? p.kh : p.qh) + ko) = h;
            *reinterpret_cast<uint2*>((part ? p.kl : p.ql) + ko) = l;
        }
        if (e.vec_ok && col + 3 < p.n) {
            if (p.residual) {
                const float4 t = res[it];
                v.x = __fadd_rn(v.x, t.x);
                v.y = __fadd_rn(v.y, t.y);
                v.z = __fadd_rn(v.z, t.z);
                v.w = __fadd_rn(v.w, t.w);
            }
            if (p.amax) amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
            if (p.Y) *reinterpret_cast<float4*>(p.Y + off) = v;
            if (QOUT && p.Yq) {
                float t0, t1, t2, t3;
                const bool ok = quant_fast_t(v.x, e.qs.hi, t0) & quant_fast_t(v.y, e.qs.hi, t1) &
                                quant_fast_t(v.z, e.qs.hi, t2) & quant_fast_t(v.w, e.qs.hi, t3);
                if (ok) {
                    *reinterpret_cast<uint32_t*>(p.Yq + off) = pack_q4(t0, t1, t2, t3);
                } else {
                    char4 q;
                    q.x = quant_exact(v.x, e.qs);
                    q.y = quant_exact(v.y, e.qs);
                    q.z = quant_exact(v.z, e.qs);
                    q.w = quant_exact(v.w, e.qs);
                    *reinterpret_cast<char4*>(p.Yq + off) = q;
                }
            }
        } else {
            const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                if (col + k >= p.n) break;
                float x = vv[k];
                if (p.residual) x = __fadd_rn(x, p.residual[off + k]);
                if (p.amax) amax = fmaxf(amax, fabsf(x));
                if (p.Y) p.Y[off + k] = x;
                if (QOUT && p.Yq) p.Yq[off + k] = quant_exact(x, e.qs);
            }
        }
    }
}

// Tile -> (m-block, n-block).  Tiles run in groups of group_m m-blocks with
// the m-block fastest inside a group, so the CTAs working at the same time
// share a few A row panels and W column panels in L2 (M-fastest order over
// all m-blocks streams the whole of A once per round of tiles).
__device__ __forceinline__ void tile_coords(const KParams& p, int tile, int& mb, int& nb) {
    if (p.group_m >= p.num_m_blocks) {  // one group: plain m-fastest order
        mb = tile % p.num_m_blocks;
        nb = tile / p.num_m_blocks;
        return;
    }
    const int per_group = p.group_m * p.num_n_blocks;
    const int g = tile / per_group, r = tile - g * per_group;
    const int first = g * p.group_m;
    const int gm = min(p.group_m, p.num_m_blocks - first);
    mb = first + r % gm;
    nb = r / gm;
}

// Lean epilogues: compile-time forms of the general epilogue for the two
// GEMM shapes of a static-scale forward, picked by the host only when every
// other output (amax, raw accumulators, attention operands, zero points) is
// off and n is a multiple of 16:
//   LEAN_GELU_Q8  y = fl32(fl64(acc * w[n]) + b[n]), GELU-erf, int8 out only
//   LEAN_F32      y = fl32(fl64(acc * w[n]) + b[n]) (+ residual), f32 out only
// with w[n] = fl64(sa * sw[n]) exact (per tensor, or per channel where
// fl64(fl64(acc * sa) * sw) = fl64(acc * (sa * sw))).  Each epilogue warp
// owns the 16-column chunks c = half + 4 i of its lane group's 32 rows: one
// tcgen05.ld of 16 columns, then the row's 16 outputs go straight from the
// lane's registers to global memory (16 int8 bytes or 64 f32 bytes per
// lane, whole 32-byte sectors), with no shared-memory staging and no barrier
// across warps (a warp's column scales and biases sit in its own shared-
// memory slot, written by its own lanes).  GELU_Q8 decides every int8 value
// in one test: the GELU error bound and the quantize margin together.
//   LEAN_QKV      y as LEAN_F32 (no residual) for a c_attn GEMM, plus the
//                 attention's fp16 hi / lo operands: Q and K row-major, V
//                 transposed, each head scaled by 2^kv_exp, and each V
//                 column's max |V| (the general epilogue's kv split)
//   LEAN_GELU_F32 y as LEAN_F32 (no residual), GELU-erf, f32 out, optional
//                 max |y| (the c_fc of a calibrating forward or of per-call
//                 calibration: its quantize comes after)
constexpr int LEAN_GELU_Q8 = 1;
constexpr int LEAN_F32 = 2;
constexpr int LEAN_QKV = 3;
constexpr int LEAN_GELU_F32 = 4;

template <int KIND, int BN>
__device__ __forceinline__ constexpr uint32_t make_idesc() {
    // instruction descriptor: [4,6) D format, [7,10) A format, [10,13) B
    // format, [15]/[16] A/B major (0 = K), [17,23) N>>3, [24,29) M>>4
    return (KIND == GEMM_I8   ? (2u << 4) | (1u << 7) | (1u << 10)    // S32 <- s8 x s8
            : KIND == GEMM_F8 ? (1u << 4) | (0u << 7) | (0u << 10)    // F32 <- e4m3 x e4m3
            : (KIND == GEMM_F16X3 || KIND == GEMM_W4) ? (1u << 4) | (0u << 7) | (0u << 10) // F32 <- f16 x f16 (kind::f16)
                              : (1u << 4) | (2u << 7) | (2u << 10))   // F32 <- tf32 x tf32
           | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);
}

// NSA / NSB operand parts per stage: 1, or 2 (high + low) for the split
// GEMMs; GEMM_W4 splits A only.
template <int KIND, int BN, int LEAN = 0>
struct Cfg {
    static constexpr int NSA = (split_kind(KIND) || KIND == GEMM_W4) ? 2 : 1;
    static constexpr int NSB = split_kind(KIND) ? 2 : 1;
    static constexpr int ELEM = (KIND == GEMM_TF32X3) ? 4 : (KIND == GEMM_F16X3 || KIND == GEMM_W4) ? 2 : 1;
    static constexpr int BKE = BK / ELEM;                         // K elements per stage
    static constexpr uint32_t A_BYTES = BM * BK;                  // one part
    static constexpr uint32_t B_BYTES = BN * BK;
    static constexpr uint32_t STAGE_BYTES = NSA * A_BYTES + NSB * B_BYTES;
    // LEAN_F32 and LEAN_QKV stage each warp's 32 x 16 f32 chunk in shared memory (2 KB
    // per warp beside its 1 KB of column scales): the ring gives up stages
    // to stay within 227 KB
    static constexpr uint32_t LEAN_EXTRA = (LEAN == 2 || LEAN == 3 || LEAN == 4) ? 32768u : 0u;
    static constexpr int STAGES =
        LEAN_EXTRA ? ((232448u - 49152u - 2u * 2u * BN * 8u - 1536u) / STAGE_BYTES < 8u
                          ? (232448u - 49152u - 2u * 2u * BN * 8u - 1536u) / STAGE_BYTES : 8)
                   : (STAGE_BYTES * 8 <= 196608) ? 8 : 196608 / STAGE_BYTES;
    // TMEM accumulator buffers: 2 (tile i+1's MMAs overlap tile i's
    // epilogue), 4 for the short promotion units of the split kinds
    static constexpr int NACC = promoted_kind(KIND) ? 4 : 2;
    static constexpr uint32_t TMEM_COLS = NACC * BN;  // 128/256/512: powers of two
    static constexpr uint32_t RING = STAGES * STAGE_BYTES;
    static constexpr uint32_t EPI = EpiOf<KIND>::EPI_WARPS * 32 * EpiOf<KIND>::CH * 4 + LEAN_EXTRA;  // per-warp 32 x CH f32 staging
    static constexpr uint32_t COLS = 2 * 2 * BN * 8;  // per-column scale and bias of a tile (f64), double-buffered
    static constexpr uint32_t SMEM = RING + EPI + COLS + 1024 /*align*/ + 512 /*barriers*/;
};

// The lean epilogue of one CTA (warps 4 .. 19; see LEAN_GELU_Q8 / LEAN_F32).
// slots: the general epilogue's staging area, 1 KB per warp here (the f64
// scale and bias of up to 64 columns).
template <int KIND, int BN, int LEAN>
__device__ __forceinline__ void lean_epilogue(const KParams& p, double* slots, uint64_t* tfull, uint64_t* tempty,
                                              uint32_t tmem_base, int warp, int lane) {
    using C = Cfg<KIND, BN, LEAN>;
    constexpr int EPW = 4;             // warps per TMEM lane group
    constexpr int LCH = 16;            // columns per chunk
    constexpr int NCH = BN / (LCH * EPW);  // chunks per warp per tile
    static_assert(NCH >= 1 && EpiOf<KIND>::EPI_WARPS == 16, "lean epilogue: 16 warps, BN >= 64");
    static_assert(16 * 64 * 2 * 8 + (LEAN != LEAN_GELU_Q8 ? 16 * 32 * LCH * 4 : 0) <= C::EPI,
                  "lean epilogue slots exceed the staging area");
    const int eg = warp & 3;
    const int half = (warp - 4) >> 2;
    double* ws = slots + (warp - 4) * 128;  // [64] scales, then [64] biases
    double* bs = ws + 64;
    // LEAN_F32, LEAN_QKV: this warp's 32 x 16 f32 staging tile (after the 16 slots);
    // float4 j of row r sits at slot j ^ ((r >> 1) & 3): conflict-free both
    // ways (lane = row when written, 4 lanes per row when read)
    float* stg = reinterpret_cast<float*>(slots + 16 * 128) + (warp - 4) * (32 * LCH);
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(eg * 32) << 16);
    const float sa = __ldg(p.scale_a);
    const float sw0 = __ldg(p.scales_w);
    const bool per_channel = p.per_channel != 0;
    InvScale qs{0.0, 0.0f, 0.0f};
    float c1 = 0.0f;
    if constexpr (LEAN == LEAN_GELU_Q8) {
        qs = make_inv_scale(static_cast<double>(__ldg(p.scale_out)));
        // an element is decided on the fast path when g hi lies farther than
        // (|g| + 1) hi 2^-19 (the fast GELU's error, widened by 2^-10) plus
        // 2^-14 (the product's rounding and hi's distance from 1/scale:
        // quant_fast_t's 2^-15, and 2^-16 more) from a half-integer
        c1 = qs.hi * 1.9092130661010742e-06f;  // hi 2^-19 (1 + 2^-10)
    }
    // f32 chunk y (lane = row) to Y rows srow0 + 8 it (+ residual res[it],
    // loaded in the store layout): transposed through the warp's staging
    // tile, then 8 rows x 64 bytes per store (each staged element is read
    // before the same lane stores it)
    float amax = 0.0f;  // LEAN_GELU_F32: this lane's max |y| (rows past m excluded)
    auto store_f32_staged = [&](const float (&y)[LCH], int srow0, int n0, const float4 (&res)[4], bool add_res) {
        __syncwarp();  // the previous chunk's staging reads are done
#pragma unroll
        for (int q = 0; q < 4; q++)
            *reinterpret_cast<float4*>(stg + lane * LCH + 4 * (q ^ ((lane >> 1) & 3))) =
                make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
        __syncwarp();
#pragma unroll
        for (int it = 0; it < 4; it++) {
            const int rl = 8 * it + (lane >> 2), c4 = lane & 3;
            float4 v = *reinterpret_cast<const float4*>(stg + rl * LCH + 4 * (c4 ^ ((rl >> 1) & 3)));
            const int rr = srow0 + 8 * it;
            if (rr < p.m) {
                if (add_res) {
                    v.x = __fadd_rn(v.x, res[it].x);
                    v.y = __fadd_rn(v.y, res[it].y);
                    v.z = __fadd_rn(v.z, res[it].z);
                    v.w = __fadd_rn(v.w, res[it].w);
                }
                if (LEAN == LEAN_GELU_F32)
                    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
                *reinterpret_cast<float4*>(p.Y + static_cast<int64_t>(rr) * p.n + n0 + 4 * c4) = v;
            }
        }
    };
    // this warp's column scales and biases of a tile: lane l holds columns l
    // and l + 32 of the warp's LCH * NCH; loaded one tile ahead, so that
    // their latency hides behind the current tile
    constexpr int PPL = (LCH * NCH + 31) / 32;
    float psw[PPL], pb[PPL];
    auto load_params = [&](int t) {
        int tmb, tnb;
        tile_coords(p, t, tmb, tnb);
#pragma unroll
        for (int q = 0; q < PPL; q++) {
            const int j = lane + 32 * q;
            const int n = min(tnb * BN + (half + EPW * (j / LCH)) * LCH + j % LCH, p.n - 1);
            psw[q] = per_channel ? __ldg(p.scales_w + n) : sw0;
            pb[q] = p.bias ? __ldg(p.bias + n) : 0.0f;
        }
    };
    // (the GELU -> int8 form loads them at its tile's start instead: the
    // prefetch registers spill there and it measured 2-3 % slower)
    constexpr bool PREF = LEAN != LEAN_GELU_Q8;
    const int num_tiles = p.num_m_blocks * p.num_n_blocks;
    if (PREF && static_cast<int>(blockIdx.x) < num_tiles) load_params(blockIdx.x);
    uint32_t tcount = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, tcount++) {
        const uint32_t b = tcount % C::NACC;
        const uint32_t aph = (tcount / C::NACC) & 1u;
        int mb, nb;
        tile_coords(p, tile, mb, nb);
        const int row = mb * BM + eg * 32 + lane;
        const bool row_ok = row < p.m;
        // this tile's column scales and biases into the warp's slot (the
        // previous tile's reads of the slot are done: same warp, program
        // order), then the next tile's loads
        if (!PREF) load_params(tile);
        __syncwarp();
#pragma unroll
        for (int q = 0; q < PPL; q++) {
            const int j = lane + 32 * q;
            if (j < LCH * NCH) {
                ws[j] = static_cast<double>(sa) * static_cast<double>(psw[q]);  // exact
                bs[j] = static_cast<double>(pb[q]);
            }
        }
        __syncwarp();
        if (PREF && tile + static_cast<int>(gridDim.x) < num_tiles) load_params(tile + gridDim.x);
        // LEAN_F32 store layout: in step it, lane l holds float4 (l & 3) of
        // row it * 8 + (l >> 2) of the warp's 32 rows
        const int srow0 = mb * BM + eg * 32 + (lane >> 2);
        float4 res[4];
        const int n00 = nb * BN + half * LCH;
        if (LEAN == LEAN_F32 && p.residual && n00 < p.n) {
#pragma unroll
            for (int it = 0; it < 4; it++) {
                const int rr = srow0 + 8 * it;
                if (rr < p.m)
                    res[it] = *reinterpret_cast<const float4*>(p.residual + static_cast<int64_t>(rr) * p.n + n00 +
                                                               4 * (lane & 3));
            }
        }
        // LEAN_QKV: each chunk's head exponent (two global loads) before the
        // accumulator wait, off the chunks' critical path
        int kv_sh[NCH];
        if constexpr (LEAN == LEAN_QKV) {
#pragma unroll
            for (int i = 0; i < NCH; i++) {
                const int n0 = nb * BN + (half + EPW * i) * LCH;
                const int part = min(n0, p.n - 1) / p.kvd;
                const int hh = (min(n0, p.n - 1) - part * p.kvd) / 64;
                kv_sh[i] = kv_head_exp(p.kv_bound, p.kvd / 64, part, hh, sa);
            }
        }
        const bool got = mbar_wait(&tfull[b], aph, p.err, DEVERR_TIMEOUT_EPILOGUE);
        if (!__all_sync(0xffffffffu, got)) break;
        tc_fence_after();
        // not unrolled: the chunk body (with its rare exact path) stays small
        // in the instruction cache; i only offsets shared memory and TMEM
#pragma unroll 1
        for (int i = 0; i < NCH; i++) {
            const int c = half + EPW * i;
            const int n0 = nb * BN + c * LCH;
            if (n0 >= p.n) break;  // warp-uniform; n is a multiple of 16
            if (LEAN == LEAN_F32 && p.residual && i > 0) {  // chunk 0's came before the wait
#pragma unroll
                for (int it = 0; it < 4; it++) {
                    const int rr = srow0 + 8 * it;
                    if (rr < p.m)
                        res[it] = *reinterpret_cast<const float4*>(p.residual + static_cast<int64_t>(rr) * p.n + n0 +
                                                                   4 * (lane & 3));
                }
            }
            uint32_t r[LCH];
            tmem_ld16(lane_base + b * BN + c * LCH, r);
            tmem_ld_wait();
            // the reference's chain, matmul.tkv:5,14,28
            float y[LCH];
#pragma unroll
            for (int j = 0; j < LCH; j += 2) {
                const double2 w2 = *reinterpret_cast<const double2*>(ws + i * LCH + j);
                const double2 b2 = *reinterpret_cast<const double2*>(bs + i * LCH + j);
                const double a0 = (KIND == GEMM_I8) ? i32_to_f64(r[j]) : static_cast<double>(__uint_as_float(r[j]));
                const double a1 =
                    (KIND == GEMM_I8) ? i32_to_f64(r[j + 1]) : static_cast<double>(__uint_as_float(r[j + 1]));
                y[j] = __double2float_rn(__dadd_rn(__dmul_rn(a0, w2.x), b2.x));
                y[j + 1] = __double2float_rn(__dadd_rn(__dmul_rn(a1, w2.y), b2.y));
            }
            if constexpr (LEAN == LEAN_GELU_Q8) {
                float g[LCH];
#pragma unroll
                for (int j = 0; j < LCH; j++) g[j] = y[j];
#pragma unroll
                for (int j = 0; j < LCH; j += 2) gelu_erf_x2(g[j], g[j + 1]);
                constexpr float M = 12582912.0f;  // 1.5 * 2^23
                float t[LCH];
                bool ok = true;
                const uint64_t HI2 = f2_pack(qs.hi, qs.hi), M2 = f2_pack(M, M);
#pragma unroll
                for (int j = 0; j < LCH; j += 2) {
                    // per element: tt = fl(g hi + M), r = tt - M (exact), d =
                    // fl(g hi - r); two elements per f32x2 instruction
                    const uint64_t G = f2_pack(g[j], g[j + 1]);
                    const uint64_t TT = f2_fma(G, HI2, M2);
                    const uint64_t D = f2_fma(G, HI2, f2_sub(M2, TT));
                    float tt[2], d[2];
                    f2_unpack(TT, tt[0], tt[1]);
                    f2_unpack(D, d[0], d[1]);
#pragma unroll
                    for (int e = 0; e < 2; e++) {
                        const float m = fmaf(fabsf(g[j + e]), c1, c1 + 6.103515625e-05f);
                        ok &= fabsf(fabsf(d[e]) - 0.5f) >= m;  // false for NaN
                        t[j + e] = fminf(fmaxf(tt[e], M - 127.0f), M + 127.0f);
                    }
                }
                if (!ok) {
                    // an element near an int8 boundary (or not finite): the
                    // reference's own GELU and quantize decide it (unrolled:
                    // the arrays stay in registers)
#pragma unroll
                    for (int j = 0; j < LCH; j++) {
                        const float tt = fmaf(g[j], qs.hi, M);
                        const float d = fmaf(g[j], qs.hi, -__fsub_rn(tt, M));
                        const float m = fmaf(fabsf(g[j]), c1, c1 + 6.103515625e-05f);
                        if (!(fabsf(fabsf(d) - 0.5f) >= m))
                            t[j] = M + static_cast<float>(quant_exact(gelu_erf_ref(y[j]), qs));
                    }
                }
                if (row_ok) {
                    uint4 o;
                    o.x = pack_q4(t[0], t[1], t[2], t[3]);
                    o.y = pack_q4(t[4], t[5], t[6], t[7]);
                    o.z = pack_q4(t[8], t[9], t[10], t[11]);
                    o.w = pack_q4(t[12], t[13], t[14], t[15]);
                    *reinterpret_cast<uint4*>(p.Yq + static_cast<int64_t>(row) * p.n + n0) = o;
                }
            } else if constexpr (LEAN == LEAN_GELU_F32) {
#pragma unroll
                for (int j = 0; j < LCH; j += 2) gelu_erf_x2(y[j], y[j + 1]);
                store_f32_staged(y, srow0, n0, res, false);
            } else if constexpr (LEAN == LEAN_QKV) {
                store_f32_staged(y, srow0, n0, res, false);
                const int part = n0 / p.kvd;  // 0 Q, 1 K, 2 V (a chunk lies inside one 64-column head)
                const int cc = n0 - part * p.kvd;
                const int hh = cc / 64;
                int sh = kv_sh[0];  // kv_sh[i] (the loop is rolled: select, no local-memory index)
#pragma unroll
                for (int i2 = 1; i2 < NCH; i2++)
                    if (i2 == i) sh = kv_sh[i2];
                const float kvf = exp2i(sh);
                if (mb == 0 && eg == 0 && lane == 0 && cc % 64 == 0)
                    p.kv_exp[part * (p.kvd / 64) + hh] = sh;  // one writer per head
                if (part < 2) {
                    uint32_t h[LCH / 2], l[LCH / 2];
#pragma unroll
                    for (int j = 0; j < LCH; j += 2) split_h2_pair(y[j] * kvf, y[j + 1] * kvf, h[j / 2], l[j / 2]);
                    if (row_ok) {
                        const int64_t ko = static_cast<int64_t>(row) * p.kvd + cc;
                        uint4* dh = reinterpret_cast<uint4*>((part ? p.kh : p.qh) + ko);
                        uint4* dl = reinterpret_cast<uint4*>((part ? p.kl : p.ql) + ko);
                        dh[0] = make_uint4(h[0], h[1], h[2], h[3]);
                        dh[1] = make_uint4(h[4], h[5], h[6], h[7]);
                        dl[0] = make_uint4(l[0], l[1], l[2], l[3]);
                        dl[1] = make_uint4(l[4], l[5], l[6], l[7]);
                    }
                } else {
                    if (row_ok) {
                        // V^T: column n0 + j is a row of V^T; lanes (consecutive
                        // tokens) write consecutive addresses
                        const int64_t vo = static_cast<int64_t>(cc) * p.vt_pitch + row;
#pragma unroll
                        for (int j = 0; j < LCH; j++) {
                            const float v = y[j] * kvf;
                            const __half hv = __float2half_rn(v);
                            p.vth[vo + static_cast<int64_t>(j) * p.vt_pitch] = hv;
                            p.vtl[vo + static_cast<int64_t>(j) * p.vt_pitch] = __float2half_rn(__fsub_rn(v, __half2float(hv)));
                        }
                    }
                    if (p.kv_vmax) {
                        // max over the warp's 32 rows of each of the 16 columns:
                        // four rounds that each keep half the columns (lane bits
                        // 16, 8, 4, 2 pick them), then lane bit 1
                        float v[LCH];
#pragma unroll
                        for (int j = 0; j < LCH; j++) v[j] = row_ok ? fabsf(y[j]) : 0.0f;
#pragma unroll
                        for (int rd = 0, hn = LCH / 2; rd < 4; rd++, hn >>= 1) {
                            const bool upper = (lane >> (4 - rd)) & 1;
#pragma unroll
                            for (int i2 = 0; i2 < LCH / 2; i2++) {
                                if (i2 < hn) {
                                    const float keep = upper ? v[i2 + hn] : v[i2];
                                    const float send = upper ? v[i2] : v[i2 + hn];
                                    v[i2] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 16 >> rd));
                                }
                            }
                        }
                        const float vm = fmaxf(v[0], __shfl_xor_sync(0xffffffffu, v[0], 1));
                        const int cj = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
                        if ((lane & 1) == 0) atomicMax(p.kv_vmax + cc + cj, __float_as_uint(vm));
                    }
                }
            } else {
                store_f32_staged(y, srow0, n0, res, p.residual != nullptr);
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[b]);
    }
    if (LEAN == LEAN_GELU_F32 && p.amax) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) atomicMax(p.amax, __float_as_uint(amax));
    }
}

template <int KIND, int BN, int LEAN>
__global__ void __launch_bounds__(EpiOf<KIND>::THREADS, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmA2, const __grid_constant__ CUtensorMap tmB2, KParams p) {
    using C = Cfg<KIND, BN, LEAN>;
    using E = EpiOf<KIND>;
    constexpr int STAGES = C::STAGES;
    constexpr int NSA = C::NSA, NSB = C::NSB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;                                // stage s: NSA parts of A_BYTES
    uint8_t* sB = smem + STAGES * NSA * C::A_BYTES;    // stage s: NSB parts of B_BYTES
    float* colv = reinterpret_cast<float*>(smem + C::RING + C::EPI);  // [2 buffers][scale BN | bias BN]
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::RING + C::EPI + C::COLS);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;
    uint64_t* tempty = tfull + C::NACC;
    uint64_t* drain = tempty + C::NACC;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < C::NACC; b++) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], E::EPI_WARPS);
        }
        mbar_init(drain, 1);
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        if (NSA == 2) tma_prefetch_desc(&tmA2);
        if (NSB == 2) tma_prefetch_desc(&tmB2);
    }
    if (warp == 2) {
        tmem_alloc(tmem_holder, C::TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    griddep_wait();  // A and the residual come from the previous kernel

    const int num_tiles = p.num_m_blocks * p.num_n_blocks;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                int mb, nb;
                tile_coords(p, tile, mb, nb);
                for (int kb = 0; kb < p.num_k_blocks; kb++, it++) {
                    const uint32_t s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1u;
                    if (!mbar_wait(&empty[s], ph ^ 1u, p.err, DEVERR_TIMEOUT_PRODUCER)) { ok = false; break; }
                    mbar_arrive_expect_tx(&full[s], p.single ? C::A_BYTES + C::B_BYTES : C::STAGE_BYTES);
                    tma_load_2d(&tmA, &full[s], sA + s * NSA * C::A_BYTES, kb * C::BKE, mb * BM);
                    tma_load_2d(&tmB, &full[s], sB + s * NSB * C::B_BYTES, kb * C::BKE, nb * BN);
                    if (NSA == 2 && !p.single)
                        tma_load_2d(&tmA2, &full[s], sA + (s * NSA + 1) * C::A_BYTES, kb * C::BKE, mb * BM);
                    if (NSB == 2 && !p.single)
                        tma_load_2d(&tmB2, &full[s], sB + (s * NSB + 1) * C::B_BYTES, kb * C::BKE, nb * BN);
                }
            }
            // every issued load lands before the CTA may exit
            const uint32_t first = it > static_cast<uint32_t>(STAGES) ? it - STAGES : 0u;
            for (uint32_t j = first; j < it; j++)
                mbar_wait(&full[j % STAGES], (j / STAGES) & 1u, p.err, DEVERR_TIMEOUT_DRAIN);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc<KIND, BN>();
            // one accumulation unit = a tile (or, split kinds, a run of
            // promote_kb k-blocks of it) in one of the NACC TMEM buffers
            const int pk = split_kind(KIND) ? p.promote_kb : p.num_k_blocks;
            uint32_t it = 0, ucount = 0;
            bool ok = true;
            if constexpr (KIND == GEMM_W4) {
                // one accumulation unit per weight group (group_ks k-steps of
                // 16, inside one stage or across several): acc = sum a_lo q +
                // a_hi q; a stage is released after its last k-step
                constexpr int KS = BK / UMMA_K;  // k-steps per stage (4)
                const int nks = p.ngroups * p.group_ks;
                for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                    uint32_t a0 = 0, b0 = 0, s = 0;
                    for (int g = 0; g < p.ngroups && ok; g++, ucount++) {
                        const uint32_t b = ucount % C::NACC;
                        const uint32_t aph = (ucount / C::NACC) & 1u;
                        if (!mbar_wait(&tempty[b], aph ^ 1u, p.err, DEVERR_TIMEOUT_MMA)) { ok = false; break; }
                        tc_fence_after();
                        const uint32_t d_tmem = tmem_base + b * BN;
                        for (int ks = g * p.group_ks; ks < (g + 1) * p.group_ks; ks++) {
                            const int kk = ks % KS;
                            if (kk == 0) {  // a new stage
                                s = it % STAGES;
                                const uint32_t ph = (it / STAGES) & 1u;
                                if (!mbar_wait(&full[s], ph, p.err, DEVERR_TIMEOUT_MMA)) { ok = false; break; }
                                tc_fence_after();
                                a0 = smem_u32(sA + s * NSA * C::A_BYTES);
                                b0 = smem_u32(sB + s * NSB * C::B_BYTES);
                            }
                            const uint64_t ad = smem_desc_k_sw128(a0 + kk * UMMA_K);
                            const uint64_t adl = smem_desc_k_sw128(a0 + C::A_BYTES + kk * UMMA_K);
                            const uint64_t bd = smem_desc_k_sw128(b0 + kk * UMMA_K);
                            umma_f16(d_tmem, adl, bd, idesc, ks > g * p.group_ks ? 1u : 0u);
                            umma_f16(d_tmem, ad, bd, idesc, 1u);
                            if (kk == KS - 1 || ks == nks - 1) {
                                umma_commit(&empty[s]);  // stage s is free once these MMAs retire
                                it++;
                            }
                        }
                        if (!ok) break;
                        umma_commit(&tfull[b]);  // accumulator b holds the group's sum
                    }
                    // stages loaded past the last k-step (a partial last block
                    // is covered above): none, the producer loads exactly the
                    // k-blocks that hold the nks k-steps
                }
            } else
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x)
            for (int kb0 = 0; kb0 < p.num_k_blocks && ok; kb0 += pk, ucount++) {
                const uint32_t b = ucount % C::NACC;
                const uint32_t aph = (ucount / C::NACC) & 1u;
                if (!mbar_wait(&tempty[b], aph ^ 1u, p.err, DEVERR_TIMEOUT_MMA)) { ok = false; break; }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + b * BN;
                const int kb1 = min(p.num_k_blocks, kb0 + pk);
                for (int kb = kb0; kb < kb1; kb++, it++) {
                    const uint32_t s = it % STAGES;
                    const uint32_t ph = (it / STAGES) & 1u;
                    if (!mbar_wait(&full[s], ph, p.err, DEVERR_TIMEOUT_MMA)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + s * NSA * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + s * NSB * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / UMMA_K; kk++) {  // 32 bytes of K per instruction
                        const uint64_t ad = smem_desc_k_sw128(a0 + kk * UMMA_K);
                        const uint64_t bd = smem_desc_k_sw128(b0 + kk * UMMA_K);
                        const uint32_t accum = (kb > kb0 || kk > 0) ? 1u : 0u;
                        if (KIND == GEMM_I8) {
                            umma_i8(d_tmem, ad, bd, idesc, accum);
                        } else if (KIND == GEMM_F8) {
                            umma_f8(d_tmem, ad, bd, idesc, accum);
                        } else if (KIND == GEMM_F16X3) {
                            if (p.single) {  // plain fp16 operands: one product
                                umma_f16(d_tmem, ad, bd, idesc, accum);
                                continue;
                            }
                            // same three products on fp16 parts (16 K per instruction)
                            const uint64_t adl = smem_desc_k_sw128(a0 + C::A_BYTES + kk * UMMA_K);
                            const uint64_t bdl = smem_desc_k_sw128(b0 + C::B_BYTES + kk * UMMA_K);
                            umma_f16(d_tmem, adl, bd, idesc, accum);
                            umma_f16(d_tmem, ad, bdl, idesc, 1u);
                            umma_f16(d_tmem, ad, bd, idesc, 1u);
                        } else {
                            // x*w ~ xh*wh + xh*wl + xl*wh, small terms first
                            const uint64_t adl = smem_desc_k_sw128(a0 + C::A_BYTES + kk * UMMA_K);
                            const uint64_t bdl = smem_desc_k_sw128(b0 + C::B_BYTES + kk * UMMA_K);
                            umma_tf32(d_tmem, adl, bd, idesc, accum);
                            umma_tf32(d_tmem, ad, bdl, idesc, 1u);
                            umma_tf32(d_tmem, ad, bd, idesc, 1u);
                        }
                    }
                    umma_commit(&empty[s]);  // stage s is free once these MMAs retire
                }
                if (!ok) break;
                umma_commit(&tfull[b]);      // accumulator b holds the unit's sum
            }
            // all issued MMAs retire before TMEM is released
            umma_commit(drain);
            mbar_wait(drain, 0, p.err, DEVERR_TIMEOUT_DRAIN);
        }
    } else if (LEAN != 0 && warp >= 4) {
        if constexpr (LEAN != 0)
            lean_epilogue<KIND, BN, LEAN>(p, reinterpret_cast<double*>(smem + C::RING), tfull, tempty, tmem_base, warp,
                                          lane);
    } else if (LEAN == 0 && warp >= 4) {
        // ------------------------------------------------ epilogue
        // phase 1: lane = row, CH consecutive columns from TMEM -> the
        //          reference epilogue in binary64, its own operations
        //          (matmul.tkv:5,14,28: fl32(fl64(acc * fl64(sa*sw)) + b) or
        //          fl32(fl64(fl64(acc*sa) * sw) + b), FP64 at half the FP32
        //          rate on B200, two conversions per element) -> activation
        //          -> stage
        // phase 2: lanes along columns: residual, f32 / int8 stores (four
        //          lanes write one 64-byte row segment), amax
        const int eg = warp & 3;            // TMEM lane group this warp may access
        const int half = (warp - 4) >> 2;   // which of the E::EPW interleaved chunk sequences it takes
        float* stage = reinterpret_cast<float*>(smem + C::RING) + (warp - 4) * (32 * E::CH);
        const bool bias_on = p.bias != nullptr;
        const bool per_channel = p.per_channel != 0;
        // per channel: fl64(fl64(acc*sa)*sw) = fl64(acc*(sa*sw)) whenever acc*sa
        // is exact in f64 (sa*sw always is: two 24-bit significands): an f32
        // accumulator always, an int32 one while |acc| <= 127^2 K < 2^29
        const bool fold = per_channel && (KIND != GEMM_I8 || p.k < 33283);
        // zero points (per-tensor INT8 only): s = fl64(sa sw) stays in a register
        const bool asym = KIND == GEMM_I8 && p.zcol != nullptr;
        const float sa = (promoted_kind(KIND) || p.acc_only) ? 1.0f : __ldg(p.scale_a);
        const float sw0 = (promoted_kind(KIND) || p.acc_only) ? 1.0f : __ldg(p.scales_w);
        const double s_asym = static_cast<double>(sa) * static_cast<double>(sw0);
        InvScale qs{0.0, 0.0f, 0.0f};
        if (p.Yq) qs = make_inv_scale(static_cast<double>(__ldg(p.scale_out)));
        EpiCtx ec{(p.n & 3) == 0, qs, sa};
        float amax = 0.0f;
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(eg * 32) << 16);
        if constexpr (promoted_kind(KIND)) {
            // partial sums of promote_kb k-blocks each (GEMM_W4: of one weight
            // group each, times the group's scale), added in registers
            constexpr int NCH = BN / E::CH / E::EPW;  // chunks this warp owns: half, half + E::EPW, ...
            uint32_t ucount = 0;
            bool alive = true;
            const int nunits = (KIND == GEMM_W4) ? p.ngroups : (p.num_k_blocks + p.promote_kb - 1) / p.promote_kb;
            for (int tile = blockIdx.x; tile < num_tiles && alive; tile += gridDim.x) {
                int mb, nb;
                tile_coords(p, tile, mb, nb);
                const int row0 = mb * BM + eg * 32;
                float acc[NCH][E::CH];
                for (int u = 0; u < nunits; u++, ucount++) {
                    const uint32_t b = ucount % C::NACC;
                    const uint32_t aph = (ucount / C::NACC) & 1u;
                    const bool got = mbar_wait(&tfull[b], aph, p.err, DEVERR_TIMEOUT_EPILOGUE);
                    __syncwarp();
                    if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
                    tc_fence_after();
                    // G chunks per TMEM read (all of them when they fit the registers)
                    constexpr int G = (NCH > 4) ? 2 : NCH;
#pragma unroll
                    for (int i0 = 0; i0 < NCH; i0 += G) {
                        uint32_t r[G][E::CH];
#pragma unroll
                        for (int ii = 0; ii < G; ii++)
                            tmem_ld_chunk(lane_base + b * BN + (half + E::EPW * (i0 + ii)) * E::CH, r[ii]);
                        tmem_ld_wait();
#pragma unroll
                        for (int ii = 0; ii < G; ii++) {
                            const int i = i0 + ii;
                            if constexpr (KIND == GEMM_W4) {
                                // the group's scale of each column (same in every lane)
                                const int n0 = nb * BN + (half + E::EPW * i) * E::CH;
#pragma unroll
                                for (int j = 0; j < E::CH; j++) {
                                    const int n = min(n0 + j, p.n - 1);
                                    const float sc = __ldg(p.scales_w + static_cast<int64_t>(n) * p.ngroups + u);
                                    acc[i][j] = u == 0 ? __fmul_rn(__uint_as_float(r[ii][j]), sc)
                                                       : fmaf(__uint_as_float(r[ii][j]), sc, acc[i][j]);
                                }
                            } else if (u == 0) {
#pragma unroll
                                for (int j = 0; j < E::CH; j++) acc[i][j] = __uint_as_float(r[ii][j]);
                            } else {
#pragma unroll
                                for (int j = 0; j < E::CH; j++)
                                    acc[i][j] = __fadd_rn(acc[i][j], __uint_as_float(r[ii][j]));
                            }
                        }
                    }
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&tempty[b]);
                }
                if (!alive) break;
                if constexpr (KIND == GEMM_W4) {
                    // undo the rows' power-of-two scale of A (exact), then the bias
                    const int row = row0 + lane;
                    const float ra = (row < p.m) ? __ldg(p.scale_a + row) : 0.0f;
#pragma unroll
                    for (int i = 0; i < NCH; i++) {
                        const int n0 = nb * BN + (half + E::EPW * i) * E::CH;
#pragma unroll
                        for (int j = 0; j < E::CH; j++) {
                            const int n = min(n0 + j, p.n - 1);
                            acc[i][j] = __fadd_rn(acc[i][j] * ra, bias_on ? __ldg(p.bias + n) : 0.0f);
                        }
                    }
                }
                if constexpr (KIND == GEMM_F16X3) {
                  if (p.single) {
                    // matmul_fp16: y = acc + bias
                    if (bias_on) {
#pragma unroll
                        for (int i = 0; i < NCH; i++) {
                            const int n0 = nb * BN + (half + E::EPW * i) * E::CH;
#pragma unroll
                            for (int j = 0; j < E::CH; j++)
                                acc[i][j] = __fadd_rn(acc[i][j], __ldg(p.bias + min(n0 + j, p.n - 1)));
                        }
                    }
                  } else {
                    // undo the rows' power-of-two scales (exact)
                    const int row = row0 + lane;
                    const float ra = (row < p.m) ? __ldg(p.scale_a + row) : 0.0f;
                    const bool sw_vec = (reinterpret_cast<uintptr_t>(p.scales_w) & 15) == 0;
#pragma unroll
                    for (int i = 0; i < NCH; i++) {
                        const int n0 = nb * BN + (half + E::EPW * i) * E::CH;
                        // the chunk's column scales: CH / 4 16-byte loads (one
                        // address per warp) where the chunk lies inside [0, n)
                        if (sw_vec && n0 + E::CH <= p.n) {
#pragma unroll
                            for (int q4 = 0; q4 < E::CH / 4; q4++) {
                                const float4 t = __ldg(reinterpret_cast<const float4*>(p.scales_w + n0) + q4);
                                acc[i][4 * q4] = acc[i][4 * q4] * ra * t.x;
                                acc[i][4 * q4 + 1] = acc[i][4 * q4 + 1] * ra * t.y;
                                acc[i][4 * q4 + 2] = acc[i][4 * q4 + 2] * ra * t.z;
                                acc[i][4 * q4 + 3] = acc[i][4 * q4 + 3] * ra * t.w;
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < E::CH; j++)
                                acc[i][j] = acc[i][j] * ra * __ldg(p.scales_w + min(n0 + j, p.n - 1));
                        }
                    }
                  }
                }
#pragma unroll
                for (int i = 0; i < NCH; i++) {
                    const int n0 = nb * BN + (half + E::EPW * i) * E::CH;
                    if (n0 >= p.n) break;  // warp-uniform
                    __syncwarp();           // the previous chunk's staging reads are done
                    const float4 nores[E::LPR] = {};
                    stage_and_store<E, false>(p, ec, stage, acc[i], lane, row0, n0, amax, nores);
                }
            }
        } else {
        uint32_t tcount = 0;
        const int etid = threadIdx.x - 128;  // 0 .. EPI_WARPS * 32 - 1
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, tcount++) {
            const uint32_t b = tcount % C::NACC;
            const uint32_t aph = (tcount / C::NACC) & 1u;
            int mb, nb;
            tile_coords(p, tile, mb, nb);
            const int row0 = mb * BM + eg * 32;
            // while the tile's MMAs run: the tile's per-column scales and
            // bias into shared memory (buffer tcount & 1; the barrier below
            // publishes it, and the next tile's barrier keeps it alive until
            // every epilogue warp is done with this tile) and this warp's
            // residual rows toward L2
            double* csc = reinterpret_cast<double*>(colv) + (tcount & 1u) * 2 * BN;
            double* cbi = csc + BN;
            for (int i = etid; i < BN; i += E::EPI_WARPS * 32) {
                const int n = min(nb * BN + i, p.n - 1);
                const double sw = static_cast<double>(per_channel ? __ldg(p.scales_w + n) : sw0);
                // (zero points: the column's term -zpa sum_k W[n, k] instead, exact)
                csc[i] = asym ? -p.zpa * static_cast<double>(__ldg(p.zcol + n))
                              : (per_channel && !fold) ? sw : static_cast<double>(sa) * sw;  // exact in f64
                cbi[i] = static_cast<double>(bias_on ? __ldg(p.bias + n) : 0.0f);
            }
            // this lane's row: zconst - zpw sum_k A[row, k] (exact)
            const double zrow_term = (asym && row0 + lane < p.m)
                                         ? p.zconst - p.zpw * static_cast<double>(__ldg(p.zrow + row0 + lane))
                                         : 0.0;
            if (p.residual) {
                const int row = row0 + lane;
                for (int c = half; c < BN / E::CH; c += E::EPW) {
                    const int n0 = nb * BN + c * E::CH;
                    if (n0 >= p.n) break;
                    if (row < p.m) prefetch_l2(p.residual + static_cast<int64_t>(row) * p.n + n0);
                }
            }
            const bool got = mbar_wait(&tfull[b], aph, p.err, DEVERR_TIMEOUT_EPILOGUE);
            // every epilogue warp takes the same decision (and sees the scales)
            if (!named_bar_and(1, E::EPI_WARPS * 32, got)) break;
            tc_fence_after();
            float4 res_next[E::LPR];
            if (half * E::CH + nb * BN < p.n) load_residual<E>(p, ec, lane, row0, nb * BN + half * E::CH, res_next);
#pragma unroll 1
            for (int c = half; c < BN / E::CH; c += E::EPW) {
                const int n0 = nb * BN + c * E::CH;
                if (n0 >= p.n) break;  // warp-uniform
                float4 res[E::LPR];
#pragma unroll
                for (int it = 0; it < E::LPR; it++) res[it] = res_next[it];
                // the next chunk's residual is in flight while this one is evaluated
                if (c + E::EPW < BN / E::CH && n0 + E::EPW * E::CH < p.n)
                    load_residual<E>(p, ec, lane, row0, n0 + E::EPW * E::CH, res_next);
                // per-column scale and bias (shared memory, same address in every lane)
                double wv[E::CH], bdv[E::CH];
#pragma unroll
                for (int j = 0; j < E::CH / 2; j++) {
                    const double2 t = *reinterpret_cast<const double2*>(csc + c * E::CH + 2 * j);
                    const double2 u = *reinterpret_cast<const double2*>(cbi + c * E::CH + 2 * j);
                    wv[2 * j] = t.x; wv[2 * j + 1] = t.y;
                    bdv[2 * j] = u.x; bdv[2 * j + 1] = u.y;
                }
                uint32_t r[E::CH];
                __syncwarp();
                tmem_ld_chunk(lane_base + b * BN + c * E::CH, r);
                tmem_ld_wait();
                if (p.acc_out && row0 + lane < p.m) {
                    int32_t* dst = p.acc_out + static_cast<int64_t>(row0 + lane) * p.n + n0;
#pragma unroll
                    for (int j = 0; j < E::CH; j++)
                        if (n0 + j < p.n) dst[j] = static_cast<int32_t>(r[j]);
                }
                if (p.acc_only) continue;  // MatMulInteger: the accumulators are the result
                float y[E::CH];
#pragma unroll
                for (int j = 0; j < E::CH; j++) {
                    const double a = (KIND == GEMM_I8) ? static_cast<double>(static_cast<int>(r[j]))
                                                       : static_cast<double>(__uint_as_float(r[j]));
                    const double v = (per_channel && !fold) ? __dmul_rn(__dmul_rn(a, static_cast<double>(sa)), wv[j])
                                     : asym ? __dmul_rn(__dadd_rn(__dadd_rn(a, zrow_term), wv[j]), s_asym)
                                            : __dmul_rn(a, wv[j]);
                    y[j] = __double2float_rn(__dadd_rn(v, bdv[j]));
                }
                float kvf = 1.0f;
                if (p.vth) {
                    const int part = n0 / p.kvd;  // 0 Q, 1 K, 2 V
                    const int hh = (n0 - part * p.kvd) / 64;
                    const int sh = kv_head_exp(p.kv_bound, p.kvd / 64, part, hh, sa);
                    kvf = exp2i(sh);
                    if (row0 == 0 && lane == 0 && (n0 - part * p.kvd) % 64 == 0)
                        p.kv_exp[part * (p.kvd / 64) + hh] = sh;  // one writer per head
                    if (part == 2 && row0 + lane < p.m) {
                        // V part, transposed: column n0 + j -> row of V^T; lanes
                        // (consecutive tokens) write consecutive addresses
                        const int64_t vo = static_cast<int64_t>(n0 - 2 * p.kvd) * p.vt_pitch + row0 + lane;
#pragma unroll
                        for (int j = 0; j < E::CH; j++) {
                            const float v = y[j] * kvf;
                            const __half h = __float2half_rn(v);
                            p.vth[vo + static_cast<int64_t>(j) * p.vt_pitch] = h;
                            p.vtl[vo + static_cast<int64_t>(j) * p.vt_pitch] = __float2half_rn(__fsub_rn(v, __half2float(h)));
                        }
                    }
                    if (part == 2 && p.kv_vmax) {  // each V column's max |V| (warp-uniform branch)
                        static_assert(E::CH == 8, "the column exchange below assumes 8-column chunks");
                        // max over the warp's 32 rows of each of the 8 columns: three
                        // rounds that each keep half the columns (lane bits 16, 8, 4
                        // pick them), then the last two lane bits
                        float v[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) v[j] = (row0 + lane < p.m) ? fabsf(y[j]) : 0.0f;
#pragma unroll
                        for (int rd = 0, half_n = 4; rd < 3; rd++, half_n >>= 1) {
                            const bool hi_half = (lane >> (4 - rd)) & 1;
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                if (i < half_n) {
                                    const float keep = hi_half ? v[i + half_n] : v[i];
                                    const float send = hi_half ? v[i] : v[i + half_n];
                                    v[i] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, 16 >> rd));
                                }
                            }
                        }
                        float vm = fmaxf(v[0], __shfl_xor_sync(0xffffffffu, v[0], 2));
                        vm = fmaxf(vm, __shfl_xor_sync(0xffffffffu, vm, 1));
                        const int cj = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
                        if ((lane & 3) == 0) atomicMax(p.kv_vmax + (n0 - 2 * p.kvd) + cj, __float_as_uint(vm));
                    }
                }
                if (p.act == TVQ_ACT_GELU_ERF) {
                    float pre[E::CH];
#pragma unroll
                    for (int j = 0; j < E::CH; j++) pre[j] = y[j];
#pragma unroll
                    for (int j = 0; j < E::CH; j += 2) gelu_erf_x2(y[j], y[j + 1]);
                    // the int8 output is the reference's: exact GELU where it matters
                    if (p.Yq) gelu_fix_near_boundary<E::CH>(y, pre, ec.qs.hi);
                } else if (p.act == TVQ_ACT_GELU_TANH) {
#pragma unroll
                    for (int j = 0; j < E::CH; j++) y[j] = gelu_tanh_f32(y[j]);
                } else if (p.act == TVQ_ACT_RELU) {
#pragma unroll
                    for (int j = 0; j < E::CH; j++) y[j] = y[j] > 0.0f ? y[j] : 0.0f;
                }
                stage_and_store<E, true>(p, ec, stage, y, lane, row0, n0, amax, res, kvf);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[b]);
        }
        }
        if (p.amax) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 16));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 8));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
            if (lane == 0) atomicMax(p.amax, __float_as_uint(amax));
        }
    }

    __syncwarp();  // lanes that skipped a single-thread role wait for it here
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// Y[m, n] = bias[n] (or 0): an INT4 GEMM with k = 0 (int4.tkv:232-238 with
// acc = 0).
__global__ void bias_rows_kernel(float* __restrict__ Y, const float* __restrict__ bias, int64_t m, int64_t n) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < m * n; i += (int64_t)gridDim.x * blockDim.x)
        Y[i] = bias ? bias[i % n] : 0.0f;
}

// K == 0: every accumulator is 0, only the epilogue remains (matmul.tkv:14/28
// with acc = 0).
__global__ void gemm_k0_kernel(KParams p) {
    griddep_wait();
    const int64_t total = static_cast<int64_t>(p.m) * p.n;
    if (p.acc_only) {
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
            p.acc_out[i] = 0;
        return;
    }
    const double sa = static_cast<double>(__ldg(p.scale_a));
    double inv_out = 0.0;
    if (p.Yq) {
        const double so = static_cast<double>(__ldg(p.scale_out));
        inv_out = (so > 0.00000001) ? 1.0 / so : 1.0 / 0.00000001;
    }
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int n = static_cast<int>(i % p.n);
        const double sw = static_cast<double>(__ldg(p.scales_w + (p.per_channel ? n : 0)));
        const double bb = p.bias ? static_cast<double>(p.bias[n]) : 0.0;
        const double v = p.per_channel ? __dadd_rn(__dmul_rn(__dmul_rn(0.0, sa), sw), bb) : __dadd_rn(__dmul_rn(0.0, sa * sw), bb);
        float y = apply_act(__double2float_rn(v), p.act);
        if (p.residual) y = __fadd_rn(y, p.residual[i]);
        if (p.acc_out) p.acc_out[i] = 0;
        if (p.Y) p.Y[i] = y;
        if (p.Yq) p.Yq[i] = q8_out(static_cast<double>(y) * inv_out);
        if (p.amax) atomicMax(p.amax, __float_as_uint(fabsf(y)));
    }
}

// ---------------------------------------------------------------- host side

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder() {
    std::call_once(g_encode_once, []() {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    if (!g_encode) {
        set_error(TVQ_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
        return TVQ_ERR_CUDA;
    }
    return TVQ_OK;
}

// 2-D K-major operand [rows, k] of 1-, 2- or 4-byte elements: box {128
// bytes of K, box_rows}, 128-byte swizzle.
int encode_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int box_rows, int elem, int64_t pitch) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch ? pitch : k) * elem};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK / elem), static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = elem == 4   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : elem == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                               : CU_TENSOR_MAP_DATA_TYPE_UINT8;
    CUresult r = g_encode(map, dt, 2,
                          const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error(TVQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")");
        return TVQ_ERR_CUDA;
    }
    return TVQ_OK;
}

// Tensor maps by value: a map holds only the address, shape, pitch and box
// it was encoded from, so a cached one stays valid for any later buffer at
// the same address with the same shape (nothing to invalidate when memory
// is freed).  Repeated calls on the same operands -- weights every call,
// activations of a fixed-shape step -- skip cuTensorMapEncodeTiled.  A
// small direct-mapped table, guarded by a mutex (host threads may launch
// concurrently).
struct MapKey {
    const void* ptr;
    int64_t rows, k, pitch;
    int box_rows, elem;
    bool operator==(const MapKey& o) const {
        return ptr == o.ptr && rows == o.rows && k == o.k && pitch == o.pitch && box_rows == o.box_rows &&
               elem == o.elem;
    }
};
constexpr int kMapCacheSlots = 512;
struct MapCache {
    std::mutex mu;
    MapKey key[kMapCacheSlots];
    CUtensorMap map[kMapCacheSlots];
    bool used[kMapCacheSlots] = {};
};

int make_map(CUtensorMap* map, const void* ptr, int64_t rows, int64_t k, int box_rows, int elem, int64_t pitch = 0) {
    static MapCache cache;
    const MapKey key{ptr, rows, k, pitch, box_rows, elem};
    uint64_t h = reinterpret_cast<uintptr_t>(ptr) * 0x9E3779B97F4A7C15ull;
    h ^= static_cast<uint64_t>(rows) * 0xC2B2AE3D27D4EB4Full + static_cast<uint64_t>(k) * 0x165667B19E3779F9ull;
    h ^= static_cast<uint64_t>(pitch * 131 + box_rows * 7 + elem);
    const int slot = static_cast<int>((h >> 32) % kMapCacheSlots);
    {
        std::lock_guard<std::mutex> lk(cache.mu);
        if (cache.used[slot] && cache.key[slot] == key) {
            *map = cache.map[slot];
            return TVQ_OK;
        }
    }
    const int rc = encode_map(map, ptr, rows, k, box_rows, elem, pitch);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(cache.mu);
    cache.key[slot] = key;
    cache.map[slot] = *map;
    cache.used[slot] = true;
    return TVQ_OK;
}

template <int KIND, int BN, int LEAN = 0>
int launch_tc(const KParams& p, const GemmArgs& g, int grid, cudaStream_t st) {
    using C = Cfg<KIND, BN, LEAN>;
    static int attr_done[64] = {0};  // per device
    int dev = 0;
    TVQ_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !attr_done[dev]) {
        TVQ_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<KIND, BN, LEAN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(C::SMEM)));
        attr_done[dev] = 1;
    }
    CUtensorMap ma, mb, ma2, mb2;
    int rc = make_map(&ma, g.A, p.m, p.k, BM, C::ELEM);
    if (!rc) rc = make_map(&mb, g.W, p.n, p.k, BN, C::ELEM);
    if (!rc && C::NSA == 2) rc = make_map(&ma2, g.A2 ? g.A2 : g.A, p.m, p.k, BM, C::ELEM);  // single: unused
    if (!rc && C::NSB == 2) rc = make_map(&mb2, g.W2 ? g.W2 : g.W, p.n, p.k, BN, C::ELEM);
    if (rc) return rc;
    if (C::NSA == 1) ma2 = ma;
    if (C::NSB == 1) mb2 = mb;
    return launch_pdl(gemm_tc_kernel<KIND, BN, LEAN>, dim3(grid), dim3(EpiOf<KIND>::THREADS), C::SMEM, st, ma, mb, ma2, mb2, p);
}

// Round a float to the TF32 grid (10 explicit mantissa bits), half away
// from zero, so the tensor core reads it without truncation.
__device__ __forceinline__ float round_tf32(float v) {
    const uint32_t u = __float_as_uint(v);
    if ((u & 0x7F800000u) == 0x7F800000u) return v;
    float h = __uint_as_float((u + 0x1000u) & 0xFFFFE000u);
    if ((__float_as_uint(h) & 0x7F800000u) == 0x7F800000u) h = __uint_as_float(u & 0xFFFFE000u);
    return h;
}

// x ~ hi + lo with hi and lo both on the TF32 grid: hi = tf32(x), lo =
// tf32(x - hi); |x - hi - lo| <= 2^-22 |x|.  (hi + lo == x when x itself
// has at most 22 significant bits.)
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  int64_t n) {
    griddep_wait();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float v = x[i];
        const float h = round_tf32(v);
        hi[i] = h;
        lo[i] = (h == v) ? 0.0f : round_tf32(__fsub_rn(v, h));
    }
}

// Row-scaled fp16 split, one warp per row of x [rows, k].  With s = 2^e
// chosen so that max|x| * s lies in [2^14, 2^15), x*s is exact and
// x*s = hi + lo + r with hi = fp16(x*s), lo = fp16(x*s - hi) and |r| <=
// max(2^-22 |x*s|, 2^-25) (the second term: lo in fp16's subnormal range,
// at most 2^-39 of the row's largest |x*s|).  rscale[row] = 1/s.  s is capped at 2^126 (rows with
// max|x| below 2^-111 keep fewer bits); a row holding Inf or NaN gets s = 1
// and carries it into its products.
__global__ void split_f16_rows_kernel(const float* __restrict__ x, __half* __restrict__ hi, __half* __restrict__ lo,
                                      float* __restrict__ rscale, int64_t rows, int64_t k,
                                      const int64_t* __restrict__ perm, int* err) {
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t r = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); r < rows; r += warps) {
        const float* xr = x + r * k;
        float m = 0.0f;
        // element j of the row is x[r, perm[j]] with an act-order permutation
        auto at = [&](int64_t j) -> float {
            if (!perm) return xr[j];
            const int64_t pj = __ldg(perm + j);
            if (pj < 0 || pj >= k) {
                record_error(err, DEVERR_BAD_INDEX);
                return 0.0f;
            }
            return xr[pj];
        };
        for (int64_t j = lane; j < k; j += 32) m = fmaxf(m, fabsf(at(j)));  // fmaxf drops NaN: checked below
        bool bad = false;
        for (int64_t j = lane; j < k; j += 32) bad |= !isfinite(at(j));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        bad = __any_sync(0xffffffffu, bad);
        int sh = 0;
        if (!bad && m > 0.0f) {
            int e;
            frexpf(m, &e);  // m in [2^(e-1), 2^e)
            sh = min(15 - e, 126);
        }
        if (lane == 0) rscale[r] = exp2i(-sh);
        for (int64_t j = lane; j < k; j += 32) {
            const float v = at(j) * exp2i(sh);
            const __half h = __float2half_rn(v);
            hi[r * k + j] = h;
            lo[r * k + j] = __float2half_rn(v - __half2float(h));
        }
    }
}

}  // namespace

int launch_split_f16_rows(const float* x, void* hi, void* lo, float* rscale, int64_t rows, int64_t k,
                          cudaStream_t st, const int64_t* perm) {
    if (rows <= 0) return TVQ_OK;
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    const int grid = static_cast<int>(std::min<int64_t>((rows + 7) / 8, ds->sm_count * 8));
    return launch_pdl(split_f16_rows_kernel, dim3(grid), dim3(256), 0, st, x, static_cast<__half*>(hi),
                      static_cast<__half*>(lo), rscale, rows, k, perm, ds->d_error);
}

int make_tma_f32_sw128(CUtensorMap* map, const float* ptr, int64_t rows, int64_t cols, int box_rows, int64_t pitch) {
    int rc = get_encoder();
    if (rc) return rc;
    if (pitch == 0) pitch = cols;
    TVQ_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && pitch % 4 == 0 && pitch >= cols, TVQ_ERR_UNSUPPORTED,
              "TMA operand must be 16-byte aligned with a 16-byte row pitch");
    return make_map(map, ptr, rows, cols, box_rows, 4, pitch);
}

int make_tma_f16_sw128(CUtensorMap* map, const void* ptr, int64_t rows, int64_t cols, int box_rows, int64_t pitch) {
    int rc = get_encoder();
    if (rc) return rc;
    if (pitch == 0) pitch = cols;
    TVQ_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0 && pitch % 8 == 0 && pitch >= cols, TVQ_ERR_UNSUPPORTED,
              "TMA operand must be 16-byte aligned with a 16-byte row pitch");
    return make_map(map, ptr, rows, cols, box_rows, 2, pitch);
}

int launch_gemm(const GemmArgs& g, cudaStream_t st) {
    TVQ_CHECK(g.m >= 0 && g.n >= 0 && g.k >= 0, TVQ_ERR_INVALID, "negative GEMM size");
    TVQ_CHECK(g.m < (1ll << 31) && g.n < (1ll << 31) && g.k < 133143, TVQ_ERR_UNSUPPORTED,
              "GEMM size out of range (k must stay below 133143 for exact int32 accumulation)");
    if (g.m == 0 || g.n == 0) return TVQ_OK;
    const bool acc_only = g.kind == GEMM_I8 && g.acc_out && !g.Y && !g.Yq && !g.amax;
    TVQ_CHECK(g.kind >= GEMM_I8 && g.kind <= GEMM_W4, TVQ_ERR_INVALID, "unknown GEMM kind");
    const bool split = split_kind(g.kind);
    const bool w4 = g.kind == GEMM_W4;
    const bool single = g.kind == GEMM_F16X3 && !g.A2 && !g.W2;
    const bool asym = g.zp_rows || g.zp_cols;
    TVQ_CHECK(g.kind == GEMM_TF32X3 || single || acc_only || (g.scale_a && g.scales_w), TVQ_ERR_INVALID,
              "scale pointers are required");
    TVQ_CHECK(!asym || (g.kind == GEMM_I8 && g.zp_rows && g.zp_cols && !g.per_channel && !acc_only && !g.kh &&
                        g.zp_k >= 0 && g.zp_k <= g.k),
              TVQ_ERR_INVALID, "zero points need an INT8 GEMM with per-tensor scales and both sum vectors");
    TVQ_CHECK(!asym || (std::llabs(g.zp_a) <= (1ll << 17) && std::llabs(g.zp_w) <= (1ll << 17)), TVQ_ERR_UNSUPPORTED,
              "zero points beyond +-2^17 (the corrected accumulator must stay exact in binary64)");
    TVQ_CHECK(!w4 || (g.group_size > 0 && g.group_size % 16 == 0 && g.k % g.group_size == 0), TVQ_ERR_UNSUPPORTED,
              "the INT4 GEMM needs k a multiple of group_size, group_size a multiple of 16");
    TVQ_CHECK(!w4 || (!g.Yq && !g.residual && g.act == 0 && g.Y && !g.amax), TVQ_ERR_INVALID,
              "the INT4 GEMM writes f32 Y (+ bias) only");
    TVQ_CHECK(!split || (!g.Yq && (single || !g.bias) && !g.residual && g.act == 0 && g.Y && !g.amax),
              TVQ_ERR_INVALID, "the split fp32 GEMM writes plain f32 Y only");
    TVQ_CHECK(!g.Yq || g.scale_out, TVQ_ERR_INVALID, "int8 output needs scale_out");
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    TVQ_CHECK(ds->cc_major == 10, TVQ_ERR_UNSUPPORTED, "the tcgen05 GEMM needs an sm_100 device");

    KParams p{};
    p.m = static_cast<int>(g.m);
    p.n = static_cast<int>(g.n);
    p.k = static_cast<int>(g.k);
    p.bias = g.bias;
    p.residual = g.residual;
    p.Y = g.Y;
    p.Yq = g.Yq;
    p.acc_out = g.acc_out;
    p.scale_a = g.scale_a;
    p.scales_w = g.scales_w;
    p.per_channel = (acc_only || split || w4) ? 0 : g.per_channel;
    p.group_ks = w4 ? static_cast<int>(g.group_size / 16) : 0;
    p.ngroups = w4 ? static_cast<int>(g.k / g.group_size) : 0;
    p.qh = static_cast<__half*>(g.qh);
    p.ql = static_cast<__half*>(g.ql);
    p.kh = static_cast<__half*>(g.kh);
    p.kl = static_cast<__half*>(g.kl);
    p.vth = static_cast<__half*>(g.vth);
    p.vtl = static_cast<__half*>(g.vtl);
    p.kvd = g.kvd;
    p.vt_pitch = g.vt_pitch;
    p.kv_exp = g.kv_exp;
    p.kv_bound = g.kv_bound;
    p.kv_vmax = g.kv_vmax;
    p.single = single ? 1 : 0;
    if (asym) {
        p.zrow = g.zp_rows;
        p.zcol = g.zp_cols;
        p.zpa = static_cast<double>(g.zp_a);
        p.zpw = static_cast<double>(g.zp_w);
        p.zconst = static_cast<double>(g.zp_k * g.zp_a * g.zp_w);  // |.| < 2^52: exact
    }
    p.acc_only = acc_only ? 1 : 0;
    p.act = g.act;
    p.scale_out = g.scale_out;
    p.amax = g.amax;
    p.err = ds->d_error;
    p.num_m_blocks = static_cast<int>((g.m + BM - 1) / BM);
    const int elem = (g.kind == GEMM_TF32X3) ? 4 : (g.kind == GEMM_F16X3 || w4) ? 2 : 1;
    p.num_k_blocks = static_cast<int>((g.k * elem + BK - 1) / BK);
    p.promote_kb = g.kind == GEMM_F16X3 ? F16_PROMOTE_KB : TF32_PROMOTE_KB;
    if (const char* env = getenv("TVQ_TF32_PROMOTE_KB")) p.promote_kb = std::max(1, atoi(env));

    if (g.k == 0 && split && !single) {
        TVQ_CUDA(cudaMemsetAsync(g.Y, 0, sizeof(float) * g.m * g.n, st));
        return TVQ_OK;
    }
    if (g.k == 0 && (w4 || single)) {
        const int grid = static_cast<int>(std::min<int64_t>((g.m * g.n + 255) / 256, ds->sm_count * 8));
        return launch_pdl(bias_rows_kernel, dim3(grid), dim3(256), 0, st, g.Y, g.bias, g.m, g.n);
    }
    if (g.k == 0) {
        const int64_t total = g.m * g.n;
        int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, ds->sm_count * 8));
        return launch_pdl(gemm_k0_kernel, dim3(grid), dim3(256), 0, st, p);
    }
    TVQ_CHECK((g.k * elem) % 16 == 0, TVQ_ERR_UNSUPPORTED, "k must be a multiple of 16 bytes (TMA row pitch)");
    TVQ_CHECK(((reinterpret_cast<uintptr_t>(g.A) | reinterpret_cast<uintptr_t>(g.W)) & 15) == 0, TVQ_ERR_UNSUPPORTED,
              "A and W must be 16-byte aligned");
    TVQ_CHECK(!split || single ||
                  (g.A2 && g.W2 && ((reinterpret_cast<uintptr_t>(g.A2) | reinterpret_cast<uintptr_t>(g.W2)) & 15) == 0),
              TVQ_ERR_UNSUPPORTED, "the split GEMM needs 16-byte aligned low parts");
    TVQ_CHECK(!w4 || (g.A2 && (reinterpret_cast<uintptr_t>(g.A2) & 15) == 0), TVQ_ERR_UNSUPPORTED,
              "the INT4 GEMM needs a 16-byte aligned low part of A");
    TVQ_CHECK(!g.Y || (reinterpret_cast<uintptr_t>(g.Y) & 15) == 0, TVQ_ERR_UNSUPPORTED, "Y must be 16-byte aligned");
    TVQ_CHECK(!g.residual || (reinterpret_cast<uintptr_t>(g.residual) & 15) == 0, TVQ_ERR_UNSUPPORTED,
              "residual must be 16-byte aligned");
    TVQ_CHECK(!g.Yq || (reinterpret_cast<uintptr_t>(g.Yq) & 15) == 0, TVQ_ERR_UNSUPPORTED,
              "Yq must be 16-byte aligned");
    TVQ_CHECK(!g.kh || (g.kind == GEMM_I8 && g.qh && g.ql && g.kl && g.vth && g.vtl && g.kv_exp && g.kv_bound &&
                        g.n == 3 * g.kvd && g.kvd % 64 == 0 && g.vt_pitch >= g.m && g.act == 0 && !g.residual),
              TVQ_ERR_INVALID, "attention operand split needs an INT8 qkv GEMM with N = 3 kvd");
    rc = get_encoder();
    if (rc) return rc;

    // The lean epilogue where every output but the one it writes is off
    // (TVQ_GEMM_LEAN=0 keeps the general one: A/B checks and tuning).
    int lean = 0;
    {
        static const bool lean_off = [] {
            const char* e = getenv("TVQ_GEMM_LEAN");
            return e && atoi(e) == 0;
        }();
        const bool fold_ok = !g.per_channel || g.kind == GEMM_F8 || g.k < 33283;
        const bool plain_amax = (g.kind == GEMM_I8 || g.kind == GEMM_F8) && !acc_only && !asym && !g.acc_out &&
                                !g.kh && g.n % 16 == 0 && fold_ok && !lean_off;
        const bool plain = plain_amax && !g.amax;
        if (plain && g.kind == GEMM_I8 && g.act == TVQ_ACT_GELU_ERF && g.Yq && !g.Y && !g.residual) lean = LEAN_GELU_Q8;
        if (plain && g.act == TVQ_ACT_NONE && g.Y && !g.Yq) lean = LEAN_F32;
        if (plain_amax && g.act == TVQ_ACT_GELU_ERF && g.Y && !g.Yq && !g.residual) lean = LEAN_GELU_F32;
        // the c_attn form with the attention operands (the checks below
        // still apply to g.kh)
        const bool plain_kv = g.kind == GEMM_I8 && !acc_only && !asym && !g.acc_out && !g.amax && g.kh &&
                              g.n % 16 == 0 && fold_ok && !lean_off;
        if (plain_kv && g.act == TVQ_ACT_NONE && g.Y && !g.Yq && !g.residual) lean = LEAN_QKV;
    }
    // Tile width: the widest N tile that still gives every SM a tile.
    int bn = g.force_bn;
    if (bn == 0) {  // TVQ_GEMM_BN=64|128|256 pins the tile width (tuning)
        static const int env_bn = [] {
            const char* e = getenv("TVQ_GEMM_BN");
            const int v = e ? atoi(e) : 0;
            return (v == 64 || v == 128 || v == 256) ? v : 0;
        }();
        bn = env_bn;
    }
    // their partial sums live in registers (BN 256 with a 16-warp epilogue
    // measured slower for the LM head: 381 vs 356 us, two 96 KB stages)
    if ((split || w4) && bn > 128) bn = 128;
    if (bn == 0 && (split || w4)) {
        // The split forms keep 128 (their N = 64 MMAs are issue-bound and
        // re-read A per N tile) unless that leaves SMs without a tile.
        bn = (static_cast<int64_t>(p.num_m_blocks) * ((g.n + 127) / 128) >= ds->sm_count) ? 128 : 64;
    } else if (bn == 0) {
        // Tile width with the least time on the busiest SM: rounds of tiles
        // (ceil(tiles / SMs)) x the time of one tile, the slower of its K
        // loop and its epilogue (which overlap across consecutive tiles).
        // Per 128-byte k-block a 128 x BN tile takes ~0.37 / 0.45 / 0.53 us
        // at BN 64 / 128 / 256 (operand traffic bounds the narrow tiles, so
        // wider tiles do more work per byte), and the exact epilogue ~0.55 ns
        // per output element; ~1 us of fixed cost per tile.  (Measured on
        // B200 over the GPT-2 124M and XL layer shapes.)
        const int64_t mblk = p.num_m_blocks;
        double best = -1.0;
        for (int cand : {256, 128, 64}) {
            const int64_t tiles = mblk * ((g.n + cand - 1) / cand);
            const double t_kb = cand == 256 ? 0.53 : cand == 128 ? 0.45 : 0.37;
            const double t_tile = std::max(p.num_k_blocks * t_kb, 128.0 * cand * 0.55e-3) + 1.0;
            const double cost = static_cast<double>((tiles + ds->sm_count - 1) / ds->sm_count) * t_tile;
            if (best < 0.0 || cost < best * 0.999) {  // ties go to the wider tile
                best = cost;
                bn = cand;
            }
        }
    }
    p.num_n_blocks = static_cast<int>((g.n + bn - 1) / bn);
    p.group_m = 16;
    const int tiles = p.num_m_blocks * p.num_n_blocks;
    const int grid = std::min(tiles, ds->sm_count);
    if (g.kind == GEMM_I8) {
        if (lean == LEAN_GELU_Q8) {
            if (bn == 256) return launch_tc<GEMM_I8, 256, LEAN_GELU_Q8>(p, g, grid, st);
            if (bn == 128) return launch_tc<GEMM_I8, 128, LEAN_GELU_Q8>(p, g, grid, st);
            return launch_tc<GEMM_I8, 64, LEAN_GELU_Q8>(p, g, grid, st);
        }
        if (lean == LEAN_F32) {
            if (bn == 256) return launch_tc<GEMM_I8, 256, LEAN_F32>(p, g, grid, st);
            if (bn == 128) return launch_tc<GEMM_I8, 128, LEAN_F32>(p, g, grid, st);
            return launch_tc<GEMM_I8, 64, LEAN_F32>(p, g, grid, st);
        }
        if (lean == LEAN_GELU_F32) {
            if (bn == 256) return launch_tc<GEMM_I8, 256, LEAN_GELU_F32>(p, g, grid, st);
            if (bn == 128) return launch_tc<GEMM_I8, 128, LEAN_GELU_F32>(p, g, grid, st);
            return launch_tc<GEMM_I8, 64, LEAN_GELU_F32>(p, g, grid, st);
        }
        if (lean == LEAN_QKV) {
            if (bn == 256) return launch_tc<GEMM_I8, 256, LEAN_QKV>(p, g, grid, st);
            if (bn == 128) return launch_tc<GEMM_I8, 128, LEAN_QKV>(p, g, grid, st);
            return launch_tc<GEMM_I8, 64, LEAN_QKV>(p, g, grid, st);
        }
        if (bn == 256) return launch_tc<GEMM_I8, 256>(p, g, grid, st);
        if (bn == 128) return launch_tc<GEMM_I8, 128>(p, g, grid, st);
        return launch_tc<GEMM_I8, 64>(p, g, grid, st);
    }
    if (g.kind == GEMM_F8) {
        if (lean == LEAN_F32) {
            if (bn == 256) return launch_tc<GEMM_F8, 256, LEAN_F32>(p, g, grid, st);
            if (bn == 128) return launch_tc<GEMM_F8, 128, LEAN_F32>(p, g, grid, st);
            return launch_tc<GEMM_F8, 64, LEAN_F32>(p, g, grid, st);
        }
        if (bn == 256) return launch_tc<GEMM_F8, 256>(p, g, grid, st);
        if (bn == 128) return launch_tc<GEMM_F8, 128>(p, g, grid, st);
        return launch_tc<GEMM_F8, 64>(p, g, grid, st);
    }
    if (g.kind == GEMM_F16X3) {
        if (bn >= 128) return launch_tc<GEMM_F16X3, 128>(p, g, grid, st);
        return launch_tc<GEMM_F16X3, 64>(p, g, grid, st);
    }
    if (w4) {
        if (bn >= 128) return launch_tc<GEMM_W4, 128>(p, g, grid, st);
        return launch_tc<GEMM_W4, 64>(p, g, grid, st);
    }
    if (bn >= 128) return launch_tc<GEMM_TF32X3, 128>(p, g, grid, st);
    return launch_tc<GEMM_TF32X3, 64>(p, g, grid, st);
}

int launch_split_tf32(const float* x, float* hi, float* lo, int64_t n, cudaStream_t st) {
    if (n <= 0) return TVQ_OK;
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, ds->sm_count * 8));
    return launch_pdl(split_tf32_kernel, dim3(grid), dim3(256), 0, st, x, hi, lo, n);
}

}  // namespace tvq
