// tvq_attn_tc.cu -- causal attention over packed sequences on the
// 5th-generation tensor cores, head dim 64.
//
// gpt2_attention, tv/training/gpt2_ref.tkv:360-395 (scores q.k / sqrt(hd),
// causal softmax, context = P V), per head, token t of the sequence [s0, s1)
// attending to u in [s0, t].  qkv rows are [Q | K | V] with heads contiguous.
//
// fp32 accuracy on FP16 tensor cores (kind::f16): every operand x is scaled
// by a power of two s (so that its largest value sits in [2^14, 2^15)) and
// split into hi = fp16(x s) and lo = fp16(x s - hi) (|x s - hi - lo| <=
// max(2^-22 |x s|, 2^-25)), and each product is formed as xl*yh + xh*yl +
// xh*yh.  The scales: Q, K and V per head (kv_exp, written with the split
// operands), P = 2^(x - m) in (0, 1] by 2^14.  They are powers of two and are undone exactly: the scores before
// the softmax, the output at the end.  The scores of one 64-key block and
// the P*V partial of one block are each summed in TMEM over K = 64 only; the
// running output is kept in registers with IEEE adds (the tensor core's own
// accumulation is less exact than IEEE fp32 over long sums).
//
// Operands: Q and K as fp16 hi/lo [T, d] and V transposed, V^T hi/lo [d,
// Tp] (keys contiguous, Tp = T rounded up to 8), written by the c_attn GEMM's
// epilogue (or launch_split_kv); the attention kernel brings the query tile
// (A operand of S) and 64-key blocks of K and V^T into shared memory with
// TMA, the blocks through two 2-stage rings, as K-major B operands (of S =
// Q K^T and of P V).  P (hi/lo) is written to tensor memory,
// double-buffered, as the A operand of P V, so the softmax of block j never
// waits for P V of block j-1.
//
// Persistent: one CTA per SM works through (128-query tile, head, key range)
// units, units sorted longest first and dealt to the CTAs in snake order;
// the rings and TMEM buffers run on per-CTA block counts across units, and
// the Q tile is reloaded once the previous unit's S products have read it.
// 384 threads:
//   warp 0      TMA producer (Q, then K blocks)
//   warp 1      MMA issuer for S_j = Q K_j^T into TMEM S[j&1] (M 128, N 64,
//               K 64)
//   warp 2      TMEM allocator (512 columns), then TMA producer of V^T blocks
//   warp 3      MMA issuer for PV_j = P_j V_j into TMEM O[j&1]
//               (a tcgen05.mma costs its issuing thread ~65 cycles whatever
//               N, so the two product streams get one issuer each)
//   warps 4-11  softmax, two warps per TMEM lane group (32 query rows), one
//               per 32-key half of each block: per block the row max
//               exchanged between the pair through shared memory, online
//               softmax in base 2, P (hi/lo) to TMEM, and the previous PV
//               partial folded into the register accumulator (each warp owns
//               32 of the 64 output columns)
// Every wait is a bounded mbarrier wait; on a timeout the kernel records an
// error, drains its MMAs and TMA loads, frees TMEM and returns.
//
// Work items are those of the fp32 kernel (tvq_glue.cu) with 128-row query
// tiles: tiles[i] = {q0, s0, s1, 0}, split[i] = {key begin, key end, partial
// slot or -1, merge entry}; the partials (unnormalised O, m, l) of one query
// tile are merged by the CTA that writes the last of them (a counter per
// entry and head, reset by that CTA).
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>

#include "tvq_common.cuh"
#include "tvq_exact.cuh"
#include "tvq_glue.h"
#include "tvq_kernels.h"

namespace tvq {

namespace {

constexpr int TQ = 128;  // query rows per CTA (TMEM lanes, MMA M)
constexpr int TK = 64;   // keys per block
constexpr int HD = 64;   // head dim
constexpr int NTHREADS = 384;

// shared memory (1024-byte aligned regions), every row 128 bytes = 64 fp16
// with the 128-byte swizzle:
//   Q hi, Q lo      128 query rows x 64 head columns: 16 KB each (TMA)
//   K ring [2]      per stage K hi, K lo: 64 key rows x 64 head columns
//   V^T ring [2]    per stage V^T hi, V^T lo: 64 head rows x 64 keys
constexpr uint32_t PART = TK * 128;                  // 8 KB
constexpr uint32_t QPART = TQ * 128;                 // 16 KB
constexpr uint32_t OFF_QH = 0, OFF_QL = QPART;
constexpr uint32_t KSTAGE = 2 * PART;                // 16 KB: hi then lo
constexpr uint32_t OFF_K = 2 * QPART;                // + s * KSTAGE
constexpr uint32_t OFF_V = OFF_K + 2 * KSTAGE;       // + s * KSTAGE
constexpr uint32_t OFF_RED = OFF_V + 2 * KSTAGE;     // float [2][2][128] row maxima
constexpr uint32_t OFF_LSUM = OFF_RED + 2 * 2 * TQ * 4;  // float [2][128] row sums
// exact-int8 collection: int flag[128], int2 row[128], 4 ints, float row max[128]
constexpr uint32_t OFF_FIX = OFF_LSUM + 2 * TQ * 4;
// exact-int8 bookkeeping: undecided-column masks [row][half], the unit's
// collected rows {q, row max} and their masks, 4 control words, row maxima
constexpr uint32_t OFF_BAR = OFF_FIX + TQ * 8 + TQ * 8 + TQ * 8 + 16 + TQ * 4;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 512 + 1024;

// tensor memory columns: S[2], O[2] (64 f32 each), P[2] (hi 32 + lo 32
// columns each, two fp16 keys per column)
constexpr uint32_t COL_S = 0, COL_O = 128, COL_P = 256;
constexpr uint32_t TMEM_COLS = 512;

// kind::f16, D f32, A and B fp16 K-major, N = 64, M = 128 (both products)
constexpr uint32_t IDESC = (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(64 >> 3) << 17) |
                           (static_cast<uint32_t>(TQ >> 4) << 24);

// device error codes: the wait that gave up first (tens digit: 3 TMA
// producer, 4 MMA issuer, 5 softmax)
enum : int {
    DEVERR_ATTN_K_EMPTY = 31, DEVERR_ATTN_V_EMPTY = 32, DEVERR_ATTN_TMA_DRAIN = 33,
    DEVERR_ATTN_Q_FULL = 41, DEVERR_ATTN_K_FULL = 42, DEVERR_ATTN_S_EMPTY = 43, DEVERR_ATTN_P_FULL = 44,
    DEVERR_ATTN_O_EMPTY = 45, DEVERR_ATTN_V_FULL = 46, DEVERR_ATTN_MMA_DRAIN = 47,
    DEVERR_ATTN_S_FULL = 51, DEVERR_ATTN_XCH = 52, DEVERR_ATTN_O_FULL = 53, DEVERR_ATTN_LXCH = 55,
    DEVERR_ATTN_Q_EMPTY = 34
};

// D[tmem] (+)= A[tmem] * B^T for FP16 operands, A read from tensor memory
// (lane = row of A, two K elements per 32-bit column).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
        " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// 2^x, MUFU approximation (relative error ~2^-22; subnormal results flush
// to zero, 2^-126 of the row maximum)
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// hi / lo fp16 pair of two scaled values, packed two per 32-bit word
// (element a in the low half).
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(__fsub_rn(a, hf.x), __fsub_rn(b, hf.y));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// The P split of the softmax, for 0 <= a, b <= 2^14: hi = the value rounded
// to fp16's 11 significant bits with integer operations (exact in fp16 for
// values >= 2^-14), lo = the exact remainder; one packed conversion each
// (|a - hi - lo| <= max(2^-22 a, 2^-25), as split_h2).
__device__ __forceinline__ void split_p2(float a, float b, uint32_t& hi, uint32_t& lo) {
    uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    ua = (ua + 0xFFFu + ((ua >> 13) & 1u)) & 0xFFFFE000u;  // nearest, ties to even
    ub = (ub + 0xFFFu + ((ub >> 13) & 1u)) & 0xFFFFE000u;
    const float ha = __uint_as_float(ua), hb = __uint_as_float(ub);
    const __half2 h = __floats2half2_rn(ha, hb);
    const __half2 l = __floats2half2_rn(__fsub_rn(a, ha), __fsub_rn(b, hb));
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// split_p2 with the pair already packed (the remainder as one f32x2 subtract)
__device__ __forceinline__ void split_p2x(uint64_t E, float a, float b, uint32_t& hi, uint32_t& lo) {
    uint32_t ua = __float_as_uint(a), ub = __float_as_uint(b);
    ua = (ua + 0xFFFu + ((ua >> 13) & 1u)) & 0xFFFFE000u;  // nearest, ties to even
    ub = (ub + 0xFFFu + ((ub >> 13) & 1u)) & 0xFFFFE000u;
    const float ha = __uint_as_float(ua), hb = __uint_as_float(ub);
    const __half2 h = __floats2half2_rn(ha, hb);
    float la, lb;
    f2_unpack(f2_sub(E, f2_pack(ha, hb)), la, lb);
    const __half2 l = __floats2half2_rn(la, lb);
    hi = *reinterpret_cast<const uint32_t*>(&h);
    lo = *reinterpret_cast<const uint32_t*>(&l);
}

// Q (part 0) or K (part 1) of qkv [T, 3d] -> fp16 hi / lo [T, d] under the
// head scales 2^kv_exp[part heads + h] (standalone path; the session's
// c_attn epilogue writes the same)
__global__ void split_qk16_kernel(const float* __restrict__ qkv, int T, int d, int part,
                                  const int* __restrict__ kv_exp, uint2* __restrict__ kh, uint2* __restrict__ kl) {
    griddep_wait();
    const int d4 = d >> 2;
    const int64_t n = static_cast<int64_t>(T) * d4;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / d4;
        const int c4 = static_cast<int>(i - t * d4);
        const float f = exp2i(kv_exp[part * (d / HD) + (4 * c4) / HD]);
        const float4 v = __ldg(reinterpret_cast<const float4*>(qkv + t * 3 * d) + part * d4 + c4);
        uint2 h, l;
        split_h2(v.x * f, v.y * f, h.x, l.x);
        split_h2(v.z * f, v.w * f, h.y, l.y);
        kh[i] = h;
        kl[i] = l;
    }
}

// V part of qkv [T, 3d] -> V^T fp16 hi / lo [d, Tp] under the head scales
// 2^kv_exp[2 heads + h]: 32 x 32 tiles through shared memory (coalesced on
// both sides); keys T..Tp-1 are written as 0.
__global__ void split_vt16_kernel(const float* __restrict__ qkv, int T, int Tp, int d, const int* __restrict__ kv_exp,
                                  __half* __restrict__ vth, __half* __restrict__ vtl) {
    __shared__ float tile[32][33];
    griddep_wait();
    const int t0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const float f = exp2i(kv_exp[2 * (d / HD) + c0 / HD]);
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int t = t0 + i;
        tile[i][threadIdx.x] = (t < T) ? __ldg(qkv + static_cast<int64_t>(t) * 3 * d + 2 * d + c0 + threadIdx.x) : 0.0f;
    }
    __syncthreads();
    const int t = t0 + threadIdx.x;
    if (t >= Tp) return;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const float v = tile[threadIdx.x][i] * f;
        const __half h = __float2half_rn(v);
        const int64_t o = static_cast<int64_t>(c0 + i) * Tp + t;
        vth[o] = h;
        vtl[o] = __float2half_rn(__fsub_rn(v, __half2float(h)));
    }
}

// max |Q|, max |K| and max |V| per head (f32 bit patterns, atomicMax) of
// qkv [T, 3d]
__global__ void kv_head_amax_kernel(const float* __restrict__ qkv, int T, int d, uint32_t* __restrict__ amax) {
    griddep_wait();
    const int heads = d / HD;
    const int part = blockIdx.y;  // 0 Q, 1 K, 2 V
    const int h = blockIdx.z;
    float m = 0.0f;
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
        const float* src = qkv + static_cast<int64_t>(t) * 3 * d + part * d + h * HD;
        for (int c = threadIdx.x; c < HD; c += blockDim.x) m = fmaxf(m, fabsf(src[c]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) atomicMax(amax + part * heads + h, __float_as_uint(m));
}

// max |V| of each V column of qkv [T, 3d] (f32 bit patterns, atomicMax):
// block x = 64 columns (one head), block y strides over the rows
__global__ void v_col_amax_kernel(const float* __restrict__ qkv, int T, int d, uint32_t* __restrict__ vcol) {
    griddep_wait();
    const int c = blockIdx.x * HD + threadIdx.x;
    float m = 0.0f;
    for (int t = blockIdx.y; t < T; t += gridDim.y) m = fmaxf(m, fabsf(qkv[static_cast<int64_t>(t) * 3 * d + 2 * d + c]));
    atomicMax(vcol + c, __float_as_uint(m));
}

__global__ void kv_exp_from_amax_kernel(const uint32_t* __restrict__ amax, int n, int* __restrict__ kv_exp) {
    griddep_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) kv_exp[i] = pow2_exp_below_2p15(__uint_as_float(amax[i]));
}

struct AttnParams {
    const float* qkv;
    const int4* tiles;
    const int4* split;
    int d, nheads;
    float scale2;  // log2(e) / sqrt(hd)
    float* out;
    int8_t* outq;
    const float* qscale;
    uint32_t* amax;
    float* part_o;
    float2* part_ml;
    const int4* comb;  // per merge entry {q0, seq end, first slot, count}; split[i].w = entry of item i
    int* counters;     // per (entry, head): partials counted in (0 between launches)
    const int* kv_exp; // [3 * nheads]: Q, K and V head scales 2^kv_exp of the split operands
    int* err;
    int nunits;        // work units: (item, head) = (u / nheads, u % nheads), items longest first
    // exact int8 output: rows whose int8 context the kernel's error bound
    // (2^-20 max |V| of the column) could round differently from the
    // reference's f64 context are recomputed by attention_fix_kernel, only
    // the columns it could not decide
    const uint32_t* vmax;  // [d] max |V| per V column (float bits) or null
    int4* fix;             // rows {q, row max (float bits), head, sequence start}
    uint2* fix_mask;       // their undecided columns (bit c of .x / .y: column c / 32 + c)
    int* fix_n;            // [0] rows, [1] rows taken by the fix-up, [2] finished fix-up CTAs
    int fix_cap;
};

// Unit k of this CTA: rounds of gridDim.x units in snake order (CTA c takes
// c in even rounds, gridDim.x - 1 - c in odd ones), so that with units
// sorted longest first every CTA's total stays within about one unit of the
// others.
__device__ __forceinline__ int unit_of(int k) {
    const int G = static_cast<int>(gridDim.x), c = static_cast<int>(blockIdx.x);
    return k * G + ((k & 1) ? (G - 1 - c) : c);
}

// One work unit: query tile [q0, q0 + 128) of the sequence ending at s1, keys
// [kb, ke) (blocks from kb rounded down to 8 keys, 16 bytes of fp16: the TMA
// rule for the V^T key coordinate; keys below kb are masked), partial slot
// (or -1) and merge entry, head.
struct Unit {
    int q0, s0, s1, kb, ke, part, entry, kb_al, nkb, head;
};

__device__ __forceinline__ Unit load_unit(const AttnParams& p, int u) {
    Unit w;
    const int item = u / p.nheads;
    w.head = u - item * p.nheads;
    const int4 tl = __ldg(p.tiles + item), sp = __ldg(p.split + item);
    w.q0 = tl.x;
    w.s0 = tl.y;
    w.s1 = tl.z;
    w.kb = sp.x;
    w.ke = sp.y;
    w.part = sp.z;
    w.entry = sp.w;
    w.kb_al = w.kb & ~7;
    w.nkb = (w.ke - w.kb_al + TK - 1) / TK;
    return w;
}

// Byte offset of the 16-byte chunk (row r, chunk c of its 128-byte row) in
// a tile of 128-byte rows with the 128-byte swizzle (chunk ^= row % 8).
__device__ __forceinline__ uint32_t sw128(int r, int c) {
    return static_cast<uint32_t>(r) * 128u + static_cast<uint32_t>((c ^ (r & 7)) << 4);
}

__global__ void __launch_bounds__(NTHREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQh, const __grid_constant__ CUtensorMap tmQl,
                        const __grid_constant__ CUtensorMap tmKh, const __grid_constant__ CUtensorMap tmKl,
                        const __grid_constant__ CUtensorMap tmVh, const __grid_constant__ CUtensorMap tmVl,
                        const AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* red = reinterpret_cast<float*>(sm + OFF_RED);    // [parity][half][row]
    float* lsum = reinterpret_cast<float*>(sm + OFF_LSUM);  // [half][row]
    uint32_t* fx_mask = reinterpret_cast<uint32_t*>(sm + OFF_FIX);      // [row][half] undecided columns
    int2* fx_row = reinterpret_cast<int2*>(sm + OFF_FIX + TQ * 8);        // collected {q, row max}
    uint2* fx_rmask = reinterpret_cast<uint2*>(sm + OFF_FIX + TQ * 16);   // their column masks
    int* fx_ctl = reinterpret_cast<int*>(sm + OFF_FIX + TQ * 24);         // count, first list slot, -, rows
    float* fx_m = reinterpret_cast<float*>(sm + OFF_FIX + TQ * 24 + 16);  // [row] row max of a flagged row
    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + OFF_BAR);
    uint64_t* k_full = bars;           // [2]
    uint64_t* k_empty = bars + 2;      // [2]
    uint64_t* v_full = bars + 4;       // [2]
    uint64_t* v_empty = bars + 6;      // [2]
    uint64_t* s_full = bars + 8;       // [2]
    uint64_t* s_empty = bars + 10;     // [2]
    uint64_t* p_full = bars + 12;      // [2]
    uint64_t* o_full = bars + 14;      // [2]
    uint64_t* o_empty = bars + 16;     // [2]
    uint64_t* q_full = bars + 18;
    uint64_t* drain = bars + 19;       // [2]: S issuer, PV issuer
    uint64_t* xch = bars + 21;         // [4 lane groups][2 parities]: row-max exchange
    uint64_t* lxch = bars + 29;        // [4]: row-sum exchange
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 33);
    uint64_t* q_empty = bars + 34;     // the S products of a unit have read its Q tile

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int b = 0; b < 2; b++) {
            mbar_init(&k_full[b], 1);
            mbar_init(&k_empty[b], 1);
            mbar_init(&v_full[b], 1);
            mbar_init(&v_empty[b], 1);
            mbar_init(&s_full[b], 1);
            mbar_init(&s_empty[b], 8);
            mbar_init(&p_full[b], 8);
            mbar_init(&o_full[b], 1);
            mbar_init(&o_empty[b], 8);
        }
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        mbar_init(&drain[0], 1);
        mbar_init(&drain[1], 1);
        for (int i = 0; i < 8; i++) mbar_init(&xch[i], 2);
        for (int i = 0; i < 4; i++) mbar_init(&lxch[i], 2);
        fence_barrier_init();
    }
    if (threadIdx.x >= 128 && threadIdx.x < 128 + 2 * TQ) fx_mask[threadIdx.x - 128] = 0u;
    if (threadIdx.x < 4) fx_ctl[threadIdx.x] = 0;
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmQh);
        tma_prefetch_desc(&tmQl);
        tma_prefetch_desc(&tmKh);
        tma_prefetch_desc(&tmKl);
        tma_prefetch_desc(&tmVh);
        tma_prefetch_desc(&tmVl);
    }
    if (warp == 2) {
        tmem_alloc(tmem_holder, TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    griddep_wait();  // qkv and the split K / V^T come from the previous kernels

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        if (lane == 0) {
            int gk = 0, nq = 0;  // K blocks and Q tiles issued so far (all units)
            bool ok = true;
            for (int k = 0; ok; k++) {
                const int u = unit_of(k);
                if (u >= p.nunits) break;
                const Unit w = load_unit(p, u);
                // the query tile (rows past the sequence only feed rows that
                // are never written; rows past T read as 0), once the previous
                // unit's S products are done with the buffer
                if (k > 0 && !mbar_wait(q_empty, (k - 1) & 1, p.err, DEVERR_ATTN_Q_EMPTY)) break;
                mbar_arrive_expect_tx(q_full, 2 * QPART);
                tma_load_2d(&tmQh, q_full, sm + OFF_QH, w.head * HD, w.q0);
                tma_load_2d(&tmQl, q_full, sm + OFF_QL, w.head * HD, w.q0);
                nq++;
                for (int j = 0; j < w.nkb; j++, gk++) {
                    const int s = gk & 1;
                    const uint32_t ph = ((gk >> 1) & 1) ^ 1;
                    const int key = w.kb_al + j * TK;  // a multiple of 8
                    if (!mbar_wait(&k_empty[s], ph, p.err, DEVERR_ATTN_K_EMPTY)) { ok = false; break; }
                    mbar_arrive_expect_tx(&k_full[s], KSTAGE);
                    uint8_t* ks = sm + OFF_K + s * KSTAGE;
                    tma_load_2d(&tmKh, &k_full[s], ks, w.head * HD, key);
                    tma_load_2d(&tmKl, &k_full[s], ks + PART, w.head * HD, key);
                }
            }
            // every issued load lands before the CTA may exit
            if (nq > 0) mbar_wait(q_full, (nq - 1) & 1, p.err, DEVERR_ATTN_TMA_DRAIN);
            for (int g2 = gk > 2 ? gk - 2 : 0; g2 < gk; g2++)
                mbar_wait(&k_full[g2 & 1], (g2 >> 1) & 1, p.err, DEVERR_ATTN_TMA_DRAIN);
        }
    } else if (warp == 2) {
        // ------------------------------------------------ TMA producer of V^T
        // (its own thread: K blocks run ahead of the PV products)
        if (lane == 0) {
            int gv = 0;  // V blocks issued so far (all units)
            bool ok = true;
            for (int k = 0; ok; k++) {
                const int u = unit_of(k);
                if (u >= p.nunits) break;
                const Unit w = load_unit(p, u);
                for (int j = 0; j < w.nkb; j++, gv++) {
                    const int s = gv & 1;
                    const uint32_t ph = ((gv >> 1) & 1) ^ 1;
                    const int key = w.kb_al + j * TK;
                    if (!mbar_wait(&v_empty[s], ph, p.err, DEVERR_ATTN_V_EMPTY)) { ok = false; break; }
                    mbar_arrive_expect_tx(&v_full[s], KSTAGE);
                    uint8_t* vs = sm + OFF_V + s * KSTAGE;
                    tma_load_2d(&tmVh, &v_full[s], vs, key, w.head * HD);
                    tma_load_2d(&tmVl, &v_full[s], vs + PART, key, w.head * HD);
                }
            }
            for (int g2 = gv > 2 ? gv - 2 : 0; g2 < gv; g2++)
                mbar_wait(&v_full[g2 & 1], (g2 >> 1) & 1, p.err, DEVERR_ATTN_TMA_DRAIN);
        }
    } else if (warp == 1) {
        // ------------------------------------------------ S issuer
        if (lane == 0) {
            const uint32_t sbase = smem_u32(sm);
            int gs = 0;  // S blocks issued so far (all units)
            bool ok = true;
            for (int k = 0; ok; k++) {
                const int u = unit_of(k);
                if (u >= p.nunits) break;
                const int nkb = load_unit(p, u).nkb;
                if (!mbar_wait(q_full, k & 1, p.err, DEVERR_ATTN_Q_FULL)) break;
                for (int j = 0; j < nkb; j++, gs++) {
                    const int b = gs & 1;
                    const uint32_t ph = (gs >> 1) & 1;
                    if (!mbar_wait(&k_full[b], ph, p.err, DEVERR_ATTN_K_FULL) ||
                        !mbar_wait(&s_empty[b], ph ^ 1, p.err, DEVERR_ATTN_S_EMPTY)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + COL_S + b * 64;
                    const uint32_t kbs = sbase + OFF_K + b * KSTAGE;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {  // 16 head columns (32 bytes) per instruction
                        const uint64_t qh = smem_desc_k_sw128(sbase + OFF_QH + kk * 32);
                        const uint64_t ql = smem_desc_k_sw128(sbase + OFF_QL + kk * 32);
                        const uint64_t kh = smem_desc_k_sw128(kbs + kk * 32);
                        const uint64_t kl = smem_desc_k_sw128(kbs + PART + kk * 32);
                        umma_f16(d_tmem, ql, kh, IDESC, kk ? 1u : 0u);
                        umma_f16(d_tmem, qh, kl, IDESC, 1u);
                        umma_f16(d_tmem, qh, kh, IDESC, 1u);
                    }
                    umma_commit(&s_full[b]);
                    umma_commit(&k_empty[b]);
                }
                if (ok) umma_commit(q_empty);  // the Q tile is free once these products complete
            }
            // all issued MMAs retire before TMEM is released
            umma_commit(&drain[0]);
            mbar_wait(&drain[0], 0, p.err, DEVERR_ATTN_MMA_DRAIN);
        }
    } else if (warp == 3) {
        // ------------------------------------------------ PV issuer
        if (lane == 0) {
            const uint32_t sbase = smem_u32(sm);
            int gp = 0;  // PV blocks issued so far (all units)
            bool ok = true;
            for (int k = 0; ok; k++) {
                const int u = unit_of(k);
                if (u >= p.nunits) break;
                const int nkb = load_unit(p, u).nkb;
                for (int i = 0; i < nkb; i++, gp++) {
                    const int b = gp & 1;
                    const uint32_t ph = (gp >> 1) & 1;
                    if (!mbar_wait(&p_full[b], ph, p.err, DEVERR_ATTN_P_FULL) ||
                        !mbar_wait(&o_empty[b], ph ^ 1, p.err, DEVERR_ATTN_O_EMPTY) ||
                        !mbar_wait(&v_full[b], ph, p.err, DEVERR_ATTN_V_FULL)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + COL_O + b * 64;
                    const uint32_t vb = sbase + OFF_V + b * KSTAGE;
                    const uint32_t pcol = tmem_base + COL_P + b * 64;  // hi: +0..31, lo: +32..63
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {  // 16 keys (32 bytes of V^T rows, 8 P columns) per instruction
                        const uint64_t vh = smem_desc_k_sw128(vb + kk * 32);
                        const uint64_t vl = smem_desc_k_sw128(vb + PART + kk * 32);
                        const uint32_t pc = 8 * kk;
                        umma_f16_ts(d_tmem, pcol + 32 + pc, vh, IDESC, kk ? 1u : 0u);
                        umma_f16_ts(d_tmem, pcol + pc, vl, IDESC, 1u);
                        umma_f16_ts(d_tmem, pcol + pc, vh, IDESC, 1u);
                    }
                    umma_commit(&o_full[b]);   // PV_i in O[b]; P[b] free again
                    umma_commit(&v_empty[b]);
                }
            }
            umma_commit(&drain[1]);
            mbar_wait(&drain[1], 0, p.err, DEVERR_ATTN_MMA_DRAIN);
        }
    } else if (warp >= 4) {
        // ------------------------------------------------ softmax
        const int g = warp & 3;          // TMEM lane group
        const int h = (warp - 4) >> 2;   // key half of each block, output half
        const int r = 32 * g + lane;     // query row of the tile = TMEM lane
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * g) << 16);
        bool alive = true;
        // 1 / scale of the int8 output, once per CTA
        InvScale qs{0.0, 0.0f, 0.0f};
        if (p.outq) qs = make_inv_scale(static_cast<double>(__ldg(p.qscale)));
        int gj = 0;  // blocks processed so far (all units)
        for (int k = 0; alive; k++) {
            const int u = unit_of(k);
            if (u >= p.nunits) break;
            const Unit w = load_unit(p, u);
            const int head = w.head, q0 = w.q0, s1 = w.s1, kb = w.kb, ke = w.ke, part = w.part;
            const int kb_al = w.kb_al, nkb = w.nkb;
            const int q = q0 + r;
            // scores: S = acc 2^-(sq + sk) exactly, times log2(e) / sqrt(hd)
            const int sq = __ldg(p.kv_exp + head), sk = __ldg(p.kv_exp + p.nheads + head),
                      sv = __ldg(p.kv_exp + 2 * p.nheads + head);
            const float xs = p.scale2 * exp2i(-sq) * exp2i(-sk);
            float o[32];
#pragma unroll
            for (int c = 0; c < 32; c++) o[c] = 0.0f;
            float m = -INFINITY, l = 0.0f, alpha_prev = 0.0f;
            for (int j = 0; j < nkb; j++) {
                const int gb = gj + j;  // this CTA's block count: the ring and TMEM buffer phases
                const int b = gb & 1;
                const uint32_t ph = (gb >> 1) & 1;
                bool got = mbar_wait(&s_full[b], ph, p.err, DEVERR_ATTN_S_FULL);
                if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
                tc_fence_after();
                uint32_t sr[32];
                tmem_ld32(lane_base + COL_S + b * 64 + 32 * h, sr);
                tmem_ld_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_empty[b]);
                // causal + key-range mask, scale to base 2: key k0 + c is visible
                // for lo <= c <= hi
                const int k0 = kb_al + j * TK + 32 * h;
                const int lo = kb - k0, hi = min(q, ke - 1) - k0;
                uint64_t x2[16];  // the scaled scores, two keys per register pair (f32x2)
                float mx = -INFINITY, mx2 = -INFINITY;
                if (lo <= 0 && hi >= 31) {  // every key of the half visible: most blocks
                    const uint64_t XS = f2_pack(xs, xs);
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        x2[c / 2] = f2_mul(f2_pack(__uint_as_float(sr[c]), __uint_as_float(sr[c + 1])), XS);
                        float a, bq;
                        f2_unpack(x2[c / 2], a, bq);
                        mx = fmaxf(mx, a);
                        mx2 = fmaxf(mx2, bq);
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < 32; c += 2) {
                        const float a = (c >= lo && c <= hi) ? __fmul_rn(__uint_as_float(sr[c]), xs) : -INFINITY;
                        const float bq = (c + 1 >= lo && c + 1 <= hi) ? __fmul_rn(__uint_as_float(sr[c + 1]), xs) : -INFINITY;
                        x2[c / 2] = f2_pack(a, bq);
                        mx = fmaxf(mx, a);
                        mx2 = fmaxf(mx2, bq);
                    }
                }
                mx = fmaxf(mx, mx2);
                // row max over both halves: exchange with the partner warp
                red[(b * 2 + h) * TQ + r] = mx;
                __syncwarp();
                if (lane == 0) mbar_arrive(&xch[g * 2 + b]);
                got = mbar_wait(&xch[g * 2 + b], ph, p.err, DEVERR_ATTN_XCH);
                if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
                mx = fmaxf(mx, red[(b * 2 + (h ^ 1)) * TQ + r]);
                const float mnew = fmaxf(m, mx);
                const float mref = (mnew == -INFINITY) ? 0.0f : mnew;  // a row with no visible key yet stays empty
                const float alpha = ex2_approx(m - mref);
                // P_j = 2^(x - m + 14) in (0, 2^14] (l and O are kept in units of
                // 2^14) as fp16 hi + lo (|error| <= max(2^-22 P, 2^-25)) into
                // P[b]; P[b] was last read by PV_{j-2}, whose completion the
                // previous iteration already waited for
                const uint64_t M14 = f2_pack(mref - 14.0f, mref - 14.0f);
                uint32_t phi[16], plo[16];
                uint64_t acc2[2] = {0ull, 0ull};  // (+0, +0) pairs
#pragma unroll
                for (int c = 0; c < 32; c += 2) {
                    float d0, d1;
                    f2_unpack(f2_sub(x2[c / 2], M14), d0, d1);
                    const float e0 = ex2_approx(d0), e1 = ex2_approx(d1);
                    const uint64_t E = f2_pack(e0, e1);
                    acc2[(c >> 1) & 1] = f2_add(acc2[(c >> 1) & 1], E);
                    split_p2x(E, e0, e1, phi[c / 2], plo[c / 2]);
                }
                float s0, s1, s2, s3;
                f2_unpack(acc2[0], s0, s1);
                f2_unpack(acc2[1], s2, s3);
                const float sum = (s0 + s1) + (s2 + s3);
                tmem_st16(lane_base + COL_P + b * 64 + 16 * h, phi);
                tmem_st16(lane_base + COL_P + b * 64 + 32 + 16 * h, plo);
                l = fmaf(l, alpha, sum);
                m = mnew;
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[b]);
                // fold PV_{j-1} into the register accumulator
                if (j >= 1) {
                    const int bp = (gb - 1) & 1;
                    got = mbar_wait(&o_full[bp], ((gb - 1) >> 1) & 1, p.err, DEVERR_ATTN_O_FULL);
                    if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
                    tc_fence_after();
                    uint32_t pv[32];
                    tmem_ld32(lane_base + COL_O + bp * 64 + 32 * h, pv);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&o_empty[bp]);
#pragma unroll
                    for (int c = 0; c < 32; c++) o[c] = fmaf(o[c], alpha_prev, __uint_as_float(pv[c]));
                }
                alpha_prev = alpha;
            }
            if (alive) {
                const int gl = gj + nkb - 1;
                const int bp = gl & 1;
                const bool got = mbar_wait(&o_full[bp], (gl >> 1) & 1, p.err, DEVERR_ATTN_O_FULL);
                alive = __all_sync(0xffffffffu, got);
                if (alive) {
                    tc_fence_after();
                    uint32_t pv[32];
                    tmem_ld32(lane_base + COL_O + bp * 64 + 32 * h, pv);
                    tmem_ld_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&o_empty[bp]);  // the next unit's PV may reuse O[bp]
#pragma unroll
                    for (int c = 0; c < 32; c++) o[c] = fmaf(o[c], alpha_prev, __uint_as_float(pv[c]));
                }
            }
            gj += nkb;
            // O was summed in units of 2^(14 + sv): back to the true scale (exact)
#pragma unroll
            for (int c = 0; c < 32; c++) o[c] = o[c] * exp2i(-sv);  // O and l both in units of 2^14 from here
            if (alive) {  // row sum over both halves
                lsum[h * TQ + r] = l;
                __syncwarp();
                if (lane == 0) mbar_arrive(&lxch[g]);
                const bool got = mbar_wait(&lxch[g], k & 1, p.err, DEVERR_ATTN_LXCH);
                alive = __all_sync(0xffffffffu, got);
                if (alive) l += lsum[(h ^ 1) * TQ + r];
            }
            // Key-chunk items: write the unnormalised partial (O, m, l); the CTA
            // that completes the set merges them (the last to count in).
            bool write_out = part < 0;
            bool merged = false;
            if (part >= 0) {
                if (alive) {
                    const int64_t slot = static_cast<int64_t>(part) * p.nheads + head;
                    float4* dst = reinterpret_cast<float4*>(p.part_o + (slot * TQ + r) * HD + 32 * h);
#pragma unroll
                    for (int c4 = 0; c4 < 8; c4++)
                        dst[c4] = make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
                    if (h == 0) p.part_ml[slot * TQ + r] = make_float2(m, l);
                }
                __threadfence();
                named_bar_sync(1, 256);  // all eight softmax warps wrote their part
                int* last_flag = reinterpret_cast<int*>(lsum);  // lsum is free again (both halves read it)
                if (threadIdx.x == 128) {
                    int* ctr = p.counters + static_cast<int64_t>(w.entry) * p.nheads + head;
                    const int prev = atomicAdd(ctr, 1);
                    const int last = (prev == p.comb[w.entry].w - 1) ? 1 : 0;
                    if (last) *ctr = 0;  // every other part has counted in: ready for the next launch
                    last_flag[TQ * 2 - 1] = last;
                }
                named_bar_sync(1, 256);
                write_out = merged = last_flag[TQ * 2 - 1] != 0;
                if (merged) __threadfence();  // the other CTAs' partials are visible from here
            }
            if (write_out && alive) {
                float am = 0.0f;
                float mfin = m;  // the row's max of the base-2 scores (after the merge: over all parts)
                if (merged) {
                    // m = max m_c, l = sum l_c 2^(m_c - m), O = sum O_c 2^(m_c - m) / l, in slot order
                    const int4 ce = p.comb[w.entry];  // {q0, seq end, first slot, count}
                    float mm = -INFINITY;
                    for (int t = 0; t < ce.w; t++) {
                        const int slot_k = ce.z + t;
                        const float mk = (slot_k == part)
                                             ? m
                                             : p.part_ml[(static_cast<int64_t>(slot_k) * p.nheads + head) * TQ + r].x;
                        mm = fmaxf(mm, mk);
                    }
                    mfin = mm;
                    float lt = 0.0f, acc[32];
#pragma unroll
                    for (int c = 0; c < 32; c++) acc[c] = 0.0f;
                    for (int t = 0; t < ce.w; t++) {
                        const int slot_k = ce.z + t;
                        const int64_t sl = static_cast<int64_t>(slot_k) * p.nheads + head;
                        const float2 ml = (slot_k == part) ? make_float2(m, l) : p.part_ml[sl * TQ + r];
                        const float wgt = (ml.x == -INFINITY) ? 0.0f : exp2f(ml.x - mm);
                        lt = fmaf(ml.y, wgt, lt);
                        if (slot_k == part) {
#pragma unroll
                            for (int c = 0; c < 32; c++) acc[c] = fmaf(o[c], wgt, acc[c]);
                        } else {
                            const float4* src = reinterpret_cast<const float4*>(p.part_o + (sl * TQ + r) * HD + 32 * h);
#pragma unroll
                            for (int c4 = 0; c4 < 8; c4++) {
                                const float4 v = src[c4];
                                acc[4 * c4] = fmaf(v.x, wgt, acc[4 * c4]);
                                acc[4 * c4 + 1] = fmaf(v.y, wgt, acc[4 * c4 + 1]);
                                acc[4 * c4 + 2] = fmaf(v.z, wgt, acc[4 * c4 + 2]);
                                acc[4 * c4 + 3] = fmaf(v.w, wgt, acc[4 * c4 + 3]);
                            }
                        }
                    }
                    const float il = 1.0f / lt;
#pragma unroll
                    for (int c = 0; c < 32; c++) o[c] = acc[c] * il;
                } else {
                    const float il = 1.0f / l;
#pragma unroll
                    for (int c = 0; c < 32; c++) o[c] = o[c] * il;
                }
                if (q < s1) {
                    const int64_t base = static_cast<int64_t>(q) * p.d + head * HD + 32 * h;
#pragma unroll
                    for (int c = 0; c < 32; c++) am = fmaxf(am, fabsf(o[c]));
                    if (p.out) {
                        float4* dst = reinterpret_cast<float4*>(p.out + base);
#pragma unroll
                        for (int c4 = 0; c4 < 8; c4++)
                            dst[c4] = make_float4(o[4 * c4], o[4 * c4 + 1], o[4 * c4 + 2], o[4 * c4 + 3]);
                    }
                    if (p.outq) {
                        // branch-free fast quantize of all 32, rare f64 fix-ups after
                        union { int8_t b[32]; uint4 u[2]; } v;
                        uint32_t bad = 0;
#pragma unroll
                        for (int c = 0; c < 32; c++) bad |= quant_fast(o[c], qs, v.b[c]) ? 0u : (1u << c);
                        if (bad) {
#pragma unroll
                            for (int c = 0; c < 32; c++)
                                if (bad & (1u << c)) v.b[c] = quant_exact(o[c], qs);
                        }
                        if (p.fix) {
                            // |o - reference| <= 2^-20 max|V| of the column (measured on
                            // B200: at most 2^-20.9 of the column's running max |V|): a
                            // value that close to an int8 rounding boundary is recomputed
                            // exactly by attention_fix_kernel
                            const float k20 = qs.hi * 9.5367431640625e-07f;
                            const uint32_t* vcol = p.vmax + head * HD + 32 * h;
                            uint32_t near = 0u;  // this half's undecided columns
#pragma unroll
                            for (int c = 0; c < 32; c++) {
                                const float mrg = fmaf(__uint_as_float(__ldg(vcol + c)), k20, 1.52587890625e-05f);
                                const float t = __fmul_rn(o[c], qs.hi);
                                const float rr = __fsub_rn(__fadd_rn(t, 12582912.0f), 12582912.0f);
                                near |= (fabsf(fabsf(__fsub_rn(t, rr)) - 0.5f) < mrg) ? (1u << c) : 0u;
                            }
                            if (near) {  // either half (both hold the same row max)
                                fx_mask[2 * r + h] = near;
                                fx_m[r] = mfin;
                            }
                        }
                        if ((reinterpret_cast<uintptr_t>(p.outq + base) & 15) == 0) {
                            uint4* dst = reinterpret_cast<uint4*>(p.outq + base);
                            dst[0] = v.u[0];
                            dst[1] = v.u[1];
                        } else {
                            uint32_t* dst = reinterpret_cast<uint32_t*>(p.outq + base);
#pragma unroll
                            for (int c4 = 0; c4 < 8; c4++)
                                dst[c4] = (c4 & 3) == 0 ? v.u[c4 >> 2].x : (c4 & 3) == 1 ? v.u[c4 >> 2].y
                                                       : (c4 & 3) == 2 ? v.u[c4 >> 2].z : v.u[c4 >> 2].w;
                        }
                    }
                }
                if (p.amax) {
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
                    if (lane == 0) atomicMax(p.amax, __float_as_uint(am));
                }
            }
            if (p.fix && p.outq && write_out) {  // write_out is uniform over the 256 softmax threads; alive may not be
                // the unit's undecided rows, once each, as one group: a unit
                // entry and its rows (all of one head and one sequence)
                named_bar_sync(3, 256);  // every mask is set
                if (h == 0 && (fx_mask[2 * r] | fx_mask[2 * r + 1])) {
                    const int slot = atomicAdd(&fx_ctl[0], 1);
                    fx_row[slot] = make_int2(q, __float_as_int(fx_m[r]));
                    fx_rmask[slot] = make_uint2(fx_mask[2 * r], fx_mask[2 * r + 1]);
                    fx_mask[2 * r] = 0u;
                    fx_mask[2 * r + 1] = 0u;
                }
                named_bar_sync(3, 256);
                if (threadIdx.x == 128) {
                    const int cnt = fx_ctl[0];
                    int b = -1;
                    if (cnt > 0) {
                        b = atomicAdd(p.fix_n, cnt);
                        if (b + cnt > p.fix_cap) {  // list full: recorded, these rows stay as computed
                            record_error(p.err, DEVERR_FIX_FULL);
                            b = -1;
                        }
                    }
                    fx_ctl[1] = b;
                    fx_ctl[3] = cnt;
                    fx_ctl[0] = 0;
                }
                named_bar_sync(3, 256);
                const int cnt = fx_ctl[3], b = fx_ctl[1];
                const int i = threadIdx.x - 128;
                if (b >= 0 && i < cnt) {
                    p.fix[b + i] = make_int4(fx_row[i].x, fx_row[i].y, head, w.s0);
                    p.fix_mask[b + i] = fx_rmask[i];
                }
            }
            // the eight softmax warps leave the unit loop together (each unit
            // then runs the same named barriers in every warp)
            alive = named_bar_and(2, 256, alive);
        }
    }

    __syncwarp();  // lanes that skipped a single-thread role wait for it here
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

// The undecided columns of the context rows the tensor-core kernel listed
// (AttnParams::fix), recomputed as the reference computes them
// (gpt2_ref.tkv:360-395, the oracle's tvo_attention_causal): scores q.k /
// sqrt(hd) in binary64, softmax weights with exp in binary64, the P V sum
// in binary64 and one rounding to binary32, then the exact int8 quantize.
// The row's other columns are already the reference's (their int8 values
// were decided by the kernel's error bound) and stay as written.
//
// One 16-warp CTA per listed row (persistent, one CTA per SM, rows taken
// from a counter).  Four lanes share a key: each holds 16 of q's dimensions
// in registers (binary64) and reads the matching 64 bytes of the key's K
// row, so a warp scores eight keys per step (one binary64 exp stream for
// the eight) with coalesced 16-byte loads, the next step's loads in flight
// while one step is scored, and two shuffle steps finish each dot product.  The V value of every undecided
// column (up to FIX_MAXC per pass) is loaded with the key; the weight sum
// and the column sums stay in registers until one block reduction per row.
// The weights are exp(s - c) with c the tensor-core kernel's row max (base-2
// units, times ln 2) instead of the exact max: the context sum(e_u v_u) /
// sum(e_u) does not depend on it.  The sums run in another order than the
// reference's sequential loops; that moves the binary64 result by about
// 1e-16 of its size, which changes its binary32 rounding with a probability
// of about 2^-28 per value.
constexpr int FIX_THREADS = 512;
constexpr int FIX_LPK = 4;                 // lanes per key
constexpr int FIX_KPS = 32 / FIX_LPK;      // keys per warp step
constexpr int FIX_UNROLL = 1;              // steps per load group (two groups in flight)
constexpr int FIX_MAXC = 4;                // undecided columns per pass
// RG row groups per CTA, each of FIX_THREADS / RG threads working on its
// own row (its own reductions and a named barrier of its own): one group
// (all 16 warps on a row) when the list is short and its rows long, as in
// one 1024-token sequence; several when the list holds tens of thousands of
// rows (a packed batch of requests), so that more rows have loads in flight.
template <int RG>
__global__ void __launch_bounds__(FIX_THREADS, 1) attention_fix_kernel(const float* __restrict__ qkv,
                                                                       const int4* __restrict__ rows,
                                                                       const uint2* __restrict__ masks, int* fix_n,
                                                                       int cap, int d, float* __restrict__ out,
                                                                       int8_t* __restrict__ outq,
                                                                       const float* __restrict__ qscale) {
    static_assert(RG == 1 || RG == 2 || RG == 4 || RG == 8, "1, 2, 4 or 8 row groups");
    griddep_wait();
    constexpr int NW = FIX_THREADS / 32 / RG;      // warps per row group
    constexpr int GK = NW * FIX_KPS * FIX_UNROLL;  // keys per load group of a row group
    __shared__ double red_all[RG][NW][1 + FIX_MAXC];
    __shared__ int next_row_all[RG];
    const int grp = static_cast<int>(threadIdx.x) / (32 * NW);
    const int tid = static_cast<int>(threadIdx.x) - grp * 32 * NW, lane = tid & 31, wid = tid >> 5;
    auto red = red_all[grp];
    int& next_row = next_row_all[grp];
    // the row group's barrier (named barrier 1 + grp; the whole CTA for one group)
    auto gsync = [&]() {
        if (RG == 1)
            __syncthreads();
        else
            named_bar_sync(1 + grp, 32 * NW);
    };
    constexpr int DPL = HD / FIX_LPK;  // dimensions per lane
    const int sub = lane & (FIX_LPK - 1), kq = lane / FIX_LPK;  // dimensions [DPL sub, DPL sub + DPL) of key slot kq
    const int n = min(*reinterpret_cast<const volatile int*>(fix_n), cap);
    const int64_t rs = 3LL * d;
    const InvScale qs = make_inv_scale(static_cast<double>(__ldg(qscale)));
    // rows are taken from a counter (fix_n[1]) as CTAs become free: their key
    // counts range from 1 to the sequence length
    while (true) {
        gsync();  // next_row and red[] are free
        if (tid == 0) next_row = atomicAdd(fix_n + 1, 1);
        gsync();
        const int ri = next_row;
        if (ri >= n) break;
        const int4 rw = rows[ri];
        const uint2 mk = masks[ri];
        const int q = rw.x, head = rw.z, s0 = rw.w;
        const double off = static_cast<double>(__int_as_float(rw.y)) * 0.69314718055994531;  // base 2 -> natural
        const float* base = qkv + head * HD;
        double qv[DPL];
        {
            const float4* qr = reinterpret_cast<const float4*>(base + static_cast<int64_t>(q) * rs + DPL * sub);
#pragma unroll
            for (int t = 0; t < DPL / 4; t++) {
                const float4 a = __ldg(qr + t);
                qv[4 * t] = a.x;
                qv[4 * t + 1] = a.y;
                qv[4 * t + 2] = a.z;
                qv[4 * t + 3] = a.w;
            }
        }
        uint32_t m0 = mk.x, m1 = mk.y;
        while (m0 | m1) {  // block-uniform: passes of up to FIX_MAXC undecided columns
            int col[FIX_MAXC], nc = 0;
#pragma unroll
            for (int t = 0; t < FIX_MAXC; t++) {
                col[t] = 0;
                if (m0) {
                    col[t] = __ffs(m0) - 1;
                    m0 &= m0 - 1u;
                    nc = t + 1;
                } else if (m1) {
                    col[t] = 32 + __ffs(m1) - 1;
                    m1 &= m1 - 1u;
                    nc = t + 1;
                }
            }
            double l = 0.0, acc[FIX_MAXC];
#pragma unroll
            for (int t = 0; t < FIX_MAXC; t++) acc[t] = 0.0;
            // group g, step u of this warp: keys s0 + g GK + (u NW + wid) FIX_KPS + kq
            struct Group {
                float4 k[FIX_UNROLL][DPL / 4];
                float v[FIX_UNROLL][FIX_MAXC];
            };
            auto key_of = [&](int g, int u) { return s0 + g * GK + (u * NW + wid) * FIX_KPS + kq; };
            auto load = [&](int g, Group& G) {
#pragma unroll
                for (int u = 0; u < FIX_UNROLL; u++) {
                    const int j = key_of(g, u);
#pragma unroll
                    for (int t = 0; t < DPL / 4; t++) G.k[u][t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
                    for (int t = 0; t < FIX_MAXC; t++) G.v[u][t] = 0.0f;
                    if (j <= q) {
                        const float* kj = base + static_cast<int64_t>(j) * rs;
                        const float4* kp = reinterpret_cast<const float4*>(kj + d + DPL * sub);
#pragma unroll
                        for (int t = 0; t < DPL / 4; t++) G.k[u][t] = __ldg(kp + t);
                        if (sub == 0) {
#pragma unroll
                            for (int t = 0; t < FIX_MAXC; t++)
                                if (t < nc) G.v[u][t] = __ldg(kj + 2 * d + col[t]);
                        }
                    }
                }
            };
            auto score = [&](int g, const Group& G) {
#pragma unroll
                for (int u = 0; u < FIX_UNROLL; u++) {
                    double p0 = 0.0, p1 = 0.0;
#pragma unroll
                    for (int t = 0; t < DPL / 4; t++) {
                        p0 = fma(qv[4 * t], static_cast<double>(G.k[u][t].x), p0);
                        p1 = fma(qv[4 * t + 1], static_cast<double>(G.k[u][t].y), p1);
                        p0 = fma(qv[4 * t + 2], static_cast<double>(G.k[u][t].z), p0);
                        p1 = fma(qv[4 * t + 3], static_cast<double>(G.k[u][t].w), p1);
                    }
                    double sdot = p0 + p1;
#pragma unroll
                    for (int o = 1; o < FIX_LPK; o <<= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, o);
                    if (key_of(g, u) <= q && sub == 0) {
                        const double e = exp(sdot * 0.125 - off);  // 1/sqrt(64)
                        l += e;
#pragma unroll
                        for (int t = 0; t < FIX_MAXC; t++) acc[t] = fma(e, static_cast<double>(G.v[u][t]), acc[t]);
                    }
                }
            };
            // two groups in flight: the next group's loads are issued before
            // this group is scored (the loop is unrolled twice so that both
            // register buffers stay statically indexed)
            const int ng = (q - s0) / GK + 1;  // groups holding keys [s0, q]
            Group G0, G1;
            load(0, G0);
            for (int g = 0; g < ng; g += 2) {
                if (g + 1 < ng) load(g + 1, G1);
                score(g, G0);
                if (g + 1 >= ng) break;
                if (g + 2 < ng) load(g + 2, G0);
                score(g + 1, G1);
            }
            // the block's sums (lanes other than sub == 0 hold zeros)
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                l += __shfl_xor_sync(0xffffffffu, l, o);
#pragma unroll
                for (int t = 0; t < FIX_MAXC; t++) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
            }
            gsync();  // red[] is free
            if (lane == 0) {
                red[wid][0] = l;
#pragma unroll
                for (int t = 0; t < FIX_MAXC; t++) red[wid][1 + t] = acc[t];
            }
            gsync();
            if (tid < nc) {
                double lt = 0.0, at = 0.0;
#pragma unroll
                for (int w = 0; w < NW; w++) {
                    lt += red[w][0];
                    at += red[w][1 + tid];
                }
                const float cx = __double2float_rn(at * (1.0 / lt));
                const int64_t o = static_cast<int64_t>(q) * d + head * HD + col[tid];
                if (out) out[o] = cx;
                outq[o] = quant_exact(cx, qs);
            }
        }
    }
    // the last CTA to finish resets the list for the next launch
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(fix_n + 2, 1) == static_cast<int>(gridDim.x) - 1) {
            fix_n[0] = 0;
            fix_n[1] = 0;
            fix_n[2] = 0;
        }
    }
}

// Per-head bounds of a c_attn layer's Q, K and V outputs for the epilogue's
// fp16 split (kv_head_exp): block (h, part) over the 64 output columns n of
// head h in part (0 Q, 1 K, 2 V): A = max sw[n] * 127 * sum_k |W[n,k]|, B =
// max |bias[n]|, both rounded up.  out [6 heads]: A_Q, B_Q, A_K, B_K, A_V, B_V.
__global__ void kv_head_bound_kernel(const int8_t* __restrict__ W, const float* __restrict__ sw,
                                     const float* __restrict__ bias, int k, int kvd, float* __restrict__ out) {
    const int h = blockIdx.x, part = blockIdx.y, heads = gridDim.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float ra[8], rb[8];
    float a = 0.0f, bb = 0.0f;
    for (int i = warp; i < HD; i += blockDim.x >> 5) {
        const int n = part * kvd + h * HD + i;
        int sum = 0;
        for (int c = lane; c < k; c += 32) sum += abs(static_cast<int>(W[static_cast<int64_t>(n) * k + c]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        a = fmaxf(a, __fmul_ru(__fmul_ru(fabsf(sw[n]), 127.0f), __int2float_ru(sum)));
        if (bias) bb = fmaxf(bb, fabsf(bias[n]));
    }
    if (lane == 0) {
        ra[warp] = a;
        rb[warp] = bb;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x >> 5); w++) {
            a = fmaxf(a, ra[w]);
            bb = fmaxf(bb, rb[w]);
        }
        out[(2 * part) * heads + h] = a;
        out[(2 * part + 1) * heads + h] = bb;
    }
}

}  // namespace

int attention_tc_rows() { return TQ; }

int attention_tc_pitch(int T) { return (T + 7) & ~7; }

int launch_split_kv(const float* qkv, int T, int d, void* qh, void* ql, void* kh, void* kl, void* vth, void* vtl,
                    int* kv_exp, uint32_t* amax, cudaStream_t st, uint32_t* vcol) {
    if (T <= 0) return TVQ_OK;
    TVQ_CHECK(d % HD == 0, TVQ_ERR_UNSUPPORTED, "d must be a multiple of 64");
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    const int heads = d / HD;
    TVQ_CUDA(cudaMemsetAsync(amax, 0, sizeof(uint32_t) * 3 * heads, st));
    int r = launch_pdl(kv_head_amax_kernel, dim3(std::min(T, 64), 3, heads), dim3(64), 0, st, qkv, T, d, amax);
    if (!r && vcol) {
        TVQ_CUDA(cudaMemsetAsync(vcol, 0, sizeof(uint32_t) * d, st));
        r = launch_pdl(v_col_amax_kernel, dim3(heads, std::min(T, 64)), dim3(HD), 0, st, qkv, T, d, vcol);
    }
    if (!r) r = launch_pdl(kv_exp_from_amax_kernel, dim3((3 * heads + 127) / 128), dim3(128), 0, st,
                           static_cast<const uint32_t*>(amax), 3 * heads, kv_exp);
    if (r) return r;
    const int64_t n = static_cast<int64_t>(T) * (d / 4);
    const int grid = static_cast<int>(std::min<int64_t>((n + 255) / 256, ds->sm_count * 8));
    for (int part = 0; part < 2 && !r; part++)
        r = launch_pdl(split_qk16_kernel, dim3(grid), dim3(256), 0, st, qkv, T, d, part,
                       static_cast<const int*>(kv_exp), static_cast<uint2*>(part ? kh : qh),
                       static_cast<uint2*>(part ? kl : ql));
    if (r) return r;
    const int Tp = attention_tc_pitch(T);
    return launch_pdl(split_vt16_kernel, dim3((Tp + 31) / 32, d / 32), dim3(32, 8), 0, st, qkv, T, Tp, d,
                      static_cast<const int*>(kv_exp), static_cast<__half*>(vth), static_cast<__half*>(vtl));
}

int launch_kv_head_bound(const int8_t* W, const float* sw, const float* bias, int k, int kvd, float* out,
                         cudaStream_t st) {
    TVQ_CHECK(kvd % HD == 0 && kvd > 0 && k > 0, TVQ_ERR_UNSUPPORTED, "d must be a multiple of 64");
    kv_head_bound_kernel<<<dim3(kvd / HD, 3), 256, 0, st>>>(W, sw, bias, k, kvd, out);
    TVQ_CUDA(cudaGetLastError());
    return TVQ_OK;
}

int launch_attention_tc(const float* qkv, const void* qh, const void* ql, const void* kh, const void* kl,
                        const void* vth, const void* vtl, const int* kv_exp, int T, const int4* tiles, const int4* split, int nitems, const int4* comb,
                        int ncomb, int d, int nheads, float* out, int8_t* outq, const float* qscale, uint32_t* amax,
                        float* part_o, float2* part_ml, int* counters, cudaStream_t st, const AttnFix* fix) {
    if (nitems <= 0) return TVQ_OK;
    TVQ_CHECK(nheads > 0 && d == nheads * HD, TVQ_ERR_UNSUPPORTED, "the tensor-core attention needs head dim 64");
    TVQ_CHECK(split && qh && ql && kh && kl && vth && vtl && kv_exp, TVQ_ERR_INVALID,
              "the tensor-core attention needs key ranges, split K / V^T and their head scales");
    TVQ_CHECK((reinterpret_cast<uintptr_t>(qkv) & 15) == 0 && (!out || (reinterpret_cast<uintptr_t>(out) & 15) == 0) &&
                  (!outq || (reinterpret_cast<uintptr_t>(outq) & 3) == 0),
              TVQ_ERR_UNSUPPORTED, "attention buffers must be 16-byte aligned");
    int rc = 0;
    DeviceState* ds = device_state(&rc);
    if (!ds) return rc;
    TVQ_CHECK(ds->cc_major == 10, TVQ_ERR_UNSUPPORTED, "the tcgen05 attention needs an sm_100 device");
    static bool attr[64] = {false};
    int dev = 0;
    TVQ_CUDA(cudaGetDevice(&dev));
    if (dev < 64 && !attr[dev]) {
        TVQ_CUDA(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(SMEM_BYTES)));
        attr[dev] = true;
    }
    CUtensorMap mqh, mql, mkh, mkl, mvh, mvl;
    rc = make_tma_f16_sw128(&mqh, qh, T, d, TQ);
    if (!rc) rc = make_tma_f16_sw128(&mql, ql, T, d, TQ);
    if (!rc) rc = make_tma_f16_sw128(&mkh, kh, T, d, TK);
    if (!rc) rc = make_tma_f16_sw128(&mkl, kl, T, d, TK);
    if (!rc) rc = make_tma_f16_sw128(&mvh, vth, d, T, HD, attention_tc_pitch(T));
    if (!rc) rc = make_tma_f16_sw128(&mvl, vtl, d, T, HD, attention_tc_pitch(T));
    if (rc) return rc;
    AttnParams p;
    p.qkv = qkv;
    p.tiles = tiles;
    p.split = split;
    p.d = d;
    p.nheads = nheads;
    p.scale2 = static_cast<float>(1.4426950408889634 / 8.0);  // log2(e) / sqrt(64)
    p.out = out;
    p.outq = outq;
    p.qscale = qscale;
    p.amax = amax;
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.err = ds->d_error;
    TVQ_CHECK(ncomb == 0 || (comb && counters), TVQ_ERR_INVALID, "key-chunk items need merge entries and counters");
    p.comb = comb;
    p.counters = counters;
    p.kv_exp = kv_exp;
    p.nunits = nitems * nheads;
    const bool fixing = fix && outq;
    TVQ_CHECK(!fixing || (fix->vmax && fix->list && fix->mask && fix->n && fix->cap > 0),
              TVQ_ERR_INVALID, "the exact int8 context needs the head maxima and the fix-up lists");
    p.vmax = fixing ? fix->vmax : nullptr;
    p.fix = fixing ? fix->list : nullptr;
    p.fix_mask = fixing ? fix->mask : nullptr;
    p.fix_n = fixing ? fix->n : nullptr;
    p.fix_cap = fixing ? fix->cap : 0;
    // persistent: one CTA per SM (all of TMEM) working through the units;
    // key-chunk partials are merged inside the kernel by the last CTA of each set
    const int grid = std::min(p.nunits, ds->sm_count);
    rc = launch_pdl(attention_tc_kernel, dim3(grid), dim3(NTHREADS), SMEM_BYTES, st, mqh, mql, mkh, mkl, mvh, mvl, p);
    if (rc || !fixing) return rc;
    // the listed rows' undecided columns (the list length is known on the
    // device only: a persistent grid of a few CTAs per SM)
    // row groups per CTA from the layout (the list length itself is known on
    // the device only): about 1-2 % of the (token, head) rows are listed, so
    // a layout of at least 1024 (token, head) rows per SM splits the CTA
    const int64_t row_heads = static_cast<int64_t>(T) * nheads;
    static const int env_rg = [] {  // TVQ_FIX_GROUPS=1|2|4|8 pins the row groups (tuning)
        const char* e = getenv("TVQ_FIX_GROUPS");
        const int v = e ? atoi(e) : 0;
        return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 0;
    }();
    // (measured at config 4, 131072 packed tokens x 12 heads, attention
    // stage per step: 26.0 / 24.5 / 24.0 ms with 2 / 4 / 8 row groups)
    const int rg = env_rg ? env_rg : row_heads >= 1024LL * ds->sm_count ? 8 : 1;
    auto kern = rg == 8   ? attention_fix_kernel<8>
                : rg == 4 ? attention_fix_kernel<4>
                : rg == 2 ? attention_fix_kernel<2>
                          : attention_fix_kernel<1>;
    return launch_pdl(kern, dim3(ds->sm_count), dim3(FIX_THREADS), 0, st, qkv,
                      static_cast<const int4*>(fix->list), static_cast<const uint2*>(fix->mask), fix->n, fix->cap, d,
                      out, outq, qscale);
}

}  // namespace tvq
