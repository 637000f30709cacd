// tvq_exact.cuh -- the reference's binary64 expressions, evaluated exactly
// with binary32 arithmetic plus a rare binary64 slow path.
//
// FP64 on the CUDA cores runs at a small fraction of the FP32 rate on B200,
// so the per-element f64 arithmetic of the reference's numeric model cannot
// sit on the hot path.  Each helper below computes the exact real value of
// the expression as an unevaluated sum of two floats (error-free products
// via FMA, two-sum), rounds it once, and proves from an error bound that the
// result equals what the reference's chain of f64 roundings gives.  When the
// value lies too close to a rounding boundary for that proof (probability
// about 1e-6 per element) it falls back to the f64 expression itself.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace tvq {

// clamp(int(round(v)), -127, 127) of a binary64 value, .NET semantics.
__device__ __forceinline__ int8_t q8_f64(double v) {
    if (v != v) return 0;
    double r = rint(v);
    r = fmin(fmax(r, -127.0), 127.0);
    return static_cast<int8_t>(static_cast<int>(r));
}

// calibrate_minmax symmetric (tv/quantization/engine.tkv:24-30) from a
// recorded max|x| (f32 bit pattern): scale = fl32(max(amax, 1e-8) / 127).
__device__ __forceinline__ float scale_from_amax_bits(uint32_t amax_bits) {
    double am = static_cast<double>(__uint_as_float(amax_bits));
    if (am < 0.00000001) am = 0.00000001;
    return __double2float_rn(am / 127.0);
}

// 2^s as a float, exactly, for -126 <= s <= 127 (a multiply by it is the
// ldexpf of the product: one IEEE rounding, exact unless it under- or
// overflows).
__device__ __forceinline__ float exp2i(int s) { return __int_as_float((s + 127) << 23); }

// The exponent s with bound * 2^s in [2^14, 2^15): every |x| <= bound then
// has |x 2^s| < 2^15, inside the fp16 range with room for the rounding of
// an fp16 high part.  0 for a zero, infinite or NaN bound; at most 126 in
// magnitude.
__device__ __forceinline__ int pow2_exp_below_2p15(float bound) {
    if (!(bound > 0.0f) || !(bound <= 3.40282347e38f)) return 0;
    int e;
    frexpf(bound, &e);  // bound in [2^(e-1), 2^e)
    return max(-126, min(126, 15 - e));
}

// 1/scale of tv/quantization/engine.tkv:219-222 (and :244-246), kept as a
// binary64 value and as a float pair hi + lo (|hi + lo - inv| <= 2^-48 |inv|).
struct InvScale {
    double d;
    float hi, lo;
};

__device__ __forceinline__ InvScale make_inv_scale(double scale) {
    InvScale s;
    s.d = (scale > 0.00000001) ? 1.0 / scale : 1.0 / 0.00000001;
    if (scale != scale) s.d = scale;  // NaN scale -> NaN products -> 0, as 1.0/NaN
    s.hi = __double2float_rn(s.d);
    s.lo = __double2float_rn(s.d - static_cast<double>(s.hi));
    return s;
}

// The same pair built from an already computed binary64 1/scale.
__device__ __forceinline__ InvScale make_inv_from_inv(double inv) {
    InvScale s;
    s.d = inv;
    s.hi = __double2float_rn(inv);
    s.lo = __double2float_rn(inv - static_cast<double>(s.hi));
    return s;
}

// q = clamp(int(round(fl64(x * inv))), -127, 127) exactly.
// P = x*(hi+lo) is formed as ph + pl with |ph + pl - x*inv| <= 2^-46 |x*inv|.
// rint(fl64(x*inv)) equals the integer nearest ph + pl unless x*inv lies
// within that error (plus one f64 ulp) of a half-integer; |t| is the
// distance of ph + pl to the integer r = rint(ph), so a margin of 2^-20 on
// ||t| - 1/2| is ample for |x*inv| < 256.  Branch-free: returns false when
// the binary64 expression must decide (quant_slow).
__device__ __forceinline__ bool quant_fast(float x, const InvScale& s, int8_t& out) {
    const float ph = __fmul_rn(x, s.hi);
    const float pe = fmaf(x, s.hi, -ph);  // exact rounding error of ph
    const float pl = fmaf(x, s.lo, pe);
    const float r = rintf(ph);
    const float t = __fadd_rn(__fsub_rn(ph, r), pl);
    const float at = fabsf(t);
    float q = (at > 0.5f) ? r + copysignf(1.0f, t) : r;
    const bool big = !(fabsf(ph) < 256.0f);  // NaN, Inf, or certainly saturated
    q = big ? copysignf(127.0f, ph) : q;
    q = fminf(fmaxf(q, -127.0f), 127.0f);
    q = (ph != ph) ? 0.0f : q;
    out = static_cast<int8_t>(static_cast<int>(q));
    return big || !(fabsf(at - 0.5f) < 9.5367431640625e-07f);  // 2^-20
}

static __device__ __noinline__ int8_t quant_slow(float x, double inv) { return q8_f64(static_cast<double>(x) * inv); }

__device__ __forceinline__ int8_t quant_exact(float x, const InvScale& s) {
    int8_t q;
    if (!quant_fast(x, s, q)) q = quant_slow(x, s.d);
    return q;
}

// q = clamp(int(rint(fl64(x * inv))), -127, 127) from hi = fl32(inv) alone,
// as the low byte of a float.  t = fl32(x*hi + 1.5*2^23) is 1.5*2^23 plus
// the integer r nearest the exact product x*hi (|x*hi| < 2^22; ties to even,
// as 1.5*2^23 is even), r = t - 1.5*2^23 exactly, and d = fl32(x*hi - r)
// (|d| <= 1/2, error <= 2^-25).  x*inv differs from x*hi by at most
// 2^-24 |x*hi| plus one f64 ulp, under 2^-15.9 for |x*hi| < 256, so r is
// also the integer nearest fl64(x*inv) unless ||d| - 1/2| < 2^-15; from 256
// up both saturate.  t clamped to 1.5*2^23 +- 127 holds 2^22 + q in its
// mantissa, so its low byte is q as an int8.  Returns false for NaN,
// infinities and near-ties (quant_slow decides).
__device__ __forceinline__ bool quant_fast_t(float x, float hi, float& t) {
    constexpr float M = 12582912.0f;  // 1.5 * 2^23
    const float tt = fmaf(x, hi, M);
    const float d = fmaf(x, hi, -__fsub_rn(tt, M));
    t = fminf(fmaxf(tt, M - 127.0f), M + 127.0f);
    return fabsf(__fsub_rn(fabsf(d), 0.5f)) >= 3.0517578125e-05f;  // 2^-15; false for NaN
}

// Four quant_fast_t results as four int8 bytes, the first in the low byte.
__device__ __forceinline__ uint32_t pack_q4(float t0, float t1, float t2, float t3) {
    const uint32_t lo = __byte_perm(__float_as_uint(t0), __float_as_uint(t1), 0x0040);
    const uint32_t hi = __byte_perm(__float_as_uint(t2), __float_as_uint(t3), 0x0040);
    return __byte_perm(lo, hi, 0x5410);
}

// ulp of a normal float y (|y| >= 2^-100)
__device__ __forceinline__ float ulp_of(float y) {
    return __int_as_float((__float_as_int(fabsf(y)) & 0x7F800000) - (23 << 23));
}

// fl32(fl64(x * inv)) exactly: the scaled value that the FP8 quantizer hands
// to the encoder's f32 parameter.  x * (hi + lo) is formed as ph + pl within
// 2^-44 |x * inv| of the exact product; the f64 product differs from it by
// at most one f64 ulp, so y = fl32(ph + pl) is fl32(fl64(x * inv)) unless
// ph + pl lies within 2^-40 |ph| of a float midpoint (then, and for zero,
// tiny, huge and non-finite values, the f64 product decides).
static __device__ __noinline__ float mul_round_slow(float x, double inv) {
    return __double2float_rn(static_cast<double>(x) * inv);
}

__device__ __forceinline__ float mul_round_exact(float x, const InvScale& s) {
    const float ph = __fmul_rn(x, s.hi);
    const float pe = fmaf(x, s.hi, -ph);
    const float pl = fmaf(x, s.lo, pe);
    const float y = __fadd_rn(ph, pl);
    const float ay = fabsf(y);
    const float r = __fadd_rn(__fsub_rn(ph, y), pl);
    const float u = __int_as_float((__float_as_int(ay) & 0x7F800000) - (23 << 23));
    const bool pow2 = (__float_as_int(ay) & 0x007FFFFF) == 0;
    const float half = (pow2 && (r * y < 0.0f)) ? 0.25f * u : 0.5f * u;
    const bool ok = (ay >= 7.888609052210118e-31f) && (ay < 3.0e38f) &&
                    (__fsub_rn(half, fabsf(r)) > fmaf(fabsf(ph), 9.094947017729282e-13f, 1e-37f));
    return ok ? y : mul_round_slow(x, s.d);  // zero, tiny, huge, or near a midpoint
}

// An int32 as a binary64, exactly, without the conversion unit: the double
// with high word 0x43300000 and low word a + 2^31 (a with its sign bit
// flipped) is 2^52 + 2^31 + a, and subtracting 2^52 + 2^31 is exact.
__device__ __forceinline__ double i32_to_f64(uint32_t a) {
    return __hiloint2double(0x43300000, static_cast<int>(a ^ 0x80000000u)) - 4503601774854144.0;
}

// ---- pairs of floats in one 64-bit register for the f32x2 arithmetic of
// sm_100: two independent IEEE binary32 operations per instruction, with
// the rounding of the scalar forms (.rn unless named).
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
#define TVQ_F2_BINOP(name, instr)                                  \
    __device__ __forceinline__ uint64_t name(uint64_t a, uint64_t b) { \
        uint64_t r;                                                \
        asm(instr " %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));       \
        return r;                                                  \
    }
TVQ_F2_BINOP(f2_add, "add.rn.f32x2")
TVQ_F2_BINOP(f2_sub, "sub.rn.f32x2")
TVQ_F2_BINOP(f2_mul, "mul.rn.f32x2")
TVQ_F2_BINOP(f2_sub_rd, "sub.rm.f32x2")
TVQ_F2_BINOP(f2_add_ru, "add.rp.f32x2")
#undef TVQ_F2_BINOP
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t f2_abs(uint64_t a) { return a & 0x7FFFFFFF7FFFFFFFull; }
__device__ __forceinline__ uint64_t f2_neg(uint64_t a) { return a ^ 0x8000000080000000ull; }

// two_sum on two pairs at once: S = A + B rounded, E its exact error.
__device__ __forceinline__ void two_sum2(uint64_t A, uint64_t B, uint64_t& S, uint64_t& E) {
    S = f2_add(A, B);
    const uint64_t BB = f2_sub(S, A);
    E = f2_add(f2_sub(A, f2_sub(S, BB)), f2_sub(B, BB));
}

// Error-free sum of two floats.
__device__ __forceinline__ void two_sum(float a, float b, float& s, float& e) {
    s = __fadd_rn(a, b);
    const float bb = __fsub_rn(s, a);
    e = __fadd_rn(__fsub_rn(a, __fsub_rn(s, bb)), __fsub_rn(b, bb));
}

// (ah + al) + (bh + bl) as a normalised float pair.
__device__ __forceinline__ void df_add(float ah, float al, float bh, float bl, float& rh, float& rl) {
    float s, e;
    two_sum(ah, bh, s, e);
    e = __fadd_rn(e, __fadd_rn(al, bl));
    rh = __fadd_rn(s, e);
    rl = __fsub_rn(e, __fsub_rn(rh, s));
}

}  // namespace tvq
