// tvq_e4m3.h -- the reference's E4M3 encoder (native_fp8_e4m3_encode =
// _qt_fp8_encode(x, 7, 3, 15, 0, 126), tv/quantization/types.tkv:154-191,
// 228-230, through f64_to_f32_bits, tv/runtime/f32_bits.tkv:6-57) in two
// forms that give the same byte for every binary32 bit pattern:
//
//   e4m3_encode_ref   the reference's steps one by one (int64 arithmetic,
//                     _qt_rne_rshift of types.tkv:71-93)
//   e4m3_encode_fast  the same function in 32-bit integer operations, the
//                     form the kernels use
//
// Plain C++ (host and device), so that a CPU test compiles this header with
// g++ and compares the two forms over all 2^32 inputs.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define TVQ_E4M3_HD __host__ __device__ __forceinline__
#else
#define TVQ_E4M3_HD inline
#endif

namespace tvq {

// Binary32 pattern as tv/runtime/f32_bits.tkv:6-57 produces it for an f32
// input: the IEEE pattern, except -0.0 -> 0, +/-2^-149 -> +/-0 (its
// `sh <= 0` test), NaN -> quiet NaN (that loop cannot finish on NaN/Inf).
TVQ_E4M3_HD uint32_t ref_f32_bits(uint32_t b) {
    if ((b & 0x7FFFFFFFu) == 0u) return 0u;
    if ((b & 0x7F800000u) == 0x7F800000u) return (b & 0x007FFFFFu) ? 0x7FC00000u : b;
    if ((b & 0x7FFFFFFFu) == 1u) return b & 0x80000000u;
    return b;
}

// _qt_rne_rshift, tv/quantization/types.tkv:71-93
TVQ_E4M3_HD int64_t rne_rshift(int64_t v, int64_t s) {
    if (s > 40) return 0;
    if (s <= 0) return v;
    const int64_t half = static_cast<int64_t>(1) << (s - 1);
    const int64_t q = v >> s;
    const int64_t rem = v - (q << s);
    if (rem > half) return q + 1;
    if (rem < half) return q;
    return (q & 1) ? q + 1 : q;
}

TVQ_E4M3_HD uint8_t e4m3_encode_ref(uint32_t xbits) {
    const uint32_t b = ref_f32_bits(xbits);
    const uint32_t sign = b >> 31;
    const int64_t ex = (b >> 23) & 255;
    const int64_t man = b & 8388607;
    if (ex == 255) return static_cast<uint8_t>((sign << 7) | 127u);
    int64_t e, full;
    if (ex == 0) { e = -126; full = man; } else { e = ex - 127; full = man | 8388608; }
    int64_t e8 = e + 7;
    if (e8 >= 15) return static_cast<uint8_t>((sign << 7) | 126u);
    if (e8 <= 0) {
        int64_t m = rne_rshift(full, 24 - 3 - e8);
        if (m > 7) m = 7;
        return static_cast<uint8_t>((sign << 7) | static_cast<uint32_t>(m));
    }
    int64_t r = rne_rshift(full, 23 - 3);
    if (r >= 16) {
        r = 8;
        e8 = e8 + 1;
        if (e8 >= 15) return static_cast<uint8_t>((sign << 7) | 126u);
    }
    return static_cast<uint8_t>((sign << 7) | static_cast<uint32_t>(e8 << 3) | static_cast<uint32_t>(r - 8));
}

// v >> s rounded half to even, for v < 2^24 and 1 <= s <= 24.
TVQ_E4M3_HD uint32_t rne_rshift32(uint32_t v, uint32_t s) {
    const uint32_t q = v >> s;
    const uint32_t rem = v & ((1u << s) - 1u);
    const uint32_t half = 1u << (s - 1u);
    return q + static_cast<uint32_t>((rem > half) | ((rem == half) & (q & 1u)));
}

// The same mapping, case by case on the biased binary32 exponent ex:
//   |x| = 0                 -> 0 (also -0)
//   ex = 255                -> 0x7F for NaN (its sign is dropped), sign|0x7F for Inf
//   ex >= 135 (|x| >= 256)  -> sign|126 (448)
//   ex <= 116 (|x| < 2^-10) -> sign|0 (the subnormal shift exceeds 24 bits)
//   117 <= ex <= 120        -> E4M3 subnormal m = rne(full, 141 - ex), at most 7
//   121 <= ex <= 134        -> ((ex - 121) << 3) + rne(full, 20); a mantissa
//                              carry moves into the exponent field by itself,
//                              and a code of 120 or more (exponent 15) is 126
// Every case is computed and the result selected, so the lanes of a warp
// holding values of different magnitudes do not diverge.
TVQ_E4M3_HD uint8_t e4m3_encode_fast(uint32_t xbits) {
    const uint32_t a = xbits & 0x7FFFFFFFu;
    const uint32_t s = (xbits >> 24) & 0x80u;
    const uint32_t ex = a >> 23;
    const uint32_t full = (a & 0x007FFFFFu) | 0x00800000u;
    const bool sub = ex <= 120u;
    uint32_t sh = sub ? 141u - ex : 20u;  // 20 .. 141
    sh = sh > 24u ? 24u : sh;             // the cases with a longer shift are replaced below
    const uint32_t r = rne_rshift32(full, sh);
    const uint32_t norm = ((ex - 121u) << 3) + r;  // wraps for ex < 121: replaced below
    uint32_t code = sub ? (r > 7u ? 7u : r) : (norm >= 120u ? 126u : norm);
    code = ex >= 135u ? 126u : code;
    code = ex <= 116u ? 0u : code;
    uint32_t out = s | code;
    out = a == 0u ? 0u : out;
    out = ex == 255u ? ((a & 0x007FFFFFu) ? 0x7Fu : (s | 0x7Fu)) : out;
    return static_cast<uint8_t>(out);
}

}  // namespace tvq
