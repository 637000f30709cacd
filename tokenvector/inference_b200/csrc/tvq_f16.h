// tvq_f16.h -- the reference's FP16 encoder (native_f16_encode,
// tv/quantization/types.tkv:95-127, behind fp16_from_float :256-257 and
// quantize_fp16, tv/quantization/matmul.tkv:106-114), through the same
// f64_to_f32_bits front end as the E4M3 encoder, in two forms that give the
// same 16-bit pattern for every binary32 input:
//
//   f16_encode_ref   the reference's steps one by one (int64 arithmetic)
//   f16_encode_fast  the same function in 32-bit integer operations (the
//                    form the quantize kernel runs)
//
// Where it departs from IEEE round-to-nearest (__float2half_rn): a value
// that rounds up out of the subnormal range stays at the largest subnormal
// (0x03FF) instead of becoming 2^-14; every NaN becomes the quiet NaN 0x7E00
// (the front end drops the sign and payload); -0.0 and +-2^-149 encode as +0.
//
// Plain C++ (host and device), so that a CPU test compiles this header with
// g++ and compares the two forms over all 2^32 inputs.
#pragma once
#include "tvq_e4m3.h"

namespace tvq {

TVQ_E4M3_HD uint16_t f16_encode_ref(uint32_t xbits) {
    const uint32_t b = ref_f32_bits(xbits);
    const int64_t sign = (b >> 31) & 1, ex = (b >> 23) & 255, man = b & 8388607;
    if (ex == 255) return static_cast<uint16_t>((sign << 15) | 31744 | (man != 0 ? 512 : 0));
    int64_t e, full;
    if (ex == 0) {
        e = -126;
        full = man;
    } else {
        e = ex - 127;
        full = man | 8388608;
    }
    int64_t e16 = e + 15;
    if (e16 >= 31) return static_cast<uint16_t>((sign << 15) | 31744);
    if (e16 <= 0) {
        int64_t m = rne_rshift(full, 24 - 10 - e16);
        if (m > 1023) m = 1023;
        return static_cast<uint16_t>((sign << 15) | m);
    }
    int64_t r = rne_rshift(full, 23 - 10);
    if (r >= 2048) {
        r = 1024;
        e16 = e16 + 1;
        if (e16 >= 31) return static_cast<uint16_t>((sign << 15) | 31744);
    }
    return static_cast<uint16_t>((sign << 15) | (e16 << 10) | (r - 1024));
}

// Case by case on the biased binary32 exponent ex (after the front end):
//   ex = 255               -> 0x7E00 (NaN; the front end made it positive) or sign|0x7C00
//   ex >= 143 (|x| >= 2^16) -> sign|0x7C00
//   ex <= 101              -> sign|0 (the subnormal shift, 14 - e16 >= 25,
//                             exceeds the 24-bit significand)
//   102 <= ex <= 112       -> subnormal m = rne(full, 126 - ex), at most 1023
//   113 <= ex <= 142       -> ((ex - 112) << 10) + rne(full, 13) - 1024: a
//                             mantissa carry moves into the exponent field
//                             by itself, up to 0x7C00 (Inf) from ex = 142
TVQ_E4M3_HD uint16_t f16_encode_fast(uint32_t xbits) {
    const uint32_t b = ref_f32_bits(xbits);
    const uint32_t s = (b >> 16) & 0x8000u;
    const uint32_t ex = (b >> 23) & 255u;
    const uint32_t man = b & 0x7FFFFFu;
    if (ex == 255u) return static_cast<uint16_t>(s | 0x7C00u | (man ? 0x200u : 0u));
    if (ex >= 143u) return static_cast<uint16_t>(s | 0x7C00u);
    if (ex <= 101u) return static_cast<uint16_t>(s);
    const uint32_t full = ex ? (man | 0x800000u) : man;
    if (ex <= 112u) {
        const uint32_t m = rne_rshift32(full, 126u - ex);
        return static_cast<uint16_t>(s | (m > 1023u ? 1023u : m));
    }
    return static_cast<uint16_t>(s | (((ex - 112u) << 10) + rne_rshift32(full, 13u) - 1024u));
}

}  // namespace tvq
