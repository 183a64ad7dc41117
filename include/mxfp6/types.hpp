#pragma once
// Number formats of MXFP6 (host side): FP6 E2M3 element codes, E8M0 block scales and the dense
// 6-bit packing. Same function names and results as the reference's codecs
// (reference: include/mxfp6/types.hpp:13-123); written here from the format definitions.
//
//   FP6 E2M3: bit 5 sign, bits 4..3 exponent (bias 1), bits 2..0 mantissa; no Inf/NaN.
//             exponent 0 is subnormal: value = m/8. Largest magnitude 7.5, smallest 0.125.
//   E8M0:     value = 2^(code-127); code 255 is NaN.
//   Packing:  four 6-bit codes per three bytes, least significant bits first (code i occupies
//             bits 6i..6i+5 of the little-endian 24-bit group). The B200 tensor-memory
//             accelerator's 16U6 unpack mode reads this order as 16-code / 12-byte groups.
#include <cassert>
#include <cmath>
#include <cstdint>

namespace mxfp6 {

// ---- FP6 E2M3 -----------------------------------------------------------------------------

inline float fp6_e2m3_to_float(uint8_t bits6) {
    const int exp_field = (bits6 >> 3) & 3;
    const int man_field = bits6 & 7;
    // Subnormal: m/8. Normal: (1 + m/8) * 2^(e-1) == (8 + m) * 2^(e-4).
    float mag = exp_field == 0 ? (float)man_field * 0.125f
                               : std::ldexp((float)(8 + man_field), exp_field - 4);
    return (bits6 & 0x20) ? -mag : mag;
}

namespace detail {
// Round a non-negative, exactly representable q to the nearest integer, ties to even.
inline int round_half_even_nonneg(float q) {
    float fl = std::floor(q);
    float diff = q - fl;
    int base = (int)fl;
    if (diff > 0.5f) return base + 1;
    if (diff < 0.5f) return base;
    return (base & 1) ? base + 1 : base;
}
}  // namespace detail

// Nearest E2M3 code, ties to even, magnitudes above 7.5 saturate to 7.5. A negative input that
// rounds to zero keeps its sign bit (code 0x20); -0.0 gives +0. NaN gives code 0x18 (4.0),
// which is what the reference's conversion produces on x86-64 (its (int) cast of NaN yields
// INT_MIN, whose low byte is 0, in the top binade).
inline uint8_t float_to_fp6_e2m3(float v) {
    uint8_t sign = 0;
    if (v < 0.0f) {
        sign = 0x20;
        v = -v;
    }
    if (v == 0.0f) return sign;
    if (std::isnan(v)) return 0x18;
    if (v > 7.5f) v = 7.5f;
    if (v < 1.0f) {  // subnormal binade, grid step 1/8
        int m = detail::round_half_even_nonneg(v * 8.0f);
        if (m <= 0) return sign;
        if (m >= 8) return sign | 0x08;  // rounds up to 1.0
        return sign | (uint8_t)m;
    }
    int e = v < 2.0f ? 1 : (v < 4.0f ? 2 : 3);
    float frac = v / (float)(1 << (e - 1)) - 1.0f;  // in [0,1), exact
    int m = detail::round_half_even_nonneg(frac * 8.0f);
    if (m >= 8) {  // mantissa overflow: next binade
        m = 0;
        e += 1;
        if (e > 3) return sign | 0x1F;
    }
    return sign | (uint8_t)(e << 3) | (uint8_t)m;
}

// ---- E8M0 ---------------------------------------------------------------------------------

inline float e8m0_to_float(uint8_t code) {
    if (code == 255) return NAN;
    return std::ldexp(1.0f, (int)code - 127);
}

// Nearest power of two in the log domain (midpoint sqrt(2)), codes clamped to [0,254];
// NaN -> 255, v <= 0 -> 0, +Inf -> 127 (frexp of Inf reports exponent 0 on glibc).
inline uint8_t float_to_e8m0(float v) {
    if (std::isnan(v)) return 255;
    if (v <= 0.0f) return 0;
    int e2;
    float m = std::frexp(v, &e2);  // v = m * 2^e2, m in [0.5, 1)
    int e = e2 - 1;                // v = (2m) * 2^e, 2m in [1, 2)
    if (m * 2.0f >= 1.41421356f) e += 1;
    int code = e + 127;
    return (uint8_t)(code < 0 ? 0 : (code > 254 ? 254 : code));
}

// ---- dense 6-bit packing --------------------------------------------------------------------

inline void pack_fp6x4(const uint8_t* in, uint8_t* out) {
    uint32_t g = (uint32_t)(in[0] & 0x3F) | ((uint32_t)(in[1] & 0x3F) << 6) |
                 ((uint32_t)(in[2] & 0x3F) << 12) | ((uint32_t)(in[3] & 0x3F) << 18);
    out[0] = (uint8_t)g;
    out[1] = (uint8_t)(g >> 8);
    out[2] = (uint8_t)(g >> 16);
}

inline void unpack_fp6x4(const uint8_t* in, uint8_t* out) {
    uint32_t g = (uint32_t)in[0] | ((uint32_t)in[1] << 8) | ((uint32_t)in[2] << 16);
    for (int i = 0; i < 4; i++) out[i] = (uint8_t)((g >> (6 * i)) & 0x3F);
}

inline void pack_fp6(const uint8_t* vals, int n, uint8_t* packed) {
    assert(n % 4 == 0);
    for (int i = 0; i < n / 4; i++) pack_fp6x4(vals + 4 * i, packed + 3 * i);
}

inline void unpack_fp6(const uint8_t* packed, int n, uint8_t* vals) {
    assert(n % 4 == 0);
    for (int i = 0; i < n / 4; i++) unpack_fp6x4(packed + 3 * i, vals + 4 * i);
}

inline int fp6_packed_bytes(int n) {
    assert(n % 4 == 0);
    return n / 4 * 3;
}

}  // namespace mxfp6
