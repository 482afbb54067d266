// Exact int8 digits of fp32 activations for the int8 tensor-core products (decode.cu): a value v
// of a group whose largest magnitude is m is written as v = sigma * (d0 + d1 / 128 + d2 / 128^2)
// with sigma = 2^(floor(log2 m) - 5) and |d| <= 64; the int32 sums of the three digit planes
// are recombined in fp32 (undigit) before the group's scales apply. The representation error is
// below 2^-21 of m.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace uocr {

// Power-of-two scale for a group whose largest magnitude is m: sigma = 2^(floor(log2 m) - 5),
// so |v| / sigma < 64. Returns sigma (1 for an all-zero or denormal group) and its inverse.
UOCR_DEV void digit_scale(float m, float& sigma, float& inv) {
    const int e = (int)((__float_as_uint(m) >> 23) & 0xFF);  // biased exponent
    if (e < 32) {  // zero or tiny: digits are all zero
        sigma = 1.0f;
        inv = 1.0f;
        return;
    }
    sigma = __uint_as_float((uint32_t)(e - 5) << 23);
    inv = __uint_as_float((uint32_t)(254 - (e - 5)) << 23);
}

// Three int8 digits of v / sigma (inv = 1 / sigma).
UOCR_DEV void to_digits(float v, float inv, int& d0, int& d1, int& d2) {
    const float r0 = v * inv;
    const float q0 = rintf(r0);
    const float r1 = (r0 - q0) * 128.0f;
    const float q1 = rintf(r1);
    const float r2 = (r1 - q1) * 128.0f;
    d0 = (int)q0;
    d1 = (int)q1;
    d2 = (int)rintf(r2);
}

UOCR_DEV uint32_t pack_s8x4(int a, int b, int c, int d) {
    return (uint32_t)(a & 0xFF) | ((uint32_t)(b & 0xFF) << 8) | ((uint32_t)(c & 0xFF) << 16) | ((uint32_t)d << 24);
}

// int32 sums of the three digit planes of one group -> fp32 value of sum(w * v) / sigma.
UOCR_DEV float undigit(int c0, int c1, int c2) {
    return __fmaf_rn((float)c2, 1.0f / 16384.0f, __fmaf_rn((float)c1, 1.0f / 128.0f, (float)c0));
}

}  // namespace uocr
