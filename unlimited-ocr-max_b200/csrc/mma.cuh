// Warp-level tensor-core products for the decode GEMVs (a handful of tokens against streamed
// weight rows): mma.sync m16n8k32 s8 for int8 weights and m16n8k16 bf16 for bf16 weights,
// operands taken from registers. The weights are the A operand (16 rows), the <= 8 tokens the B
// operand (8 columns). The products are HBM-bound; the tensor cores only replace the CUDA-core
// unpack and multiply-add work.
//
// Exact activations. fp32 activations are given to the s8 product as three int8 digits per
// value with a power-of-two scale per token: v = sigma * (d0 + d1 / 128 + d2 / 128^2), |d| <= 64,
// accumulated in int32 (exact) and recombined in fp32 after each 128-group, before the group's
// weight scale; the representation error is below 2^-21 of the token's largest value.
// To the bf16 product they are given as three bf16 terms v = t0 + t1 + t2 (t0 = bf16(v),
// t1 = bf16(v - t0), t2 = bf16(v - t0 - t1)), exact to ~2^-24.
//
// K order. A k-step is 32 bytes of a weight row: 32 int8 or 16 bf16 values. The mma fragments
// hold, for lane (g = lane / 4, t = lane % 4), row g and row g + 8 at logical k positions
// {4t..4t+3, 4t+16..4t+19} (s8) or {2t, 2t+1, 2t+8, 2t+9} (bf16); both operands use the same
// permutation of k, logical -> physical {8t..8t+7} bytes of the k-step, so every lane loads one
// contiguous 8-byte piece of each row (and of each token's activations).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace uocr {

// Not volatile: the compiler may interleave the products with the loads that feed them.
UOCR_DEV void mma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

UOCR_DEV void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Shared-memory loads the compiler may schedule freely (no volatile, no memory clobber). Only
// for data that cannot change while they may run: the caller derives `a` from launder() after
// the wait that published the data, and keeps the data alive until fence_regs() has consumed
// every result (see the decode kernels).
UOCR_DEV uint2 lds_u64_nv(uint32_t a) {
    uint2 v;
    asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
UOCR_DEV float lds_f32_nv(uint32_t a) {
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
// An opaque copy of `a`, ordered after every earlier volatile asm (e.g. a barrier wait): loads
// from addresses derived from it cannot move above that point.
UOCR_DEV uint32_t launder(uint32_t a) {
    asm volatile("mov.b32 %0, %0;" : "+r"(a));
    return a;
}
// Forces v to be computed before any later volatile asm (e.g. releasing the data behind it).
UOCR_DEV void fence_regs(const float (&v)[4]) {
    asm volatile("" ::"f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]));
}

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

// Three int8 digits of v / sigma (inv = 1 / sigma), packed as bytes of d0, d1, d2.
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

// int32 digit accumulators of one group -> fp32 value of sum(w * v) / sigma.
UOCR_DEV float undigit(int c0, int c1, int c2) {
    return __fmaf_rn((float)c2, 1.0f / 16384.0f, __fmaf_rn((float)c1, 1.0f / 128.0f, (float)c0));
}

// Three bf16 terms of (v0, v1) packed as bf16x2 (v0 in the low half).
UOCR_DEV void bf16_terms(float v0, float v1, uint32_t& t0, uint32_t& t1, uint32_t& t2) {
    __nv_bfloat162 a = __floats2bfloat162_rn(v0, v1);
    const float r0 = v0 - __low2float(a), r1 = v1 - __high2float(a);
    __nv_bfloat162 b = __floats2bfloat162_rn(r0, r1);
    const float s0 = r0 - __low2float(b), s1 = r1 - __high2float(b);
    __nv_bfloat162 c = __floats2bfloat162_rn(s0, s1);
    t0 = *reinterpret_cast<uint32_t*>(&a);
    t1 = *reinterpret_cast<uint32_t*>(&b);
    t2 = *reinterpret_cast<uint32_t*>(&c);
}

}  // namespace uocr
