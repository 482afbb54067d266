// Device helpers shared by every kernel of libuocr_moe.so (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define UOCR_DEV __device__ __forceinline__

namespace uocr {

// ---- status word (workspace) -------------------------------------------------------
// Device-side bounded waits never trap: they record a nonzero code here and return.
enum DeviceStatus : uint32_t {
    kStatusOk = 0,
    kStatusWaitTimeout = 1,  // a spin/mbarrier wait exceeded its iteration budget
    kStatusMisaligned = 2,   // a kernel's shared-memory window was not aligned as its operands need
    kStatusBadCount = 3,     // an exchanged row count above the receiving slot's capacity (expert-parallel)
};

UOCR_DEV void set_status(uint32_t* status, uint32_t code) {
    if (status) atomicCAS(status, 0u, code);
}

// ---- bf16 / int8 unpacking (exact) --------------------------------------------------
UOCR_DEV float bf16lo(uint32_t packed) { return __uint_as_float(packed << 16); }
UOCR_DEV float bf16hi(uint32_t packed) { return __uint_as_float(packed & 0xFFFF0000u); }
UOCR_DEV float bf16f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

// 8 bf16 (one 16-byte word) -> 8 fp32, element order preserved.
UOCR_DEV void unpack_bf16x8(const uint4& v, float (&f)[8]) {
    f[0] = bf16lo(v.x); f[1] = bf16hi(v.x);
    f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
    f[4] = bf16lo(v.z); f[5] = bf16hi(v.z);
    f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
}

// Signed int8 byte -> exact fp32 without I2F: (b ^ 0x80) is b + 128 in [0, 255];
// the fp32 with bits 0x4B000000 | u is 2^23 + u exactly; subtract 2^23 + 128.
UOCR_DEV float s8_byte_to_f32(uint32_t word_xor80, int byte) {
    uint32_t sel = 0x7650u | uint32_t(byte);  // bytes: [word.byte, 0x00, 0x00, 0x4B]
    uint32_t bits = __byte_perm(word_xor80, 0x4B000000u, sel);
    return __fsub_rn(__uint_as_float(bits), 8388736.0f);
}

// 8 int8 (two 32-bit words) -> 8 fp32, element order preserved.
UOCR_DEV void unpack_s8x8(uint32_t lo, uint32_t hi, float (&f)[8]) {
    lo ^= 0x80808080u;
    hi ^= 0x80808080u;
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = s8_byte_to_f32(lo, i);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[4 + i] = s8_byte_to_f32(hi, i);
}

UOCR_DEV uint16_t f32_to_bf16_rne(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return uint16_t((u >> 16) | 0x40u);  // NaN stays NaN
    u += 0x7FFFu + ((u >> 16) & 1u);
    return uint16_t(u >> 16);
}

UOCR_DEV int clamp_expert(int32_t e, int E) { return e < 0 ? 0 : (e >= E ? E - 1 : e); }

// ---- the softmax exponential --------------------------------------------------------
// Cody-Waite reduction x = n ln2 + r (ln 2 split in two constants derived from
// ln 2 = 0.6931471805599453...), a degree-7 Taylor polynomial of e^r (coefficients 1/k!)
// in Horner form with fused multiply-adds, and an exact scale by 2^n. Every operation is
// an explicit IEEE-rounded intrinsic, so the CPU oracle (oracle/moe_oracle.c:
// oracle_exp_f32) computes the same bits. Arguments below -80 give 0 (2^n stays normal).
UOCR_DEV float uocr_exp(float x) {
    if (!(x >= -80.0f)) return 0.0f;
    const float t = __fmul_rn(x, 1.44269504088896341f);
    const float n = rintf(t);
    float r = __fmaf_rn(-n, 0.693145751953125f, x);
    r = __fmaf_rn(-n, 1.428606765330187e-06f, r);
    float p = (float)(1.0 / 5040.0);
    p = __fmaf_rn(p, r, (float)(1.0 / 720.0));
    p = __fmaf_rn(p, r, (float)(1.0 / 120.0));
    p = __fmaf_rn(p, r, (float)(1.0 / 24.0));
    p = __fmaf_rn(p, r, (float)(1.0 / 6.0));
    p = __fmaf_rn(p, r, 0.5f);
    p = __fmaf_rn(p, r, 1.0f);
    p = __fmaf_rn(p, r, 1.0f);
    const int ni = (int)n;
    return __fmul_rn(p, __uint_as_float(uint32_t(ni + 127) << 23));
}

// SiLU for the expert epilogues (tolerance-checked path): a / (1 + e^-a).
UOCR_DEV float silu(float a) { return a / (1.0f + expf(-a)); }

// ---- loads -----------------------------------------------------------------------------
UOCR_DEV uint4 ldg_nc_v4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
UOCR_DEV uint2 ldg_nc_v2(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

UOCR_DEV float warp_sum_butterfly(float v) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    return v;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Opt a kernel into `bytes` of dynamic shared memory, calling cudaFuncSetAttribute only when
// the requirement grows (in practice on the first, eager call), so that later calls -- also
// inside CUDA-graph capture -- make no runtime configuration calls.
cudaError_t ensure_smem_optin(const void* kernel, size_t bytes);

}  // namespace uocr
