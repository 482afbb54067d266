// Symmetric per-group int8 quantisation along K (G = 128): the checkpoint format of the int8
// routed experts, computed on the GPU with the bits of the reference tool's numpy arithmetic
// (tools/quantize_int8.py:298-329, quantize_per_group):
//
//   amax  = max(max(w_g), -min(w_g))        fp32, exact
//   scale = amax / 127 (IEEE fp32 division); 1.0 when amax == 0
//   q     = clip(rint(w / scale), -127, 127) with a true fp32 division per element and rint
//           rounding half to even
//
// Every step is a correctly rounded fp32 operation, so the result is a function of the input bits
// alone and equals numpy's. A non-finite element sets *nonfinite (the host refuses the tensor; the
// outputs of such a group are unspecified).
//
// HBM-bound: per group 256 B of bf16 (512 B of fp32) read, 128 B of int8 and 4 B of scale
// written. Lane l of a warp holds 8 consecutive elements (one 16-byte bf16 load), a half-warp one
// group; a warp quantises kGroupsPerPass = 8 consecutive groups per pass with all of the pass's
// loads issued before the first reduction, and lane j < 8 computes group j's scale (one division
// and one reciprocal per lane per pass), handed to the other lanes by shuffles. Four blocks of 8
// warps per SM (64 registers) keep 64 KB of loads in flight per SM: measured 146 us for the
// 440 MB of one layer's experts (0.70 of the measured HBM copy rate), against 152 us with three
// blocks and 176-183 us with 12 or 16 groups per pass at two blocks.
//
// The per-element arithmetic, exact without a division per element:
// * amax = max |x| (an fp32 max with the absolute-value operand; equal to max(max, -min));
// * t = x * rcp(scale), both correctly rounded, is within |x/scale| * 1.5 * 2^-23 < 2.3e-5 of
//   the correctly rounded quotient fl(x/scale) (|x| <= amax, scale >= amax/127 * (1 - 2^-24), so
//   |x/scale| < 127.0001). rint changes value only across a half-integer, so wherever t is
//   farther than kTieMargin (6.1e-5) from one, rint(t) = rint(fl(x/scale)); the few elements
//   closer than that (exact .5 ties among them) take the IEEE division; the products, roundings
//   and differences run two elements per instruction (sm_100's f32x2 arithmetic);
// * rint by adding and subtracting 1.5 * 2^23 (round to nearest even for |t| < 2^22); the sum's
//   low byte is then the two's-complement int8;
// * |rint(fl(x/scale))| <= 127 for every finite x, so the reference's clip never binds.
// A scale below the smallest normal (its reciprocal could overflow) sends its group down the
// division path; a non-finite amax (a NaN-propagating max, so a NaN element shows) sets
// *nonfinite.
#include "common.cuh"
#include "kernels.h"

namespace uocr {
namespace {

constexpr int kGroup = 128;
constexpr int kPairsPerWarp = 4;
constexpr int kGroupsPerPass = 2 * kPairsPerWarp;
constexpr int kQuantThreads = 256;
constexpr float kTieMargin = 1.0f / 16384.0f;
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

template <bool VEC>
__device__ __forceinline__ void load8(const uint16_t* __restrict__ w, long long e, float v[8]) {
    uint32_t r[4];
    if constexpr (VEC) {
        const uint4 x = __ldcs(reinterpret_cast<const uint4*>(w + e));
        r[0] = x.x, r[1] = x.y, r[2] = x.z, r[3] = x.w;
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) r[i] = uint32_t(w[e + 2 * i]) | (uint32_t(w[e + 2 * i + 1]) << 16);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(r[i] << 16);
        v[2 * i + 1] = __uint_as_float(r[i] & 0xffff0000u);
    }
}

template <bool VEC>
__device__ __forceinline__ void load8(const float* __restrict__ w, long long e, float v[8]) {
    if constexpr (VEC) {
        const float4 a = __ldcs(reinterpret_cast<const float4*>(w + e));
        const float4 b = __ldcs(reinterpret_cast<const float4*>(w + e + 4));
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = w[e + i];
    }
}

// rint(q) + 1.5 * 2^23 for |q| < 2^22: the low byte is rint(q) as an int8.
__device__ __forceinline__ uint32_t rounded_bits(float q) { return __float_as_uint(__fadd_rn(q, kRoundMagic)); }

// Two fp32 lanes in one 64-bit register, operated on by the packed f32x2 instructions of sm_100
// (each lane correctly rounded, as the scalar instruction).
__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    return (static_cast<unsigned long long>(__float_as_uint(hi)) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float lo2(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v)); }
__device__ __forceinline__ float hi2(unsigned long long v) { return __uint_as_float(static_cast<uint32_t>(v >> 32)); }
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// max that returns NaN when either input is NaN (fmaxf would drop it)
__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(kQuantThreads, 4) quantize_g128_kernel(const T* __restrict__ w, long long groups,
                                                                      int8_t* __restrict__ q,
                                                                      float* __restrict__ scales,
                                                                      int* __restrict__ nonfinite) {
    constexpr int U = kPairsPerWarp;
    const int lane = threadIdx.x & 31;
    const int half = lane >> 4;
    const long long warp = (static_cast<long long>(blockIdx.x) * kQuantThreads + threadIdx.x) >> 5;
    const long long nwarps = (static_cast<long long>(gridDim.x) * kQuantThreads) >> 5;
    for (long long g0 = warp * kGroupsPerPass; g0 < groups; g0 += nwarps * kGroupsPerPass) {
        float v[U][8];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const long long g = g0 + 2 * u + half;
            if (g < groups) {
                load8<VEC>(w, g * kGroup + (lane & 15) * 8, v[u]);
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) v[u][i] = 0.f;
            }
        }
        // amax of group 2u + half in every lane of that half; lane j < 8 takes group j's
        float my_amax = 0.f;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float a = fabsf(v[u][0]);
#pragma unroll
            for (int i = 1; i < 8; ++i) a = max_nan(a, fabsf(v[u][i]));
#pragma unroll
            for (int o = 8; o; o >>= 1) a = max_nan(a, __shfl_xor_sync(0xffffffffu, a, o));
            const float mine = __shfl_sync(0xffffffffu, a, (lane & 1) * 16);
            if ((lane >> 1) == u) my_amax = mine;
        }
        const float my_scale = my_amax == 0.f ? 1.f : __fdiv_rn(my_amax, 127.f);
        const float my_inv = __frcp_rn(my_scale);
        bool bad = lane < kGroupsPerPass && g0 + lane < groups && !(my_amax <= 3.402823466e38f);
        if (lane < kGroupsPerPass && g0 + lane < groups) scales[g0 + lane] = my_scale;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const float scale = __shfl_sync(0xffffffffu, my_scale, 2 * u + half);
            const float inv = __shfl_sync(0xffffffffu, my_inv, 2 * u + half);
            const long long g = g0 + 2 * u + half;
            if (g >= groups) continue;
            const bool exact_group = scale < 0x1p-126f;
            const unsigned long long inv2 = pack2(inv, inv), magic2 = pack2(kRoundMagic, kRoundMagic);
            uint32_t y[8];
            float dmax = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const unsigned long long t2 = mul2(pack2(v[u][2 * i], v[u][2 * i + 1]), inv2);
                const unsigned long long y2 = add2(t2, magic2);
                const unsigned long long d2 = sub2(t2, sub2(y2, magic2));
                y[2 * i] = static_cast<uint32_t>(y2);
                y[2 * i + 1] = static_cast<uint32_t>(y2 >> 32);
                dmax = fmaxf(dmax, fmaxf(fabsf(lo2(d2)), fabsf(hi2(d2))));
            }
            if (exact_group || !(dmax <= 0.5f - kTieMargin)) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float tq = v[u][i] * inv;
                    const float r = __fsub_rn(__fadd_rn(tq, kRoundMagic), kRoundMagic);
                    if (exact_group || !(fabsf(__fsub_rn(tq, r)) <= 0.5f - kTieMargin))
                        y[i] = rounded_bits(__fdiv_rn(v[u][i], scale));
                }
            }
            const uint32_t lo = __byte_perm(__byte_perm(y[0], y[1], 0x0040), __byte_perm(y[2], y[3], 0x0040), 0x5410);
            const uint32_t hi = __byte_perm(__byte_perm(y[4], y[5], 0x0040), __byte_perm(y[6], y[7], 0x0040), 0x5410);
            int8_t* dst = q + g * kGroup + (lane & 15) * 8;
            if constexpr (VEC) {
                __stcs(reinterpret_cast<uint2*>(dst), make_uint2(lo, hi));
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    dst[i] = static_cast<int8_t>((lo >> (8 * i)) & 0xffu);
                    dst[4 + i] = static_cast<int8_t>((hi >> (8 * i)) & 0xffu);
                }
            }
        }
        if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(nonfinite, 1);
    }
}

template <typename T, bool VEC>
cudaError_t launch_typed(const T* w, long long groups, int8_t* q, float* scales, int* nonfinite, cudaStream_t st) {
    int dev = 0, sms = 148, per_sm = 8;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return err;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, quantize_g128_kernel<T, VEC>, kQuantThreads, 0);
    if (err != cudaSuccess) return err;
    const long long per_block = (kQuantThreads / 32) * kGroupsPerPass;
    const long long want = (groups + per_block - 1) / per_block;
    const int grid = static_cast<int>(std::min<long long>(want, static_cast<long long>(sms) * std::max(per_sm, 1)));
    quantize_g128_kernel<T, VEC><<<grid, kQuantThreads, 0, st>>>(w, groups, q, scales, nonfinite);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_quantize_g128(const void* w, bool bf16, long long groups, int8_t* q, float* scales,
                                 int* nonfinite, bool vec, cudaStream_t st) {
    if (groups <= 0) return cudaSuccess;
    if (bf16) {
        const auto* p = static_cast<const uint16_t*>(w);
        return vec ? launch_typed<uint16_t, true>(p, groups, q, scales, nonfinite, st)
                   : launch_typed<uint16_t, false>(p, groups, q, scales, nonfinite, st);
    }
    const auto* p = static_cast<const float*>(w);
    return vec ? launch_typed<float, true>(p, groups, q, scales, nonfinite, st)
               : launch_typed<float, false>(p, groups, q, scales, nonfinite, st);
}

}  // namespace uocr
