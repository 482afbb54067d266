// The reference's four MoE custom ops, 1:1 (kernels/moe_bf16.mojo, kernels/moe_int8.mojo,
// kernels/dense_bf16.mojo). Kernels only; argument checking lives in capi.cu.
//
// Each kernel has a vector-load path and a scalar path that visit the same elements in the
// same order with the same fp32 operations, so the bits never depend on which path the
// host picked (alignment, K not a multiple of the load width) -- the reference's
// ALIGNED/UNALIGNED/SCALAR property (kernels/loads.mojo:13-89).
#include "common.cuh"
#include "kernels.h"

namespace uocr {

// ---- moe_bf16_qmv --------------------------------------------------------------------
// One warp per (output column n, row s). Lane l owns the 8-element chunks c = l + 32 j
// (k = 8c .. 8c+7) and fma-chains them in ascending k; the 32 lane sums meet in an xor
// butterfly. A row reads only its own x, id and expert: its bits do not depend on the
// other rows of the call (moe_bf16.mojo:53-55).
constexpr int kQmvWarps = 4;

template <bool kVec>
__global__ void __launch_bounds__(kQmvWarps * 32)
bf16_qmv_kernel(float* __restrict__ out, const float* __restrict__ x, const int32_t* __restrict__ ids,
                const uint16_t* __restrict__ w, int E, int N, int K) {
    const int s = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * kQmvWarps + (threadIdx.x >> 5);
    if (n >= N) return;
    const int e = clamp_expert(ids[s], E);
    const uint16_t* wr = w + ((size_t)e * N + n) * K;
    const float* xr = x + (size_t)s * K;
    float acc = 0.0f;
    for (int k0 = lane * 8; k0 < K; k0 += 256) {
        if (kVec) {
            float wf[8];
            unpack_bf16x8(ldg_nc_v4(wr + k0), wf);
            const float4 xa = *reinterpret_cast<const float4*>(xr + k0);
            const float4 xb = *reinterpret_cast<const float4*>(xr + k0 + 4);
            acc = __fmaf_rn(wf[0], xa.x, acc);
            acc = __fmaf_rn(wf[1], xa.y, acc);
            acc = __fmaf_rn(wf[2], xa.z, acc);
            acc = __fmaf_rn(wf[3], xa.w, acc);
            acc = __fmaf_rn(wf[4], xb.x, acc);
            acc = __fmaf_rn(wf[5], xb.y, acc);
            acc = __fmaf_rn(wf[6], xb.z, acc);
            acc = __fmaf_rn(wf[7], xb.w, acc);
        } else {
            for (int i = 0; i < 8 && k0 + i < K; ++i) acc = __fmaf_rn(bf16f(wr[k0 + i]), xr[k0 + i], acc);
        }
    }
    acc = warp_sum_butterfly(acc);
    if (lane == 0) out[(size_t)s * N + n] = acc;
}

void launch_bf16_qmv(float* out, const float* x, const int32_t* ids, const uint16_t* w, int rows, int E, int N,
                     int K, bool vec, cudaStream_t st) {
    dim3 grid((N + kQmvWarps - 1) / kQmvWarps, rows);
    if (vec)
        bf16_qmv_kernel<true><<<grid, kQmvWarps * 32, 0, st>>>(out, x, ids, w, E, N, K);
    else
        bf16_qmv_kernel<false><<<grid, kQmvWarps * 32, 0, st>>>(out, x, ids, w, E, N, K);
}

// ---- moe_int8_qmv --------------------------------------------------------------------
// One thread per output (s, n), the reference's exact order (moe_int8.mojo:114-148):
// per group gsum = fma(q, x, gsum) over ascending k from 0, then acc = fma(scale, gsum, acc).
template <bool kVec>
__global__ void __launch_bounds__(256)
int8_qmv_kernel(float* __restrict__ out, const float* __restrict__ x, const int32_t* __restrict__ ids,
                const int8_t* __restrict__ w, const float* __restrict__ scales, int rows, int E, int N, int K,
                int groups) {
    const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (long)rows * N) return;
    const int s = (int)(idx / N);
    const int n = (int)(idx - (long)s * N);
    const int e = clamp_expert(ids[s], E);
    const int gsize = K / groups;
    const int8_t* wr = w + ((size_t)e * N + n) * K;
    const float* sr = scales + ((size_t)e * N + n) * groups;
    const float* xr = x + (size_t)s * K;
    float acc = 0.0f;
    for (int g = 0; g < groups; ++g) {
        float gsum = 0.0f;
        const int k_begin = g * gsize, k_end = k_begin + gsize;
        if (kVec) {
            for (int k0 = k_begin; k0 < k_end; k0 += 16) {
                const uint4 v = *reinterpret_cast<const uint4*>(wr + k0);
                float f[16];
                unpack_s8x8(v.x, v.y, *reinterpret_cast<float(*)[8]>(f));
                unpack_s8x8(v.z, v.w, *reinterpret_cast<float(*)[8]>(f + 8));
#pragma unroll
                for (int i = 0; i < 16; ++i) gsum = __fmaf_rn(f[i], xr[k0 + i], gsum);
            }
        } else {
            for (int kk = k_begin; kk < k_end; ++kk) gsum = __fmaf_rn((float)wr[kk], xr[kk], gsum);
        }
        acc = __fmaf_rn(sr[g], gsum, acc);
    }
    out[idx] = acc;
}

void launch_int8_qmv(float* out, const float* x, const int32_t* ids, const int8_t* w, const float* scales, int rows,
                     int E, int N, int K, int groups, bool vec, cudaStream_t st) {
    const long total = (long)rows * N;
    const int blocks = (int)((total + 255) / 256);
    if (vec)
        int8_qmv_kernel<true><<<blocks, 256, 0, st>>>(out, x, ids, w, scales, rows, E, N, K, groups);
    else
        int8_qmv_kernel<false><<<blocks, 256, 0, st>>>(out, x, ids, w, scales, rows, E, N, K, groups);
}

// ---- int8_dequant_expert -------------------------------------------------------------
// out[n, k] = bf16_rne(f32(q[e, n, k]) * scale[e, n, k / G]): one IEEE multiply, one RNE.
__global__ void __launch_bounds__(256)
int8_dequant_kernel(uint16_t* __restrict__ out, const int8_t* __restrict__ w, const float* __restrict__ scales,
                    const int32_t* __restrict__ idx, int E, int N, int K, int groups) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)N * K) return;
    const int e = clamp_expert(idx[0], E);
    const int n = (int)(i / K);
    const int k = (int)(i - (long)n * K);
    const int gsize = K / groups;
    const float q = (float)w[((size_t)e * N + n) * K + k];
    const float s = scales[((size_t)e * N + n) * groups + k / gsize];
    out[i] = f32_to_bf16_rne(__fmul_rn(q, s));
}

void launch_int8_dequant(uint16_t* out, const int8_t* w, const float* scales, const int32_t* idx, int E, int N,
                         int K, int groups, cudaStream_t st) {
    const long total = (long)N * K;
    int8_dequant_kernel<<<(int)((total + 255) / 256), 256, 0, st>>>(out, w, scales, idx, E, N, K, groups);
}

// ---- dense_bf16_qmv ------------------------------------------------------------------
// w K-blocked [K/16, N, 16]: thread (m, n) walks the K blocks in ascending order, one
// fma chain over the 16 elements of each block. Adjacent threads (adjacent n) read
// adjacent 32-byte blocks, so each block read coalesces.
template <bool kVec>
__global__ void __launch_bounds__(256)
dense_bf16_qmv_kernel(float* __restrict__ out, const float* __restrict__ x, const uint16_t* __restrict__ w, int M,
                      int N, int K) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    const int m = blockIdx.y;
    if (n >= N) return;
    const float* xr = x + (size_t)m * K;
    const int blocks = K / 16;
    float acc = 0.0f;
    for (int kb = 0; kb < blocks; ++kb) {
        const uint16_t* wb = w + ((size_t)kb * N + n) * 16;
        if (kVec) {
            float f0[8], f1[8];
            unpack_bf16x8(*reinterpret_cast<const uint4*>(wb), f0);
            unpack_bf16x8(*reinterpret_cast<const uint4*>(wb + 8), f1);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = __fmaf_rn(f0[i], xr[kb * 16 + i], acc);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = __fmaf_rn(f1[i], xr[kb * 16 + 8 + i], acc);
        } else {
            for (int i = 0; i < 16; ++i) acc = __fmaf_rn(bf16f(wb[i]), xr[kb * 16 + i], acc);
        }
    }
    out[(size_t)m * N + n] = acc;
}

void launch_dense_bf16_qmv(float* out, const float* x, const uint16_t* w, int M, int N, int K, bool vec,
                           cudaStream_t st) {
    dim3 grid((N + 255) / 256, M);
    if (vec)
        dense_bf16_qmv_kernel<true><<<grid, 256, 0, st>>>(out, x, w, M, N, K);
    else
        dense_bf16_qmv_kernel<false><<<grid, 256, 0, st>>>(out, x, w, M, N, K);
}

}  // namespace uocr
