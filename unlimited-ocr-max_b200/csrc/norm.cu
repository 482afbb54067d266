// The residual add and the RMSNorm around each MoE sublayer of the decode step
// (DecoderLayer.decode, decoder.py:702-709: x = x + mlp.decode_rows(post_attention_layernorm(x));
// RmsNorm, decoder.py:252-261: ops.rms_norm(x, gamma, eps) with the bf16 gamma cast to fp32).
//
// One fused launch between two MoE sublayers: h += add (the previous sublayer's output), then
// y = h / sqrt(mean(h^2) + eps) * gamma (the next sublayer's input). One CTA per row; the sum of
// squares is a fixed-order block reduction (fp32), the scale 1 / sqrt(.) is IEEE-rounded. Either
// half may be skipped: add == nullptr (the first norm), y == nullptr (the last residual add).
// Latency-bound (B <= 8 rows of H fp32).
#include "common.cuh"
#include "kernels.h"

namespace uocr {
namespace {

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) residual_rmsnorm_kernel(float* __restrict__ h,
                                                                        const float* __restrict__ add,
                                                                        const float* __restrict__ gamma, int H,
                                                                        float eps, float* __restrict__ y) {
    __shared__ float part[kNormThreads / 32];
    __shared__ float scale;
    float* hr = h + (size_t)blockIdx.x * H;
    const float* ar = add ? add + (size_t)blockIdx.x * H : nullptr;
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += kNormThreads) {
        float v = hr[i];
        if (ar) {
            v = __fadd_rn(v, ar[i]);
            hr[i] = v;
        }
        ss = fmaf(v, v, ss);
    }
    if (!y) return;
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int w = 0; w < kNormThreads / 32; ++w) s += part[w];
        scale = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)H), eps)));
    }
    __syncthreads();
    const float sc = scale;
    float* yr = y + (size_t)blockIdx.x * H;
    for (int i = threadIdx.x; i < H; i += kNormThreads) yr[i] = __fmul_rn(__fmul_rn(hr[i], sc), gamma[i]);
}

}  // namespace

cudaError_t launch_residual_rmsnorm(float* h, const float* add, const float* gamma, int B, int H, float eps, float* y,
                                    cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    residual_rmsnorm_kernel<<<B, kNormThreads, 0, st>>>(h, add, gamma, H, eps, y);
    return cudaGetLastError();
}

}  // namespace uocr
