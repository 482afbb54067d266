// RoPE on the decode step's fused q|k|v rows (Attention._rope, decoder.py:459-462, applied to q and
// k in Attention.decode, decoder.py:478-493): per row b and head h, with rotate_half(x) =
// concat(-x[half:], x[:half]),
//
//   q = x_q * cos[b] + rotate_half(x_q) * sin[b],   k likewise,   v = x_v unchanged,
//
// each product and the sum rounded separately in fp32 (no fused multiply-add), from the [B, 3 x
// heads x dim] output of the fused q|k|v projection into three [B, heads, dim] buffers the paged
// attention reads. cos / sin are the rows of the rotary table at each request's position
// ([B, dim]). Elementwise; one thread per output element of q and k (v is copied).
#include "common.cuh"
#include "kernels.h"

namespace uocr {
namespace {

__global__ void rope_qkv_kernel(const float* __restrict__ qkv, int B, int heads, int dim,
                                const float* __restrict__ cos, const float* __restrict__ sin, float* __restrict__ q,
                                float* __restrict__ k, float* __restrict__ v) {
    const int width = heads * dim, half = dim / 2;
    const long long total = (long long)B * width;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / width), j = (int)(i % width), d = j % dim;
        const float* row = qkv + (size_t)b * 3 * width;
        const float c = cos[(size_t)b * dim + d], s = sin[(size_t)b * dim + d];
        const int partner = d < half ? j + half : j - half;
        const float xq = row[j], rq = d < half ? -row[partner] : row[partner];
        const float xk = row[width + j], rk = d < half ? -row[width + partner] : row[width + partner];
        q[i] = __fadd_rn(__fmul_rn(xq, c), __fmul_rn(rq, s));
        k[i] = __fadd_rn(__fmul_rn(xk, c), __fmul_rn(rk, s));
        v[i] = row[2 * width + j];
    }
}

}  // namespace

cudaError_t launch_rope_qkv(const float* qkv, int B, int heads, int dim, const float* cos, const float* sin, float* q,
                            float* k, float* v, cudaStream_t st) {
    const long long total = (long long)B * heads * dim;
    if (total <= 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 255) / 256, 148 * 8);
    rope_qkv_kernel<<<grid, 256, 0, st>>>(qkv, B, heads, dim, cos, sin, q, k, v);
    return cudaGetLastError();
}

}  // namespace uocr
