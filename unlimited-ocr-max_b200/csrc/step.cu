// The two elementwise pieces of the decode step that are neither a projection nor a norm:
//
// * the token embedding (EmbeddingTable, decoder.py:241-249: a gather of the bf16 table's rows),
//   widened to the fp32 residual stream; token ids are clamped into [0, vocab);
// * the dense FFN's activation (GatedMlp.decode_rows, decoder.py:276-278: silu(gate(x)) * up(x)) on
//   the fused gate|up projection's output [B, 2 x I]: silu(g) = g / (1 + e^-g) in fp32, times u.
//
// Both elementwise (one thread per output element, 16-byte loads where the rows allow).
#include "common.cuh"
#include "kernels.h"

namespace uocr {
namespace {

__global__ void embed_rows_kernel(const uint16_t* __restrict__ table, int V, int H, const int32_t* __restrict__ ids,
                                  int B, float* __restrict__ out) {
    const long long total = (long long)B * H;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / H), d = (int)(i % H);
        const int tok = min(max(ids[b], 0), V - 1);
        out[i] = bf16f(table[(size_t)tok * H + d]);
    }
}

__global__ void silu_mul_kernel(const float* __restrict__ gu, int B, int I, float* __restrict__ out) {
    const long long total = (long long)B * I;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int b = (int)(i / I), j = (int)(i % I);
        const float g = gu[(size_t)b * 2 * I + j], u = gu[(size_t)b * 2 * I + I + j];
        out[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.f, expf(-g))), u);
    }
}

int grid_for(long long total) { return (int)std::min<long long>((total + 255) / 256, 148 * 8); }

}  // namespace

cudaError_t launch_embed_rows(const uint16_t* table, int V, int H, const int32_t* ids, int B, float* out,
                              cudaStream_t st) {
    const long long total = (long long)B * H;
    if (total <= 0) return cudaSuccess;
    embed_rows_kernel<<<grid_for(total), 256, 0, st>>>(table, V, H, ids, B, out);
    return cudaGetLastError();
}

cudaError_t launch_silu_mul(const float* gu, int B, int I, float* out, cudaStream_t st) {
    const long long total = (long long)B * I;
    if (total <= 0) return cudaSuccess;
    silu_mul_kernel<<<grid_for(total), 256, 0, st>>>(gu, B, I, out);
    return cudaGetLastError();
}

}  // namespace uocr
