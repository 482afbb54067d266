// Weight layout transforms, run once at load (the part of weight_adapters.stack_expert_weights
// that concerns the MoE tensors, unlimited_ocr_max/weight_adapters.py:121-163, re-laid out
// into the blocks of layout.h). Bit copies only.
#include "common.cuh"
#include "kernels.h"
#include "layout.h"

namespace uocr {

// Copy `words` 32-bit words, the CTA's threads striding over them.
__device__ void copy_words(uint32_t* dst, const uint32_t* src, long words) {
    for (long i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
}

// `rows` rows of `rb` bytes from src (contiguous) to dst rows of rb + kRowPad bytes (padding zeroed).
__device__ void copy_rows_padded(char* dst, const char* src, long rows, size_t rb) {
    const long wr = (long)(rb / 4), wp = (long)((rb + kRowPad) / 4);
    for (long i = threadIdx.x; i < rows * wp; i += blockDim.x) {
        const long r = i / wp, c = i - r * wp;
        reinterpret_cast<uint32_t*>(dst)[i] = c < wr ? reinterpret_cast<const uint32_t*>(src)[r * wr + c] : 0u;
    }
}

// One CTA per (block, expert): gate/up rows [pP, pP+P) and, for int8, their scales.
__global__ void pack_w13_kernel(const char* gate, const char* up, const float* gs, const float* us, int I, int H,
                                int G, int esz, int P, size_t block_bytes, char* out) {
    const long b = blockIdx.x, e = blockIdx.y;
    const long row0 = e * I + b * P;  // first source row (gate and up share row numbers)
    const size_t rb = (size_t)H * esz, prb = rb + kRowPad;
    char* dst = out + (e * (I / P) + b) * block_bytes;
    copy_rows_padded(dst, gate + row0 * rb, P, rb);
    copy_rows_padded(dst + P * prb, up + row0 * rb, P, rb);
    if (gs) {
        const long ng = H / G;
        float* ds = reinterpret_cast<float*>(dst + 2 * P * prb);
        copy_words(reinterpret_cast<uint32_t*>(ds), reinterpret_cast<const uint32_t*>(gs + row0 * ng), P * ng);
        copy_words(reinterpret_cast<uint32_t*>(ds + P * ng), reinterpret_cast<const uint32_t*>(us + row0 * ng),
                   P * ng);
    }
}

cudaError_t launch_pack_w13(const void* gate, const void* up, const float* gs, const float* us, int E, int I, int H,
                            int G, bool int8, void* out, cudaStream_t st) {
    const int P = w13_pairs(int8);
    dim3 grid((unsigned)(I / P), (unsigned)E);
    pack_w13_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const char*>(gate), reinterpret_cast<const char*>(up),
                                          int8 ? gs : nullptr, int8 ? us : nullptr, I, H, G, int8 ? 1 : 2, P,
                                          w13_block_bytes(H, G, int8), reinterpret_cast<char*>(out));
    return cudaGetLastError();
}

// One CTA per (block, expert): down rows [32b, 32b+32) and, for int8, their scales.
__global__ void pack_w2_kernel(const char* down, const float* ds, int H, int I, int G, int esz, size_t block_bytes,
                               char* out) {
    const long b = blockIdx.x, e = blockIdx.y;
    const long row0 = e * H + b * kW2Rows;
    const size_t rb = (size_t)I * esz;
    char* dst = out + (e * (H / kW2Rows) + b) * block_bytes;
    copy_rows_padded(dst, down + row0 * rb, kW2Rows, rb);
    if (ds) {
        const long ng = I / G;
        copy_words(reinterpret_cast<uint32_t*>(dst + kW2Rows * (rb + kRowPad)),
                   reinterpret_cast<const uint32_t*>(ds + row0 * ng), kW2Rows * ng);
    }
}

cudaError_t launch_pack_w2(const void* down, const float* ds, int E, int H, int I, int G, bool int8, void* out,
                           cudaStream_t st) {
    dim3 grid((unsigned)(H / kW2Rows), (unsigned)E);
    pack_w2_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const char*>(down), int8 ? ds : nullptr, H, I, G,
                                         int8 ? 1 : 2, w2_block_bytes(I, G, int8), reinterpret_cast<char*>(out));
    return cudaGetLastError();
}

// shared experts: gate/up [S*I, H] -> bf16 w13 blocks of S pseudo-experts; down [H, S*I] ->
// bf16 w2 rows [S*H] of I elements (+ padding)
__global__ void pack_shared_down_kernel(const uint16_t* down, long S, long I, long H, uint16_t* out) {
    const long j = blockIdx.x, s = blockIdx.y;
    const uint16_t* src = down + j * S * I + s * I;
    uint16_t* dst = out + (s * H + j) * (I + kRowPad / 2);
    for (long i = threadIdx.x; i < I + kRowPad / 2; i += blockDim.x) dst[i] = i < I ? src[i] : 0;
}

cudaError_t launch_pack_shared(const uint16_t* gate, const uint16_t* up, const uint16_t* down, long S, long I, long H,
                               uint16_t* w13, uint16_t* w2, cudaStream_t st) {
    cudaError_t err = launch_pack_w13(gate, up, nullptr, nullptr, (int)S, (int)I, (int)H, 128, false, w13, st);
    if (err != cudaSuccess) return err;
    pack_shared_down_kernel<<<dim3((unsigned)H, (unsigned)S), 128, 0, st>>>(down, S, I, H, w2);
    return cudaGetLastError();
}

}  // namespace uocr
