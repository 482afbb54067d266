// Weight layout transforms, run once at load (the part of weight_adapters.stack_expert_weights
// that concerns the MoE tensors, unlimited_ocr_max/weight_adapters.py:121-163, re-laid out
// for this library's kernels). Bit copies only.
#include "common.cuh"
#include "kernels.h"

namespace uocr {

// Copy `bytes` bytes (a multiple of 4) from src to dst with 32-bit words, one row per CTA.
__device__ void copy_row_words(uint32_t* dst, const uint32_t* src, long words) {
    for (long i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
}

// gate/up [E, I, H] -> [E, 2I, H], rows interleaved in blocks of 128:
// packed row 256b + r    <- gate row 128b + r
// packed row 256b+128+r  <- up   row 128b + r
__global__ void pack_gate_up_kernel(const char* gate, const char* up, long I, long row_bytes, char* out) {
    const long prow = blockIdx.x;          // packed row within the expert
    const long e = blockIdx.y;
    const long blk = prow / 256, r = prow % 256;
    const bool is_up = r >= 128;
    const long src_row = blk * 128 + (r % 128);
    const char* src = (is_up ? up : gate) + (e * I + src_row) * row_bytes;
    char* dst = out + (e * 2 * I + prow) * row_bytes;
    copy_row_words(reinterpret_cast<uint32_t*>(dst), reinterpret_cast<const uint32_t*>(src), row_bytes / 4);
}

cudaError_t launch_pack_gate_up(const void* gate, const void* up, long E, long I, long H, int esz, void* out,
                                cudaStream_t st) {
    dim3 grid((unsigned)(2 * I), (unsigned)E);
    pack_gate_up_kernel<<<grid, 128, 0, st>>>(reinterpret_cast<const char*>(gate), reinterpret_cast<const char*>(up),
                                              I, H * esz, reinterpret_cast<char*>(out));
    return cudaGetLastError();
}

// shared experts: gate/up [S*I, H] -> [S, 2I, H] (interleaved as above); down [H, S*I] -> [S, H, I]
__global__ void pack_shared_gate_up_kernel(const uint16_t* gate, const uint16_t* up, long I, long H, uint16_t* out) {
    const long prow = blockIdx.x, s = blockIdx.y;
    const long blk = prow / 256, r = prow % 256;
    const long src_row = s * I + blk * 128 + (r % 128);
    const uint16_t* src = (r >= 128 ? up : gate) + src_row * H;
    uint16_t* dst = out + (s * 2 * I + prow) * H;
    copy_row_words(reinterpret_cast<uint32_t*>(dst), reinterpret_cast<const uint32_t*>(src), H / 2);
}

__global__ void pack_shared_down_kernel(const uint16_t* down, long S, long I, long H, uint16_t* out) {
    const long j = blockIdx.x, s = blockIdx.y;
    const uint16_t* src = down + j * S * I + s * I;
    uint16_t* dst = out + (s * H + j) * I;
    for (long i = threadIdx.x; i < I; i += blockDim.x) dst[i] = src[i];
}

cudaError_t launch_pack_shared(const uint16_t* gate, const uint16_t* up, const uint16_t* down, long S, long I, long H,
                               uint16_t* w13, uint16_t* w2, cudaStream_t st) {
    pack_shared_gate_up_kernel<<<dim3((unsigned)(2 * I), (unsigned)S), 128, 0, st>>>(gate, up, I, H, w13);
    pack_shared_down_kernel<<<dim3((unsigned)H, (unsigned)S), 128, 0, st>>>(down, S, I, H, w2);
    return cudaGetLastError();
}

}  // namespace uocr
