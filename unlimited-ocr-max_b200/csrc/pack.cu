// Weight layout transforms, run once at load (the part of weight_adapters.stack_expert_weights
// that concerns the MoE tensors, unlimited_ocr_max/weight_adapters.py:121-163, re-laid out
// into the swizzled items of layout.h). Bit copies only.
#include "common.cuh"
#include "kernels.h"
#include "layout.h"

namespace uocr {

// One CTA per item: `atoms` atoms of 128 rows over K elements [k0, k0 + atoms * ak), 16-byte
// chunks; row r's source is row_ptr(r) (element size esz). int8: scales [atom][row] from
// scale_ptr(r)[group of the atom].
template <class RowFn, class ScaleFn>
__device__ void pack_item(char* dst, int atoms, int ak, int esz, int k0, bool int8, RowFn row_ptr, ScaleFn scale_ptr) {
    const int chunks = atoms * kRowBlock * 8;  // 8 chunks of 16 bytes per atom row
    for (int i = threadIdx.x; i < chunks; i += blockDim.x) {
        const int a = i / (kRowBlock * 8), rem = i - a * kRowBlock * 8, r = rem >> 3, cc = rem & 7;
        const char* src = row_ptr(r) + (size_t)(k0 + a * ak) * esz + cc * 16;
        *reinterpret_cast<uint4*>(dst + (size_t)a * kAtomBytes + atom_offset(r, cc * 16)) =
            *reinterpret_cast<const uint4*>(src);
    }
    if (int8) {
        float* sc = reinterpret_cast<float*>(dst + (size_t)atoms * kAtomBytes);
        for (int i = threadIdx.x; i < atoms * kRowBlock; i += blockDim.x) {
            const int a = i / kRowBlock, r = i - a * kRowBlock;
            sc[i] = scale_ptr(r)[(k0 + a * ak) / 128];
        }
    }
}

// grid (items per row block x row blocks, E): gate/up pairs [64 rb, 64 rb + 64) of expert e.
// Source rows: gate/up + (e * estride + p * ld) elements; scales [E * I][H / 128].
__global__ void pack_w13_kernel(const char* gate, const char* up, const float* gs, const float* us, int I, int H,
                                long estride, long ld, int esz, bool int8, char* out) {
    const int nk = w13_items(H, int8);
    const int rb = blockIdx.x / nk, ki = blockIdx.x - rb * nk, e = blockIdx.y;
    const size_t ib = w13_item_bytes(int8);
    char* dst = out + (size_t)e * w13_expert_bytes(I, H, int8) + ((size_t)rb * nk + ki) * ib;
    auto pair = [&](int r) { return 64 * rb + (r >> 4) * 8 + (r & 7); };
    auto row_ptr = [&](int r) {
        return ((r & 15) >= 8 ? up : gate) + ((size_t)e * estride + (size_t)pair(r) * ld) * esz;
    };
    auto scale_ptr = [&](int r) {
        return ((r & 15) >= 8 ? us : gs) + ((size_t)e * I + pair(r)) * (H / 128);
    };
    pack_item(dst, w13_atoms(), atom_k(int8), esz, ki * w13_atoms() * atom_k(int8), int8, row_ptr, scale_ptr);
}

cudaError_t launch_pack_w13(const void* gate, const void* up, const float* gs, const float* us, int E, int I, int H,
                            bool int8, long estride, long ld, void* out, cudaStream_t st) {
    dim3 grid((unsigned)((I / 64) * w13_items(H, int8)), (unsigned)E);
    pack_w13_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const char*>(gate), reinterpret_cast<const char*>(up),
                                          int8 ? gs : nullptr, int8 ? us : nullptr, I, H, estride, ld, int8 ? 1 : 2,
                                          int8, reinterpret_cast<char*>(out));
    return cudaGetLastError();
}

// grid (items per row block x row blocks, E): output rows [128 rb, 128 rb + 128) of expert e.
// Source rows: down + (e * estride + j * ld) elements; scales [E * H][I / 128].
__global__ void pack_w2_kernel(const char* down, const float* ds, int H, int I, long estride, long ld, int esz,
                               bool int8, char* out) {
    const int nk = w2_items(I, int8);
    const int rb = blockIdx.x / nk, ki = blockIdx.x - rb * nk, e = blockIdx.y;
    char* dst = out + (size_t)e * w2_expert_bytes(H, I, int8) + (size_t)rb * w2_rb_bytes(I, int8) +
                w2_item_offset(int8, ki);
    auto row_ptr = [&](int r) { return down + ((size_t)e * estride + (size_t)(kRowBlock * rb + r) * ld) * esz; };
    auto scale_ptr = [&](int r) { return ds + ((size_t)e * H + kRowBlock * rb + r) * (I / 128); };
    pack_item(dst, w2_item_atoms(I, int8, ki), atom_k(int8), esz, ki * kW2Atoms * atom_k(int8), int8, row_ptr,
              scale_ptr);
}

cudaError_t launch_pack_w2(const void* down, const float* ds, int E, int H, int I, bool int8, long estride, long ld,
                           void* out, cudaStream_t st) {
    dim3 grid((unsigned)((H / kRowBlock) * w2_items(I, int8)), (unsigned)E);
    pack_w2_kernel<<<grid, 256, 0, st>>>(reinterpret_cast<const char*>(down), int8 ? ds : nullptr, H, I, estride, ld,
                                         int8 ? 1 : 2, int8, reinterpret_cast<char*>(out));
    return cudaGetLastError();
}

// Shared experts: gate/up [S*I, H] -> bf16 w13 items of S pseudo-experts (expert s = rows
// [sI, (s+1)I)); down [H, S*I] -> bf16 w2 items (pseudo-expert s = columns [sI, (s+1)I)).
cudaError_t launch_pack_shared(const uint16_t* gate, const uint16_t* up, const uint16_t* down, long S, long I, long H,
                               uint16_t* w13, uint16_t* w2, cudaStream_t st) {
    cudaError_t err = launch_pack_w13(gate, up, nullptr, nullptr, (int)S, (int)I, (int)H, false, I * H, H, w13, st);
    if (err != cudaSuccess) return err;
    return launch_pack_w2(down, nullptr, (int)S, (int)H, (int)I, false, I, S * I, w2, st);
}

}  // namespace uocr
