// Packed expert-weight layouts (host and device). Weights are repacked once at load into
// contiguous blocks sized for one bulk copy each: a decode work item is exactly one block, so
// the streaming kernels issue one large copy per item instead of one per row and scale run.
// Every packed row is followed by 16 bytes of padding: rows of a block then start on different
// shared-memory banks, so the tensor-core fragment loads (8 rows x 8 bytes per lane group) are
// conflict-free.
//
// gate|up "w13", per expert, I / P blocks of P row pairs (P = 8 for bf16, 16 for int8):
//     [gate rows pP .. pP+P-1 | up rows pP .. pP+P-1          (2P rows of row_bytes)
//      | int8 only: gate scales (P x H/G fp32) | up scales (P x H/G fp32)]
//   For bf16 this is the [E*2I, H] row matrix (row stride H + 8 elements) with gate and up rows
//   interleaved in groups of 8: the prefill GEMM reads it through a 2-D tensor map (a 256-row
//   tile = 128 gate + 128 up rows, paired column c <-> c + 8 within every 16).
// down "w2", per expert, H / 32 blocks of 32 rows:
//     [rows (32 rows of row_bytes) | int8 only: scales (32 x I/G fp32)]
//   For bf16 this is the [E*H, I] row matrix with row stride I + 8 elements.
// Shared experts (always bf16): w13_shared as bf16 w13 with S pseudo-experts (shared expert q
// owns intermediate rows [qI, (q+1)I) of the checkpoint's shared MLP); w2_shared as bf16 w2.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace uocr {

constexpr int kW2Rows = 32;   // rows per down block
constexpr int kRowPad = 16;   // bytes after every packed row

// bytes of one packed row of K elements
__host__ __device__ inline size_t packed_row_bytes(int K, bool int8) {
    return (size_t)K * (int8 ? 1 : 2) + kRowPad;
}
__host__ __device__ inline int w13_pairs(bool int8) { return int8 ? 16 : 8; }
__host__ __device__ inline size_t w13_block_bytes(int H, int G, bool int8) {
    const size_t P = (size_t)w13_pairs(int8);
    return 2 * P * packed_row_bytes(H, int8) + (int8 ? 2 * P * (size_t)(H / G) * 4 : 0);
}
__host__ __device__ inline size_t w13_expert_bytes(int I, int H, int G, bool int8) {
    return (size_t)(I / w13_pairs(int8)) * w13_block_bytes(H, G, int8);
}
__host__ __device__ inline size_t w2_block_bytes(int I, int G, bool int8) {
    return (size_t)kW2Rows * packed_row_bytes(I, int8) + (int8 ? (size_t)kW2Rows * (I / G) * 4 : 0);
}
__host__ __device__ inline size_t w2_expert_bytes(int H, int I, int G, bool int8) {
    return (size_t)(H / kW2Rows) * w2_block_bytes(I, G, int8);
}

}  // namespace uocr
