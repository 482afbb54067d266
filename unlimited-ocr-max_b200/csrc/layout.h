// Packed expert-weight layouts (host and device). Weights are repacked once at load into the
// shared-memory image the tcgen05 tensor cores read: K-major rows in 128-byte-swizzle atoms.
//
// Atom: R rows x 128 bytes of one K range (128 int8 or 64 bf16 elements); byte c of row r sits at
//     r * 128 + (((c / 16) ^ (r % 8)) * 16) + c % 16
// (the 128-byte swizzle, 8-row groups 1024 bytes apart), so a block copied verbatim to a
// 1024-byte-aligned shared-memory address is a valid SWIZZLE_128B K-major MMA operand.
//
// Row block: 128 rows (the MMA's M). Item: the row block's atoms over one K range plus, for
// int8, their fp32 scales [atom][128 rows] (one 128-element group per int8 atom):
//     [atom 0: 128 rows x 128 B][atom 1]...[int8: scales of atom 0 (128 fp32)][atom 1]...
// A decode work item is exactly one item: one bulk copy.
//
// gate|up "w13", per expert I/64 row blocks of 64 row pairs, rows interleaved in groups of 8
// (rows 16i..16i+7 = gate pairs 8i..8i+7, rows 16i+8..16i+15 = the matching up pairs), each
// row block H / item_k items of 2 atoms (int8: K 256 = 2 groups; bf16: K 128).
// down "w2", per expert H/128 row blocks of 128 output rows, each of items of 2 atoms (int8: K
// 256 = 2 groups, the last item 1 atom when I/128 is odd; bf16: K 128).
// For bf16 the items of a row block are its atoms back to back, so the whole stack is the 4-D
// array [row block][K / 64 atoms][128 rows][128 B]: the prefill GEMM reads 256-row tiles of it
// through a 4-D tensor map (two consecutive row blocks, one atom) without swizzling.
// Shared experts (always bf16): w13_shared / w2_shared in the bf16 layouts with S pseudo-experts
// (shared expert q owns intermediate rows [qI, (q+1)I) of the checkpoint's shared MLP).
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace uocr {

constexpr int kRowBlock = 128;    // rows of a row block
constexpr int kAtomRowBytes = 128;
constexpr int kAtomBytes = kRowBlock * kAtomRowBytes;  // 16 KB

// byte offset of (row r, byte c) inside an atom
__host__ __device__ inline uint32_t atom_offset(int r, int c) {
    return (uint32_t)r * 128u + ((((uint32_t)c >> 4) ^ ((uint32_t)r & 7u)) << 4) + ((uint32_t)c & 15u);
}

__host__ __device__ inline int w13_atoms() { return 2; }
constexpr int kW2Atoms = 2;  // atoms of a full down item (int8 and bf16)
// K elements of one atom
__host__ __device__ inline int atom_k(bool int8) { return int8 ? 128 : 64; }
__host__ __device__ inline size_t item_bytes(int atoms, bool int8) {
    return (size_t)atoms * kAtomBytes + (int8 ? (size_t)atoms * kRowBlock * 4 : 0);
}
// items per row block, and item bytes, of the gate|up and down stacks
__host__ __device__ inline int w13_items(int H, bool int8) { return H / (w13_atoms() * atom_k(int8)); }
__host__ __device__ inline size_t w13_item_bytes(bool int8) { return item_bytes(w13_atoms(), int8); }
// down items of a row block: K atoms I / atom_k in items of kW2Atoms (the last may be shorter)
__host__ __device__ inline int w2_atoms_total(int I, bool int8) { return I / atom_k(int8); }
__host__ __device__ inline int w2_items(int I, bool int8) { return (w2_atoms_total(I, int8) + kW2Atoms - 1) / kW2Atoms; }
__host__ __device__ inline int w2_item_atoms(int I, bool int8, int ki) {
    const int left = w2_atoms_total(I, int8) - ki * kW2Atoms;
    return left < kW2Atoms ? left : kW2Atoms;
}
__host__ __device__ inline size_t w2_item_offset(bool int8, int ki) { return (size_t)ki * item_bytes(kW2Atoms, int8); }
__host__ __device__ inline size_t w2_rb_bytes(int I, bool int8) {
    const int n = w2_items(I, int8);
    return w2_item_offset(int8, n - 1) + item_bytes(w2_item_atoms(I, int8, n - 1), int8);
}
__host__ __device__ inline size_t w13_expert_bytes(int I, int H, bool int8) {
    return (size_t)(I / 64) * w13_items(H, int8) * w13_item_bytes(int8);
}
__host__ __device__ inline size_t w2_expert_bytes(int H, int I, bool int8) {
    return (size_t)(H / kRowBlock) * w2_rb_bytes(I, int8);
}
// row of the gate|up row block holding gate (up = 0) or up (up = 1) pair p (0..63)
__host__ __device__ inline int w13_block_row(int p, int up) { return (p >> 3) * 16 + up * 8 + (p & 7); }

}  // namespace uocr
