// Decode-step MoE sublayer (MoE.decode_rows, unlimited_ocr_max/decoder.py:641-655) for
// B <= 8 tokens: HBM-bound weight streaming.
//
// Pairs. Routed (token t, slot s) is pair t*k + s; shared expert q's copy of token t is
// pair k*B + q*B + t. Every pair is one SwiGLU expert evaluation:
//   h[p, n]  = silu(Wg[e, n, :] . x[t]) * (Wu[e, n, :] . x[t])          (gate/up kernel)
//   y[p, j]  = Wd[e, j, :] . h[p]                                      (down kernel)
//   out[t,j] = sum_s w[t,s] * y[t*k+s, j] + sum_q y[k*B+q*B+t, j]        (combine kernel)
// Work items are (expert slot, row block). Expert slots 0..S-1 are the shared experts;
// slot S+r is the r-th distinct routed expert in ascending id. Every item reads its rows
// of the expert ONCE for all the pairs routed to that expert (the reference's "read once"
// property, kernels/moe_routing.mojo:1-16). A pair's sums use only its own token and
// expert, so its bits do not depend on B or on which tokens share an expert.
#include "common.cuh"
#include "kernels.h"

namespace uocr {

constexpr int kDecWarps = 8;
constexpr int kDecRowsPerWarp = 4;
constexpr int kDecRowsPerCta = kDecWarps * kDecRowsPerWarp;  // 32
constexpr int kMaxB = 8;

struct ExpertSlot {
    int valid;
    int expert;             // routed expert id, or shared expert index
    int shared;             // 1 for a shared expert
    int count;              // pairs served
    int pair[kMaxB];        // pair index per served token
    int token[kMaxB];       // token index per served pair
    float weight[kMaxB];    // routing weight (1 for shared)
};

// Resolve blockIdx.y into the expert slot this CTA serves (thread 0 only).
__device__ void resolve_slot(ExpertSlot& es, int u, const DecodeArgs& a) {
    es.valid = 0;
    es.count = 0;
    const int kB = a.topk * a.B;
    if (u < a.S) {
        es.valid = 1;
        es.shared = 1;
        es.expert = u;
        es.count = a.B;
        for (int t = 0; t < a.B; ++t) {
            es.pair[t] = kB + u * a.B + t;
            es.token[t] = t;
            es.weight[t] = 1.0f;
        }
        return;
    }
    unsigned long long used = 0ull;
    for (int p = 0; p < kB; ++p) used |= 1ull << clamp_expert(a.ids[p], a.E);
    int r = u - a.S;
    if (r >= __popcll(used)) return;
    for (int i = 0; i < r; ++i) used &= used - 1ull;  // drop the r lowest set bits
    const int e = __ffsll(used) - 1;
    es.valid = 1;
    es.shared = 0;
    es.expert = e;
    for (int p = 0; p < kB; ++p) {
        if (clamp_expert(a.ids[p], a.E) == e) {
            es.pair[es.count] = p;
            es.token[es.count] = p / a.topk;
            es.weight[es.count] = a.wts[p];
            ++es.count;
        }
    }
}

// One 8-element chunk of a weight row (bf16 or int8) as fp32.
template <bool kInt8>
UOCR_DEV void load_chunk(const void* row, int k0, float (&f)[8]) {
    if (kInt8) {
        const uint2 v = ldg_nc_v2(reinterpret_cast<const int8_t*>(row) + k0);
        unpack_s8x8(v.x, v.y, f);
    } else {
        unpack_bf16x8(ldg_nc_v4(reinterpret_cast<const uint16_t*>(row) + k0), f);
    }
}

UOCR_DEV float dot8(const float (&w)[8], const float* xs) {
    const float4 xa = *reinterpret_cast<const float4*>(xs);
    const float4 xb = *reinterpret_cast<const float4*>(xs + 4);
    float d = __fmul_rn(w[0], xa.x);
    d = __fmaf_rn(w[1], xa.y, d);
    d = __fmaf_rn(w[2], xa.z, d);
    d = __fmaf_rn(w[3], xa.w, d);
    d = __fmaf_rn(w[4], xb.x, d);
    d = __fmaf_rn(w[5], xb.y, d);
    d = __fmaf_rn(w[6], xb.z, d);
    d = __fmaf_rn(w[7], xb.w, d);
    return d;
}

// ---- gate/up + SwiGLU -----------------------------------------------------------------
// CTA = (row block of 32 intermediate rows, expert slot); warp = 4 rows, one at a time;
// lane l reads the 8-element chunks k0 = 8l + 256j of the gate row and the up row.
template <bool kRoutedInt8>
__global__ void __launch_bounds__(kDecWarps * 32)
decode_gate_up_kernel(DecodeArgs a) {
    extern __shared__ float xs[];  // [count][H]
    __shared__ ExpertSlot es;
    if (threadIdx.x == 0) resolve_slot(es, blockIdx.y, a);
    __syncthreads();
    if (!es.valid) return;
    const int H = a.H, I = a.I, c = es.count;
    for (int i = threadIdx.x; i < c * H; i += blockDim.x) {
        const int ci = i / H;
        xs[i] = a.x[(size_t)es.token[ci] * H + (i - ci * H)];
    }
    __syncthreads();

    const bool int8 = kRoutedInt8 && !es.shared;
    const size_t expert_rows = (size_t)2 * I;
    const void* wbase;
    const float* sbase = nullptr;
    if (es.shared) {
        wbase = a.w13_shared + (size_t)es.expert * expert_rows * H;
    } else if (kRoutedInt8) {
        wbase = reinterpret_cast<const int8_t*>(a.w13) + (size_t)es.expert * expert_rows * H;
        sbase = a.s13 + (size_t)es.expert * expert_rows * (H / a.G);
    } else {
        wbase = reinterpret_cast<const uint16_t*>(a.w13) + (size_t)es.expert * expert_rows * H;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gsz = a.G;
    for (int i = 0; i < kDecRowsPerWarp; ++i) {
        const int n = blockIdx.x * kDecRowsPerCta + warp * kDecRowsPerWarp + i;
        if (n >= I) break;
        const int pg = (n / 128) * 256 + (n % 128);  // packed gate row
        const int pu = pg + 128;                     // packed up row
        const size_t esz = int8 ? 1 : 2;
        const char* rg = reinterpret_cast<const char*>(wbase) + (size_t)pg * H * esz;
        const char* ru = reinterpret_cast<const char*>(wbase) + (size_t)pu * H * esz;
        float ag[kMaxB], au[kMaxB];
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) ag[q] = au[q] = 0.0f;
        for (int k0 = lane * 8; k0 < H; k0 += 256) {
            float wgf[8], wuf[8];
            float sg = 1.0f, su = 1.0f;
            if (int8) {
                load_chunk<true>(rg, k0, wgf);
                load_chunk<true>(ru, k0, wuf);
                sg = sbase[(size_t)pg * (H / gsz) + k0 / gsz];
                su = sbase[(size_t)pu * (H / gsz) + k0 / gsz];
            } else {
                load_chunk<false>(rg, k0, wgf);
                load_chunk<false>(ru, k0, wuf);
            }
#pragma unroll
            for (int q = 0; q < kMaxB; ++q) {
                if (q < c) {
                    const float* xq = xs + q * H + k0;
                    if (int8) {
                        ag[q] = __fmaf_rn(sg, dot8(wgf, xq), ag[q]);
                        au[q] = __fmaf_rn(su, dot8(wuf, xq), au[q]);
                    } else {
                        ag[q] = __fadd_rn(ag[q], dot8(wgf, xq));
                        au[q] = __fadd_rn(au[q], dot8(wuf, xq));
                    }
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) {
            if (q < c) {
                const float g = warp_sum_butterfly(ag[q]);
                const float u = warp_sum_butterfly(au[q]);
                if (lane == 0) a.h[(size_t)es.pair[q] * I + n] = silu(g) * u;
            }
        }
    }
}

// ---- down ---------------------------------------------------------------------------------
template <bool kRoutedInt8>
__global__ void __launch_bounds__(kDecWarps * 32)
decode_down_kernel(DecodeArgs a) {
    extern __shared__ float hs[];  // [count][I]
    __shared__ ExpertSlot es;
    if (threadIdx.x == 0) resolve_slot(es, blockIdx.y, a);
    __syncthreads();
    if (!es.valid) return;
    const int H = a.H, I = a.I, c = es.count;
    for (int i = threadIdx.x; i < c * I; i += blockDim.x) {
        const int ci = i / I;
        hs[i] = a.h[(size_t)es.pair[ci] * I + (i - ci * I)];
    }
    __syncthreads();
    const bool int8 = kRoutedInt8 && !es.shared;
    const void* wbase;
    const float* sbase = nullptr;
    if (es.shared) {
        wbase = a.w2_shared + (size_t)es.expert * H * I;
    } else if (kRoutedInt8) {
        wbase = reinterpret_cast<const int8_t*>(a.w2) + (size_t)es.expert * H * I;
        sbase = a.s2 + (size_t)es.expert * H * (I / a.G);
    } else {
        wbase = reinterpret_cast<const uint16_t*>(a.w2) + (size_t)es.expert * H * I;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gsz = a.G;
    for (int i = 0; i < kDecRowsPerWarp; ++i) {
        const int j = blockIdx.x * kDecRowsPerCta + warp * kDecRowsPerWarp + i;
        if (j >= H) break;
        const size_t esz = int8 ? 1 : 2;
        const char* rw = reinterpret_cast<const char*>(wbase) + (size_t)j * I * esz;
        float acc[kMaxB];
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) acc[q] = 0.0f;
        for (int k0 = lane * 8; k0 < I; k0 += 256) {
            float wf[8];
            float sc = 1.0f;
            if (int8) {
                load_chunk<true>(rw, k0, wf);
                sc = sbase[(size_t)j * (I / gsz) + k0 / gsz];
            } else {
                load_chunk<false>(rw, k0, wf);
            }
#pragma unroll
            for (int q = 0; q < kMaxB; ++q) {
                if (q < c) {
                    const float d = dot8(wf, hs + q * I + k0);
                    acc[q] = int8 ? __fmaf_rn(sc, d, acc[q]) : __fadd_rn(acc[q], d);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) {
            if (q < c) {
                const float v = warp_sum_butterfly(acc[q]);
                if (lane == 0) a.y[(size_t)es.pair[q] * H + j] = v;
            }
        }
    }
}

// ---- combine ------------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
decode_combine_kernel(DecodeArgs a) {
    const int t = blockIdx.x;
    const int kB = a.topk * a.B;
    for (int j = threadIdx.x; j < a.H; j += blockDim.x) {
        float acc = 0.0f;
        for (int s = 0; s < a.topk; ++s) {
            const int p = t * a.topk + s;
            acc = __fmaf_rn(a.wts[p], a.y[(size_t)p * a.H + j], acc);
        }
        for (int q = 0; q < a.S; ++q) acc = __fadd_rn(acc, a.y[(size_t)(kB + q * a.B + t) * a.H + j]);
        a.out[(size_t)t * a.H + j] = acc;
    }
}

cudaError_t launch_decode_experts(const DecodeArgs& a, cudaStream_t st) {
    const int slots = a.S + a.topk * a.B;
    {
        const size_t smem = sizeof(float) * (size_t)a.B * a.H;
        dim3 grid((a.I + kDecRowsPerCta - 1) / kDecRowsPerCta, slots);
        auto k = a.int8 ? decode_gate_up_kernel<true> : decode_gate_up_kernel<false>;
        cudaError_t err = ensure_smem_optin(reinterpret_cast<const void*>(k), smem);
        if (err != cudaSuccess) return err;
        k<<<grid, kDecWarps * 32, smem, st>>>(a);
    }
    {
        const size_t smem = sizeof(float) * (size_t)a.B * a.I;
        dim3 grid((a.H + kDecRowsPerCta - 1) / kDecRowsPerCta, slots);
        auto k = a.int8 ? decode_down_kernel<true> : decode_down_kernel<false>;
        cudaError_t err = ensure_smem_optin(reinterpret_cast<const void*>(k), smem);
        if (err != cudaSuccess) return err;
        k<<<grid, kDecWarps * 32, smem, st>>>(a);
    }
    decode_combine_kernel<<<a.B, 256, 0, st>>>(a);
    return cudaGetLastError();
}

}  // namespace uocr
