// Prefill MoE sublayer (MoE.__call__, unlimited_ocr_max/decoder.py:657-667; the accelerator path
// _routed_native, decoder.py:606-614, which routes through moe_create_indices +
// grouped_matmul_ragged): tokens are permuted into expert-contiguous rows and the expert
// products run as grouped GEMMs on the tcgen05 tensor cores (bf16 operands, fp32 accumulate).
//
//   route      route.cu (bit-exact gate)
//   permute    counting sort of the T*k (token, slot) entries by expert, stable in entry order
//              (chunk histograms -> scan -> warp-match ranks), then the rows cast to bf16:
//              xperm[p] = bf16(x[token of p]); rows [kT, (k+1)T) hold bf16(x) in token order, the
//              A operand of both shared experts
//   GEMM1      per group (64 routed experts + S shared): [rows, H] x w13[e]^T -> 2I packed gate|up
//              columns, SwiGLU in the epilogue -> h[rows, I] bf16
//   GEMM2      per group: [rows, I] x w2[e]^T -> y[rows, H], rounded to bf16
//   combine    out[t] = sum_s w[t,s] * y[dest(t,s)] + sum_q y[shared q, t] (fixed order)
//
// GEMM: persistent CTAs, one per SM; warp 0 issues TMA loads of A (128 x 64) and B (256 x 64)
// tiles into a 4-stage shared-memory ring (128-byte swizzle); warp 1 allocates 512 TMEM columns
// and one of its threads issues tcgen05.mma (M=128, N=256, K=16 per instruction) into one of
// two TMEM accumulators; warps 2-5 drain the other accumulator (tcgen05.ld), so the epilogue
// of one tile overlaps the MMAs of the next. Rows of a tile past its group's end are computed
// and discarded. No TMA or bulk load uses cluster multicast (each CTA loads its own tiles); the
// CTA-pair GEMM's MMA-completion commit signals both CTAs' mbarriers with one multicast arrival.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

#include <cuda_bf16.h>

#include <cstdlib>
#include <cstring>
#include "kernels.h"
#include "layout.h"
#include "sm100.cuh"

namespace uocr {

// ======================================================================================
// permute
// ======================================================================================
constexpr int kChunk = 256;  // entries per histogram chunk (one CTA, one thread each)

// Entry q (row q / topk) takes part: always, or (expert-parallel peer mode) when its row lies inside
// the valid part of its source slot, rows [slot * cap, slot * cap + slot_counts[slot]).
UOCR_DEV bool entry_in_slot(int q, int topk, const int* slot_counts, int cap) {
    if (!slot_counts) return true;
    const int row = q / topk;
    return row - (row / cap) * cap < slot_counts[row / cap];
}

__global__ void __launch_bounds__(kChunk) prefill_hist_kernel(const int32_t* __restrict__ ids, int n, int E, int topk,
                                                              const int* __restrict__ slot_counts, int cap,
                                                              int* __restrict__ chunk_counts) {
    __shared__ int hist[64];
    if (threadIdx.x < 64) hist[threadIdx.x] = 0;
    __syncthreads();
    const int q = blockIdx.x * kChunk + threadIdx.x;
    if (q < n && entry_in_slot(q, topk, slot_counts, cap) && ids[q] >= 0)
        atomicAdd(&hist[clamp_expert(ids[q], E)], 1);  // < 0: no expert for the entry
    __syncthreads();
    if (threadIdx.x < 64) chunk_counts[blockIdx.x * 64 + threadIdx.x] = hist[threadIdx.x];
}

// One CTA: per expert, exclusive prefix of the chunk histograms; the group tables of both GEMMs.
// Thread (part, e): expert e over a 1/kScanParts slice of the chunks (the slices' loads in flight at
// once), the slices' sums combined per expert, then the experts' prefix by two warp scans.
constexpr int kScanThreads = 1024, kScanParts = kScanThreads / 64;
__global__ void __launch_bounds__(kScanThreads) prefill_scan_kernel(const int* __restrict__ chunk_counts, int nchunks,
                                                                    int E, int S, int T, int topk,
                                                                    int* __restrict__ chunk_base,
                                                                    PrefillPlan* __restrict__ plan1,
                                                                    PrefillPlan* __restrict__ plan2,
                                                                    int* __restrict__ n_valid) {
    // n_valid[0]: routed entries with an expert; n_valid[32 + e]: entries of expert e
    __shared__ int psum[kScanParts][64];
    __shared__ int total[64];
    __shared__ int base[65];
    __shared__ int half0;  // experts 0-31's entries
    const int e = threadIdx.x & 63, part = threadIdx.x >> 6, lane = threadIdx.x & 31;
    const int per = (nchunks + kScanParts - 1) / kScanParts;
    const int c0 = min(nchunks, part * per), c1 = min(nchunks, c0 + per);
    int sum = 0;
    if (e < E)
        for (int c = c0; c < c1; ++c) sum += chunk_counts[c * 64 + e];
    psum[part][e] = sum;
    __syncthreads();
    int tot = 0, incl = 0;
    if (threadIdx.x < 64) {
        for (int q = 0; q < kScanParts; ++q) tot += psum[q][e];
        total[e] = tot;
        n_valid[32 + e] = tot;
        incl = tot;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += v;
        }
        if (e == 31) half0 = incl;
    }
    __syncthreads();
    if (threadIdx.x < 64) {
        const int excl = incl - tot + (e >= 32 ? half0 : 0);
        base[e] = excl;
        if (e == 63) {
            base[64] = excl + tot;
            *n_valid = excl + tot;  // routed entries with an expert: rows [0, n) of the permuted A
        }
    }
    __syncthreads();
    if (e < E) {
        int acc = base[e];
        for (int q = 0; q < part; ++q) acc += psum[q][e];
        for (int c = c0; c < c1; ++c) {
            chunk_base[c * 64 + e] = acc;
            acc += chunk_counts[c * 64 + e];
        }
    }
    if (threadIdx.x == 0) {
        const int kT = topk * T;
        int ng = 0, mt = 0;
        for (int g = 0; g < E + S; ++g) {
            PrefillGroup G1, G2;
            if (g < E) {
                G1.a_base = base[g]; G1.out_base = base[g]; G1.rows = total[g]; G1.wrow0 = g; G1.shared = 0;
                G2 = G1;
            } else {
                const int q = g - E;
                G1.a_base = kT; G1.out_base = kT + q * T; G1.rows = T; G1.wrow0 = q; G1.shared = 1;
                G2.a_base = kT + q * T; G2.out_base = kT + q * T; G2.rows = T; G2.wrow0 = q; G2.shared = 1;
            }
            if (G1.rows == 0) continue;
            plan1->mtile_prefix[ng] = mt;
            plan2->mtile_prefix[ng] = mt;
            plan1->g[ng] = G1;
            plan2->g[ng] = G2;
            mt += (G1.rows + 127) / 128;
            ++ng;
        }
        plan1->mtile_prefix[ng] = mt;
        plan2->mtile_prefix[ng] = mt;
        plan1->ngroups = ng;
        plan2->ngroups = ng;
    }
}

// Rank of each entry among the entries of its expert (stable in entry order) -> destination row.
__global__ void __launch_bounds__(kChunk) prefill_scatter_kernel(const int32_t* __restrict__ ids, int n, int E,
                                                                 int topk, const int* __restrict__ slot_counts,
                                                                 int cap, const int* __restrict__ chunk_base,
                                                                 int* __restrict__ dest, int* __restrict__ src_tok) {
    __shared__ int wcount[kChunk / 32][64];
    const int q = blockIdx.x * kChunk + threadIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < (kChunk / 32) * 64; i += kChunk) (&wcount[0][0])[i] = 0;
    __syncthreads();
    const int e = (q < n && entry_in_slot(q, topk, slot_counts, cap) && ids[q] >= 0) ? clamp_expert(ids[q], E) : -1;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(same & ((1u << lane) - 1u));
    if (e >= 0 && rank_in_warp == 0) wcount[warp][e] = __popc(same);
    __syncthreads();
    if (e >= 0) {
        int before = 0;
        for (int w = 0; w < warp; ++w) before += wcount[w][e];
        const int p = chunk_base[blockIdx.x * 64 + e] + before + rank_in_warp;
        dest[q] = p;
        src_tok[p] = q / topk;
    } else if (q < n) {
        dest[q] = -1;
    }
}

// xperm[p] = bf16(x[src_tok[p]]) for p < n_valid; with shared experts also xperm[kT + t] =
// bf16(x[t]). x is fp32 (converted) or already bf16 (copied). One warp per row.
__global__ void __launch_bounds__(256) prefill_gather_kernel(const float* __restrict__ x, const uint16_t* __restrict__ xb,
                                                             int T, int H, int kT, int shared,
                                                             const int* __restrict__ n_valid,
                                                             const int* __restrict__ src_tok,
                                                             uint16_t* __restrict__ xperm) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= kT + (shared ? T : 0)) return;
    if (row < kT && row >= *n_valid) return;
    const int t = row < kT ? src_tok[row] : row - kT;
    uint16_t* dst = xperm + (size_t)row * H;
    if (xb) {
        const uint16_t* src = xb + (size_t)t * H;
        for (int k = lane * 8; k < H; k += 256)
            *reinterpret_cast<uint4*>(dst + k) = *reinterpret_cast<const uint4*>(src + k);
        return;
    }
    const float* src = x + (size_t)t * H;
    for (int k0 = lane * 8; k0 < H; k0 += 4 * 256) {
        float4 a[4], b[4];  // up to four 8-element steps per lane, loads issued before the stores
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = k0 + u * 256;
            if (k < H) {
                a[u] = *reinterpret_cast<const float4*>(src + k);
                b[u] = *reinterpret_cast<const float4*>(src + k + 4);
            }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int k = k0 + u * 256;
            if (k < H) {
                uint4 o;
                o.x = (uint32_t)f32_to_bf16_rne(a[u].x) | ((uint32_t)f32_to_bf16_rne(a[u].y) << 16);
                o.y = (uint32_t)f32_to_bf16_rne(a[u].z) | ((uint32_t)f32_to_bf16_rne(a[u].w) << 16);
                o.z = (uint32_t)f32_to_bf16_rne(b[u].x) | ((uint32_t)f32_to_bf16_rne(b[u].y) << 16);
                o.w = (uint32_t)f32_to_bf16_rne(b[u].z) | ((uint32_t)f32_to_bf16_rne(b[u].w) << 16);
                *reinterpret_cast<uint4*>(dst + k) = o;
            }
        }
    }
}

// int8 items (layout.h) -> the bf16 row-block layout [row block][K / 64 atoms][128 rows][128 B]:
// each bf16 element is bf16_rne(f32(q) * scale), int8_dequant_expert's bits
// (kernels/moe_int8.mojo:330-340). Thread: one 16-byte int8 chunk (16 elements) of four rows r,
// r + 32, r + 64, r + 96 (the four loads issued first; a warp's loads are whole 128-byte row
// segments), each to two 16-byte bf16 chunks. `atoms` int8 atoms per item (the last item of a row
// block possibly shorter). Row blocks of experts that received no rows (`expert_rows`, from the
// scan) are skipped: their bf16 copy is never read.
__global__ void __launch_bounds__(256) prefill_dequant_kernel(const unsigned char* __restrict__ w, long nrb, int K,
                                                              int atoms, int rb_per_expert,
                                                              const int* __restrict__ expert_rows,
                                                              unsigned char* __restrict__ out) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int nk16 = K / 16;
    const long per_rb = 32L * nk16;
    if (i >= nrb * per_rb) return;
    const long rb = i / per_rb;
    if (expert_rows[rb / rb_per_expert] == 0) return;
    const int rem = (int)(i - rb * per_rb), rq = rem / nk16, k = 16 * (rem - rq * nk16);
    // items of `atoms` atoms of 128 elements, the last one possibly shorter (layout.h)
    const int ik = atoms * 128, ki = k / ik, a = (k % ik) / 128, c = k % 128;
    const int nitems = (K / 128 + atoms - 1) / atoms, left = K / 128 - ki * atoms;
    const int here = left < atoms ? left : atoms;  // atoms of this item
    const size_t rb_bytes = (size_t)(nitems - 1) * item_bytes(atoms, true) + item_bytes((K / 128) - (nitems - 1) * atoms, true);
    const unsigned char* item = w + (size_t)rb * rb_bytes + (size_t)ki * item_bytes(atoms, true);
    const float* scl = reinterpret_cast<const float*>(item + (size_t)here * kAtomBytes) + a * kRowBlock;
    uint4 v[4];
    float sc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int r = rq + 32 * j;
        v[j] = *reinterpret_cast<const uint4*>(item + (size_t)a * kAtomBytes + atom_offset(r, c));
        sc[j] = scl[r];
    }
    unsigned char* dst = out + ((size_t)rb * (K / 64) + k / 64) * kAtomBytes;
    const int c2 = (k % 64) * 2;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int r = rq + 32 * j;
        float f0[8], f1[8];
        unpack_s8x8(v[j].x, v[j].y, f0);
        unpack_s8x8(v[j].z, v[j].w, f1);
        uint32_t o[8];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            o[q] = (uint32_t)f32_to_bf16_rne(__fmul_rn(f0[2 * q], sc[j])) |
                   ((uint32_t)f32_to_bf16_rne(__fmul_rn(f0[2 * q + 1], sc[j])) << 16);
            o[4 + q] = (uint32_t)f32_to_bf16_rne(__fmul_rn(f1[2 * q], sc[j])) |
                       ((uint32_t)f32_to_bf16_rne(__fmul_rn(f1[2 * q + 1], sc[j])) << 16);
        }
        *reinterpret_cast<uint4*>(dst + atom_offset(r, c2)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(dst + atom_offset(r, c2 + 16)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

// out[t][j] (+)= sum_s w[t,s] * y[dest[t*k+s]][j] (entries without an expert skipped)
//              + sum_q y[kT + q*T + t][j]                     (S shared experts)
// (y is bf16; each thread 8 columns, the rows' 16-byte loads issued before the sums)
__global__ void __launch_bounds__(256) prefill_combine_kernel(const uint16_t* __restrict__ y, const float* __restrict__ wts,
                                                              const int* __restrict__ dest, int T, int H, int topk,
                                                              int S, int accumulate, float* __restrict__ out) {
    const int t = blockIdx.x;
    const int kT = topk * T;
    for (int j = threadIdx.x * 8; j < H; j += blockDim.x * 8) {
        float acc[8];
        if (accumulate) {
            const float4 a0 = *reinterpret_cast<const float4*>(out + (size_t)t * H + j);
            const float4 a1 = *reinterpret_cast<const float4*>(out + (size_t)t * H + j + 4);
            acc[0] = a0.x; acc[1] = a0.y; acc[2] = a0.z; acc[3] = a0.w;
            acc[4] = a1.x; acc[5] = a1.y; acc[6] = a1.z; acc[7] = a1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
        }
        for (int s = 0; s < topk; ++s) {
            const int d = dest[t * topk + s];
            if (d < 0) continue;
            const float w = wts[t * topk + s];
            float v[8];
            unpack_bf16x8(*reinterpret_cast<const uint4*>(y + (size_t)d * H + j), v);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(w, v[i], acc[i]);
        }
        for (int q = 0; q < S; ++q) {
            float v[8];
            unpack_bf16x8(*reinterpret_cast<const uint4*>(y + (size_t)(kT + q * T + t) * H + j), v);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], v[i]);
        }
        *reinterpret_cast<float4*>(out + (size_t)t * H + j) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(out + (size_t)t * H + j + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

// Expert-parallel peer mode: received row n = q * cap + r (source q, position r) of the valid part
// of its slot -> bf16(sum_s w[n,s] * y[dest[n*k+s]]) (the same fp32 fma chain from +0 as
// prefill_combine_kernel, then rounded to nearest even) stored straight into rank q's exchange
// buffer, partial slot `rank`, row r. The grid's last CTA then sets every rank q's part_flag[rank]
// to (epoch << 1) | fail, fail when slot q's rows were not processed (its wait failed, or its count
// was refused) or a bounded wait of these products gave up (`status`).
__global__ void __launch_bounds__(256) ep_partials_kernel(const uint16_t* __restrict__ y, const float* __restrict__ wts,
                                                          const int* __restrict__ dest, int topk, EpPeers P,
                                                          size_t part_off, size_t sig_off,
                                                          const int* __restrict__ slot_counts,
                                                          const int* __restrict__ slot_fail, const uint32_t* status,
                                                          unsigned int* __restrict__ done) {
    const int n = blockIdx.x, H = P.H;
    const int q = n / P.cap, r = n - q * P.cap;
    if (r < slot_counts[q]) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(P.buf[q] + part_off) + ((size_t)P.rank * P.cap + r) * H;
        for (int j = threadIdx.x * 8; j < H; j += blockDim.x * 8) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
            for (int s = 0; s < topk; ++s) {
                const int d = dest[n * topk + s];
                if (d < 0) continue;
                const float w = wts[n * topk + s];
                float v[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(y + (size_t)d * H + j), v);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc[i] = __fmaf_rn(w, v[i], acc[i]);
            }
            uint4 o;
            o.x = (uint32_t)f32_to_bf16_rne(acc[0]) | ((uint32_t)f32_to_bf16_rne(acc[1]) << 16);
            o.y = (uint32_t)f32_to_bf16_rne(acc[2]) | ((uint32_t)f32_to_bf16_rne(acc[3]) << 16);
            o.z = (uint32_t)f32_to_bf16_rne(acc[4]) | ((uint32_t)f32_to_bf16_rne(acc[5]) << 16);
            o.w = (uint32_t)f32_to_bf16_rne(acc[6]) | ((uint32_t)f32_to_bf16_rne(acc[7]) << 16);
            *reinterpret_cast<uint4*>(dst + j) = o;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0u;  // for the next call
            __threadfence_system();
            const unsigned long long any = *reinterpret_cast<const volatile uint32_t*>(status) != 0u ? 1ull : 0ull;
            for (int p = 0; p < P.world; ++p) {
                EpSig* sig = reinterpret_cast<EpSig*>(P.buf[p] + sig_off) + P.rank;
                const unsigned long long f = any | (slot_fail[p] ? 1ull : 0ull);
                st_release_sys_u64(&sig->part_flag, (P.epoch << 1) | f);
            }
        }
    }
}

// ======================================================================================
// grouped GEMM on tcgen05
// ======================================================================================
constexpr int kBM = 128, kBN = 256, kBK = 64;
constexpr int kGStages = 4;
constexpr uint32_t kATile = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kBTile = kBN * kBK * 2;  // 32 KB
constexpr int kGemmThreads = 192;           // producer, MMA, 4 epilogue warps
constexpr uint32_t kTmemCols = 512;         // two 256-column accumulators

enum GemmEpi : int { kEpiSwiGLU = 0, kEpiY = 1 };  // GEMM1: SwiGLU -> bf16 h; GEMM2: bf16 y
constexpr uint32_t kPlanBytes = (sizeof(PrefillPlan) + 127) & ~127u;

// byte offset of 16-byte chunk `ch` of row `row` in a 32 x 128-byte staging buffer
UOCR_DEV uint32_t stage_off(int row, int ch) { return (uint32_t)row * 128u + ((uint32_t)(ch ^ (row & 7)) << 4); }
UOCR_DEV void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
UOCR_DEV uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}

struct GemmSmem {
    uint64_t full[kGStages], empty[kGStages], tfull[2], tempty[2], done;
    uint32_t tmem_base;
    int abort_flag;
};

UOCR_DEV void gemm_decode_tile(const PrefillPlan& P, int NT, int tile, int& g, int& mloc, int& n) {
    const int mt = tile / NT;
    n = tile - mt * NT;
    g = 0;
    while (P.mtile_prefix[g + 1] <= mt) ++g;
    mloc = mt - P.mtile_prefix[g];
}

// Bounded single-thread mbarrier wait that also honours the CTA abort flag.
UOCR_DEV bool gwait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            set_status(status, kStatusWaitTimeout);
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

// Epilogue of one 128 x kBN accumulator (TMEM columns from `taddr`, this warp's 32 lanes): the
// SwiGLU pairs to bf16 h, or the fp32 y, for the tile's rows below rows_valid.
// SiLU for the GEMM1 epilogue: a / (1 + e^-a) with the fast exponential and division intrinsics
// (h is rounded to bf16 right after; the limits hold: e^-a = inf gives -0, e^-a = 0 gives a).
UOCR_DEV float silu_fast(float a) { return __fdividef(a, 1.0f + __expf(-a)); }

// Epilogue of one 128 x kBN accumulator (TMEM columns from `taddr`, this warp's 32 lanes): the
// SwiGLU pairs to bf16 h, or the fp32 y, for the tile's rows below rows_valid. The TMEM load of
// chunk c + 1 is in flight while chunk c is processed. Rows leave through the warp's staging
// buffer (32 rows x 128 B, chunks XOR-swizzled by row) as 16-byte stores covering 4 whole
// 128-byte row segments per instruction.
template <int kEpi>
UOCR_DEV void gemm_epilogue_tile(uint32_t taddr, const PrefillGroup& G, int mloc, int n, int rows_valid, void* out,
                                 int out_ld, uint32_t stage, int quarter, int lane) {
    constexpr int kChunks = kBN / 32;
    const size_t tile_row0 = (size_t)G.out_base + (size_t)mloc * kBM + quarter * 32;
    uint32_t r[2][32];
    tmem_ld_32x32b_x32(taddr, r[0]);
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        tmem_wait_ld_tie(r[c & 1]);
        if (c + 1 < kChunks) tmem_ld_32x32b_x32(taddr + (c + 1) * 32, r[(c + 1) & 1]);
        const uint32_t* rc = r[c & 1];
        if (kEpi == kEpiSwiGLU) {
            // tile columns in groups of 16: 8 gate rows then the same 8 up rows, so columns
            // [32c, 32c + 32) give h columns [16c, 16c + 16) of this tile's 128
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c0 = (2 * i) / 8 * 16 + (2 * i) % 8;  // gate column of h column 2i
                const float g0 = __uint_as_float(rc[c0]), g1 = __uint_as_float(rc[c0 + 1]);
                const float u0 = __uint_as_float(rc[c0 + 8]), u1 = __uint_as_float(rc[c0 + 9]);
                const __nv_bfloat162 hv = __floats2bfloat162_rn(silu_fast(g0) * u0, silu_fast(g1) * u1);
                pk[i] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            const int q = 2 * (c & 3);
            st_shared_v4(stage + stage_off(lane, q), pk[0], pk[1], pk[2], pk[3]);
            st_shared_v4(stage + stage_off(lane, q + 1), pk[4], pk[5], pk[6], pk[7]);
            if ((c & 3) == 3) {
                __syncwarp();
                uint16_t* h0 = reinterpret_cast<uint16_t*>(out) + (size_t)n * (kBN / 2) + (c >> 2) * 64;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int row = i * 4 + (lane >> 3), ch = lane & 7;
                    const uint4 v = ld_shared_v4(stage + stage_off(row, ch));
                    if (quarter * 32 + row < rows_valid)
                        *reinterpret_cast<uint4*>(h0 + (tile_row0 + row) * out_ld + ch * 8) = v;
                }
                __syncwarp();
            }
        } else {
            // y rounded to bf16: chunk c's 32 columns are half a 128-byte row segment, written out
            // every second chunk
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const __nv_bfloat162 yv = __floats2bfloat162_rn(__uint_as_float(rc[2 * i]), __uint_as_float(rc[2 * i + 1]));
                pk[i] = *reinterpret_cast<const uint32_t*>(&yv);
            }
            const int q = 4 * (c & 1);
#pragma unroll
            for (int v = 0; v < 4; ++v)
                st_shared_v4(stage + stage_off(lane, q + v), pk[4 * v], pk[4 * v + 1], pk[4 * v + 2], pk[4 * v + 3]);
            if (c & 1) {
                __syncwarp();
                uint16_t* y0 = reinterpret_cast<uint16_t*>(out) + (size_t)n * kBN + (c >> 1) * 64;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int row = i * 4 + (lane >> 3), ch = lane & 7;
                    const uint4 v = ld_shared_v4(stage + stage_off(row, ch));
                    if (quarter * 32 + row < rows_valid)
                        *reinterpret_cast<uint4*>(y0 + (tile_row0 + row) * out_ld + ch * 8) = v;
                }
                __syncwarp();
            }
        }
    }
}

template <int kEpi>
__global__ void __launch_bounds__(kGemmThreads, 1)
grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmBs, const PrefillPlan* __restrict__ plan_g, int NT, int KT,
                    int b_rows_per_group, void* __restrict__ out, int out_ld, uint32_t* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + kGStages * kATile;
    GemmSmem* gs = reinterpret_cast<GemmSmem*>(smem + kGStages * (kATile + kBTile));
    PrefillPlan* P = reinterpret_cast<PrefillPlan*>(reinterpret_cast<uint8_t*>(gs) + 256);
    // epilogue staging: 4 KB per epilogue warp (32 rows x 128 B, 16-byte chunks XOR-swizzled by row)
    const uint32_t stage_base = smem_addr(reinterpret_cast<uint8_t*>(P) + kPlanBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    volatile int* abort_flag = &gs->abort_flag;

    for (int i = tid; i < (int)(sizeof(PrefillPlan) / 4); i += blockDim.x)
        reinterpret_cast<int*>(P)[i] = reinterpret_cast<const int*>(plan_g)[i];
    if (tid == 0) {
        for (int s = 0; s < kGStages; ++s) {
            mbar_init(&gs->full[s], 1);
            mbar_init(&gs->empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&gs->tfull[a], 1);
            mbar_init(&gs->tempty[a], 4);
        }
        mbar_init(&gs->done, 1);
        gs->abort_flag = 0;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmBs);
    }
    if (warp == 1) tmem_alloc(&gs->tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = gs->tmem_base;
    const int total = P->mtile_prefix[P->ngroups] * NT;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer ----------------
            int s = 0;
            uint32_t round = 0;
            for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
                int g, mloc, n;
                gemm_decode_tile(*P, NT, tile, g, mloc, n);
                const PrefillGroup& G = P->g[g];
                const int a_row = G.a_base + mloc * kBM;
                const int b_row = G.wrow0 * b_rows_per_group + n * kBN;
                const CUtensorMap* mb = G.shared ? &tmBs : &tmB;
                for (int kt = 0; kt < KT; ++kt) {
                    if (round > 0 && !gwait(&gs->empty[s], (round - 1) & 1, abort_flag, status)) break;
                    mbar_arrive_expect_tx(&gs->full[s], kATile + kBTile);
                    tma_load_2d(sA + s * kATile, &tmA, kt * kBK, a_row, &gs->full[s]);
                    tma_load_4d(sB + s * kBTile, mb, 0, 0, kt, b_row / kRowBlock, &gs->full[s]);
                    if (++s == kGStages) { s = 0; ++round; }
                }
            }
            // copies still in flight complete before the CTA may exit
            for (int i = 0; i < kGStages; ++i) {
                int ss = s - 1 - i;
                uint32_t rr = round;
                if (ss < 0) { ss += kGStages; if (rr == 0) break; --rr; }
                mbar_wait(&gs->full[ss], rr & 1, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (lane == 0) {
            // ---------------- MMA issuer ----------------
            constexpr uint32_t idesc = umma_idesc_bf16(kBM, kBN);
            int s = 0, acc = 0;
            uint32_t round = 0, around = 0;
            bool issued = false;
            for (int tile = blockIdx.x; tile < total && !*abort_flag; tile += gridDim.x) {
                if (around > 0 && !gwait(&gs->tempty[acc], (around - 1) & 1, abort_flag, status)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)acc * kBN;
                bool ok = true;
                for (int kt = 0; kt < KT; ++kt) {
                    if (!gwait(&gs->full[s], round & 1, abort_flag, status)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = umma_desc_sw128(smem_addr(sA + s * kATile));
                    const uint64_t bd = umma_desc_sw128(smem_addr(sB + s * kBTile));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_f16(tmem_d, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
                    issued = true;
                    umma_commit(&gs->empty[s]);
                    if (++s == kGStages) { s = 0; ++round; }
                }
                if (!ok) break;
                umma_commit(&gs->tfull[acc]);
                if (++acc == 2) { acc = 0; ++around; }
            }
            if (issued) {
                // every MMA of this CTA has completed before TMEM is released
                umma_commit(&gs->done);
                mbar_wait(&gs->done, 0, nullptr);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: warps 2..5 own TMEM lanes 32*(warp%4) .. +31 ----------------
        const int quarter = warp & 3;
        const uint32_t stage = stage_base + (uint32_t)(warp - 2) * 4096u;
        int acc = 0;
        uint32_t around = 0;
        for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
            int g, mloc, n;
            gemm_decode_tile(*P, NT, tile, g, mloc, n);
            const PrefillGroup& G = P->g[g];
            if (!mbar_wait_warp(&gs->tfull[acc], around & 1, abort_flag, status)) break;
            tc_fence_after();
            const int rows_valid = min(kBM, G.rows - mloc * kBM);
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)acc * kBN;
            gemm_epilogue_tile<kEpi>(taddr, G, mloc, n, rows_valid, out, out_ld, stage, quarter, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&gs->tempty[acc]);
            if (++acc == 2) { acc = 0; ++around; }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// ---- CTA-pair variant: 256 x 256 tiles on tcgen05.mma.cta_group::2 -------------------------
// A cluster of two CTAs computes a pair tile: m-tiles 2p (CTA 0) and 2p + 1 (CTA 1) of one group
// against a 256-column slice of its weights. Each CTA stages its own 128 A rows and its half
// (128 rows) of the B slice per K step, 32 KB instead of the single-CTA kernel's 48 KB for the
// same flops per CTA, so six stages fit. Both CTAs' TMA loads complete on CTA 0's `full`
// barrier (CTA 0 expects the bytes of both); CTA 0's MMA thread issues the pair MMAs and
// commits to the `empty` / `tfull` barriers of both CTAs. Each CTA drains its own accumulator
// (its 128 rows, all 256 columns) and arrives on CTA 0's `tempty` (8 arrivals: 4 warps x 2
// CTAs). A group with an odd number of m-tiles leaves the second CTA of its last pair tile
// without rows: it computes and discards them. Every wait is bounded; every path reaches the
// closing cluster barrier.
constexpr int kPStages = 6;
constexpr uint32_t kBHalfTile = 128 * kBK * 2;  // 16 KB

struct PairSmem {
    uint64_t full[kPStages], empty[kPStages], tfull[2], tempty[2], done;
    uint32_t tmem_base;
    int abort_flag;
    int pair_prefix[kPrefillMaxGroups + 1];
};

UOCR_DEV void pair_decode_tile(const int* pp, int NT, int tile, int& g, int& mp, int& n) {
    const int pt = tile / NT;
    n = tile - pt * NT;
    g = 0;
    while (pp[g + 1] <= pt) ++g;
    mp = pt - pp[g];
}

template <int kEpi>
__global__ void __launch_bounds__(kGemmThreads, 1)
grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmBs, const PrefillPlan* __restrict__ plan_g, int NT,
                         int KT, int b_rows_per_group, void* __restrict__ out, int out_ld, uint32_t* status) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + kPStages * kATile;
    PairSmem* ps = reinterpret_cast<PairSmem*>(smem + kPStages * (kATile + kBHalfTile));
    PrefillPlan* P = reinterpret_cast<PrefillPlan*>(reinterpret_cast<uint8_t*>(ps) + ((sizeof(PairSmem) + 127) & ~127u));
    const uint32_t stage_base = smem_addr(reinterpret_cast<uint8_t*>(P) + kPlanBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
    volatile int* abort_flag = &ps->abort_flag;

    for (int i = tid; i < (int)(sizeof(PrefillPlan) / 4); i += blockDim.x)
        reinterpret_cast<int*>(P)[i] = reinterpret_cast<const int*>(plan_g)[i];
    __syncthreads();
    if (tid == 0) {
        for (int st = 0; st < kPStages; ++st) {
            mbar_init(&ps->full[st], 1);
            mbar_init(&ps->empty[st], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&ps->tfull[a], 1);
            mbar_init(&ps->tempty[a], 8);
        }
        mbar_init(&ps->done, 1);
        ps->abort_flag = 0;
        ps->pair_prefix[0] = 0;
        for (int g = 0; g < P->ngroups; ++g)
            ps->pair_prefix[g + 1] = ps->pair_prefix[g] + (P->mtile_prefix[g + 1] - P->mtile_prefix[g] + 1) / 2;
        fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
        tma_prefetch_desc(&tmBs);
    }
    if (warp == 1) tmem_alloc_pair(&ps->tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers are initialised before any cross-CTA arrival
    tc_fence_after();
    const uint32_t tmem_base = ps->tmem_base;
    const int total = ps->pair_prefix[P->ngroups] * NT;

    if (warp == 0) {
        if (lane == 0) {
            // ---------------- TMA producer (both CTAs) ----------------
            int s = 0;
            uint32_t round = 0;
            for (int tile = cid; tile < total && !*abort_flag; tile += ncl) {
                int g, mp, n;
                pair_decode_tile(ps->pair_prefix, NT, tile, g, mp, n);
                const PrefillGroup& G = P->g[g];
                const int a_row = G.a_base + (2 * mp + (int)rank) * kBM;
                const int b_rb = (G.wrow0 * b_rows_per_group + n * kBN) / kRowBlock + (int)rank;
                const CUtensorMap* mb = G.shared ? &tmBs : &tmB;
                bool ok = true;
                for (int kt = 0; kt < KT; ++kt) {
                    if (round > 0 && !gwait(&ps->empty[s], (round - 1) & 1, abort_flag, status)) { ok = false; break; }
                    if (leader) mbar_arrive_expect_tx(&ps->full[s], 2 * (kATile + kBHalfTile));
                    const uint32_t lf = mapa_shared(smem_addr(&ps->full[s]), 0);
                    tma_load_2d_pair(sA + s * kATile, &tmA, kt * kBK, a_row, lf);
                    tma_load_4d_pair(sB + s * kBHalfTile, mb, 0, 0, kt, b_rb, lf);
                    if (++s == kPStages) { s = 0; ++round; }
                }
                if (!ok) break;
            }
            if (leader) {
                // every copy counted on CTA 0's barriers (both CTAs') has landed before exit
                for (int i = 0; i < kPStages; ++i) {
                    int ss = s - 1 - i;
                    uint32_t rr = round;
                    if (ss < 0) { ss += kPStages; if (rr == 0) break; --rr; }
                    mbar_wait(&ps->full[ss], rr & 1, status);
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        if (leader && lane == 0) {
            // ---------------- pair MMA issuer (CTA 0) ----------------
            constexpr uint32_t idesc = umma_idesc_bf16(2 * kBM, kBN);
            int s = 0, acc = 0;
            uint32_t round = 0, around = 0;
            bool issued = false;
            for (int tile = cid; tile < total && !*abort_flag; tile += ncl) {
                if (around > 0 && !gwait(&ps->tempty[acc], (around - 1) & 1, abort_flag, status)) break;
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t)acc * kBN;
                bool ok = true;
                for (int kt = 0; kt < KT; ++kt) {
                    if (!gwait(&ps->full[s], round & 1, abort_flag, status)) { ok = false; break; }
                    tc_fence_after();
                    const uint64_t ad = umma_desc_sw128(smem_addr(sA + s * kATile));
                    const uint64_t bd = umma_desc_sw128(smem_addr(sB + s * kBHalfTile));
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk)
                        umma_f16_pair(tmem_d, ad + 2 * kk, bd + 2 * kk, idesc, (kt | kk) != 0 ? 1u : 0u);
                    issued = true;
                    umma_commit_pair_both(&ps->empty[s]);
                    if (++s == kPStages) { s = 0; ++round; }
                }
                if (!ok) break;
                umma_commit_pair_both(&ps->tfull[acc]);
                if (++acc == 2) { acc = 0; ++around; }
            }
            if (issued) {
                // every pair MMA has completed before either CTA releases its TMEM
                umma_commit_pair_own(&ps->done);
                mbar_wait(&ps->done, 0, status);
            }
        }
        __syncwarp();
    } else {
        // ---------------- epilogue (both CTAs): warps 2..5 own TMEM lanes 32*(warp%4) .. +31 ----
        const int quarter = warp & 3;
        const uint32_t stage = stage_base + (uint32_t)(warp - 2) * 4096u;
        int acc = 0;
        uint32_t around = 0;
        for (int tile = cid; tile < total; tile += ncl) {
            int g, mp, n;
            pair_decode_tile(ps->pair_prefix, NT, tile, g, mp, n);
            const PrefillGroup& G = P->g[g];
            const int mloc = 2 * mp + (int)rank;
            if (!mbar_wait_warp(&ps->tfull[acc], around & 1, abort_flag, status)) break;
            tc_fence_after();
            const int rows_valid = min(kBM, G.rows - mloc * kBM);  // <= 0: the pair's empty half
            const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)acc * kBN;
            gemm_epilogue_tile<kEpi>(taddr, G, mloc, n, rows_valid, out, out_ld, stage, quarter, lane);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_addr(&ps->tempty[acc]), 0));
            if (++acc == 2) { acc = 0; ++around; }
        }
    }
    __syncthreads();
    cluster_sync_all();  // no cross-CTA arrival or MMA write is pending past this point
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}

// ======================================================================================
// host side
// ======================================================================================
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D bf16 [rows, cols] with a row stride of `ld` elements, box {64, box_rows}, 128-byte
// swizzle, zero fill out of bounds.
static bool make_map_bf16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
                          uint64_t ld) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {64, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The bf16 row-block weights (layout.h) as the 4-D array [nrb][K / 64][128 rows][64 elements],
// box {64, 128, 1, 2}: 256 rows (two consecutive row blocks) of one 64-element atom, already
// swizzled in memory, so copied without swizzling into a 1024-byte-aligned tile.
static bool make_map_bf16_blocks(CUtensorMap* m, const void* base, uint64_t nrb, uint64_t K, uint32_t box_blocks = 2) {
    auto fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[4] = {64, 128, K / 64, nrb};
    const cuuint64_t strides[3] = {128, (cuuint64_t)kAtomBytes, (cuuint64_t)(K / 64) * kAtomBytes};
    const cuuint32_t box[4] = {64, 128, 1, box_blocks};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

size_t gemm_smem_bytes() {
    return 1024 + kGStages * (kATile + kBTile) + 256 + kPlanBytes + 4 * 4096;
}

static cudaError_t launch_gemm(int epi, const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& Bs,
                               const PrefillPlan* plan, int NT, int KT, int b_rows_per_group, void* out, int out_ld,
                               int max_tiles, int max_ctas, uint32_t* status, cudaStream_t st) {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const size_t smem = gemm_smem_bytes();
    const void* fn = epi == kEpiSwiGLU ? reinterpret_cast<const void*>(grouped_gemm_kernel<kEpiSwiGLU>)
                                       : reinterpret_cast<const void*>(grouped_gemm_kernel<kEpiY>);
    cudaError_t err = ensure_smem_optin(fn, smem);
    if (err != cudaSuccess) return err;
    int grid = std::max(1, std::min(sms, max_tiles));
    if (max_ctas > 0) grid = std::min(grid, max_ctas);
    if (epi == kEpiSwiGLU)
        grouped_gemm_kernel<kEpiSwiGLU><<<grid, kGemmThreads, smem, st>>>(A, B, Bs, plan, NT, KT, b_rows_per_group, out,
                                                                         out_ld, status);
    else
        grouped_gemm_kernel<kEpiY><<<grid, kGemmThreads, smem, st>>>(A, B, Bs, plan, NT, KT, b_rows_per_group, out,
                                                                      out_ld, status);
    return cudaGetLastError();
}

size_t gemm_pair_smem_bytes() {
    return 1024 + kPStages * (kATile + kBHalfTile) + ((sizeof(PairSmem) + 127) & ~127u) + kPlanBytes + 4 * 4096;
}

// Pair-tile launch: clusters of 2 CTAs, as many clusters as fit at once (one CTA per SM).
static cudaError_t launch_gemm_pair(int epi, const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& Bs,
                                    const PrefillPlan* plan, int NT, int KT, int b_rows_per_group, void* out,
                                    int out_ld, int max_pair_tiles, int max_ctas, uint32_t* status, cudaStream_t st) {
    const size_t smem = gemm_pair_smem_bytes();
    const void* fn = epi == kEpiSwiGLU ? reinterpret_cast<const void*>(grouped_gemm_pair_kernel<kEpiSwiGLU>)
                                       : reinterpret_cast<const void*>(grouped_gemm_pair_kernel<kEpiY>);
    cudaError_t err = ensure_smem_optin(fn, smem);
    if (err != cudaSuccess) return err;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    static int max_clusters = 0;  // per process: the device and kernel shape do not change
    if (max_clusters == 0) {
        int dev = 0, sms = 148;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        cfg.gridDim = dim3((unsigned)(sms & ~1));
        int n = 0;
        err = cudaOccupancyMaxActiveClusters(&n, fn, &cfg);
        if (err != cudaSuccess) return err;
        if (n < 1) return cudaErrorInvalidConfiguration;
        max_clusters = n;
    }
    int clusters = std::max(1, std::min(max_clusters, max_pair_tiles));
    if (max_ctas > 0) clusters = std::max(1, std::min(clusters, max_ctas / 2));
    cfg.gridDim = dim3((unsigned)(2 * clusters));
    if (epi == kEpiSwiGLU)
        err = cudaLaunchKernelEx(&cfg, grouped_gemm_pair_kernel<kEpiSwiGLU>, A, B, Bs, plan, NT, KT, b_rows_per_group,
                                 out, out_ld, status);
    else
        err = cudaLaunchKernelEx(&cfg, grouped_gemm_pair_kernel<kEpiY>, A, B, Bs, plan, NT, KT, b_rows_per_group, out,
                                 out_ld, status);
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}

// Which grouped GEMM runs: the pair kernel when the groups are deep enough that an odd last
// m-tile per group wastes little (on average at least kPairMinRows rows per group), else the
// single-CTA kernel. UOCR_PREFILL_GEMM=pair|single overrides (diagnostics).
constexpr int kPairMinRows = 384;
static bool use_pair_gemm(long rows, int groups) {
    static int mode = -1;
    if (mode < 0) {
        const char* e = getenv("UOCR_PREFILL_GEMM");
        mode = (e && strcmp(e, "pair") == 0) ? 1 : (e && strcmp(e, "single") == 0) ? 2 : 0;
    }
    if (mode == 1) return true;
    if (mode == 2) return false;
    return groups > 0 && rows >= (long)kPairMinRows * groups;
}

PrefillLayout prefill_layout(int T, int H, int I, int E, int S, int topk, bool int8) {
    auto al = [](size_t n) { return (n + 255) & ~size_t(255); };
    PrefillLayout d{};
    const size_t kT = (size_t)topk * T;
    const size_t nchunks = (kT + kChunk - 1) / kChunk;
    size_t off = 0;
    d.status = off; off += kCtlClearBytes;  // status region (cleared whole after a failure)
    d.n_valid = off; off += 512;  // the valid-row count, then per-expert rows (from byte 128)
    d.ids = off; off += al(sizeof(int32_t) * kT);
    d.wts = off; off += al(sizeof(float) * kT);
    d.chunk_counts = off; off += al(sizeof(int) * (nchunks ? nchunks : 1) * 64);
    d.chunk_base = off; off += al(sizeof(int) * (nchunks ? nchunks : 1) * 64);
    d.plan1 = off; off += al(sizeof(PrefillPlan));
    d.plan2 = off; off += al(sizeof(PrefillPlan));
    d.dest = off; off += al(sizeof(int) * kT);
    d.src_tok = off; off += al(sizeof(int) * kT);
    d.xperm = off; off += al(sizeof(uint16_t) * (kT + T) * H);
    d.h = off; off += al(sizeof(uint16_t) * (kT + (size_t)S * T) * I);
    d.y = off; off += al(sizeof(uint16_t) * (kT + (size_t)S * T) * H);
    d.w13 = d.w2 = 0;
    if (int8) {
        d.w13 = off; off += al(sizeof(uint16_t) * (size_t)E * 2 * I * H);
        d.w2 = off; off += al(sizeof(uint16_t) * (size_t)E * H * I);
    }
    d.total = off;
    return d;
}

cudaError_t launch_prefill(const PrefillArgs& a, char* ws, const PrefillLayout& d, cudaStream_t st) {
    const int T = a.T, H = a.H, I = a.I, E = a.E, k = a.topk;
    const int S = a.use_shared ? a.S : 0;  // shared-expert groups in the GEMMs
    const int kT = k * T;
    const int nchunks = (kT + kChunk - 1) / kChunk;
    int32_t* ids = a.ids;
    float* wts = a.wts;
    int* chunk_counts = reinterpret_cast<int*>(ws + d.chunk_counts);
    int* chunk_base = reinterpret_cast<int*>(ws + d.chunk_base);
    PrefillPlan* plan1 = reinterpret_cast<PrefillPlan*>(ws + d.plan1);
    PrefillPlan* plan2 = reinterpret_cast<PrefillPlan*>(ws + d.plan2);
    int* dest = reinterpret_cast<int*>(ws + d.dest);
    int* src_tok = reinterpret_cast<int*>(ws + d.src_tok);
    int* n_valid = reinterpret_cast<int*>(ws + d.n_valid);
    uint16_t* xperm = reinterpret_cast<uint16_t*>(ws + d.xperm);
    uint16_t* h = reinterpret_cast<uint16_t*>(ws + d.h);
    uint16_t* y = reinterpret_cast<uint16_t*>(ws + d.y);
    uint32_t* status = a.status ? a.status : reinterpret_cast<uint32_t*>(ws + d.status);
    const int cap = a.peers ? a.peers->cap : 1;
    const int* slots = a.peers ? a.slot_counts : nullptr;

    cudaError_t err = cudaSuccess;
    if (a.route && k > 0) {
        err = launch_route(a.x, T, H, a.router, E, a.bias, k, ids, wts, st);
        if (err != cudaSuccess) return err;
    }
    if (nchunks > 0) prefill_hist_kernel<<<nchunks, kChunk, 0, st>>>(ids, kT, E, k, slots, cap, chunk_counts);
    prefill_scan_kernel<<<1, kScanThreads, 0, st>>>(chunk_counts, nchunks, E, S, T, k, chunk_base, plan1, plan2, n_valid);
    if (nchunks > 0)
        prefill_scatter_kernel<<<nchunks, kChunk, 0, st>>>(ids, kT, E, k, slots, cap, chunk_base, dest, src_tok);
    const int grows = kT + (S ? T : 0);
    if (grows > 0)
        prefill_gather_kernel<<<(grows + 7) / 8, 256, 0, st>>>(a.x, a.x_bf16, T, H, kT, S > 0, n_valid, src_tok, xperm);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;

    const void* w13 = a.w13;
    const void* w2 = a.w2;
    if (a.int8 && k > 0) {
        unsigned char* w13d = reinterpret_cast<unsigned char*>(ws + d.w13);
        unsigned char* w2d = reinterpret_cast<unsigned char*>(ws + d.w2);
        const long nrb13 = (long)E * (2 * I / kRowBlock), nrb2 = (long)E * (H / kRowBlock);
        const long n13 = nrb13 * 32 * (H / 16), n2 = nrb2 * 32 * (I / 16);
        prefill_dequant_kernel<<<(unsigned)((n13 + 255) / 256), 256, 0, st>>>(
            reinterpret_cast<const unsigned char*>(a.w13), nrb13, H, w13_atoms(), 2 * I / kRowBlock, n_valid + 32, w13d);
        prefill_dequant_kernel<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(
            reinterpret_cast<const unsigned char*>(a.w2), nrb2, I, kW2Atoms, H / kRowBlock, n_valid + 32, w2d);
        w13 = w13d;
        w2 = w2d;
    }
    // upper bound of m-tiles (the plan holds the exact count on the device)
    const int max_mtiles = (kT + 127) / 128 + (k > 0 ? E : 0) + S * ((T + 127) / 128);
    CUtensorMap mA1, mB1, mBs1, mA2, mB2, mBs2;
    if (!make_map_bf16(&mA1, xperm, (uint64_t)kT + T, H, kBM, H) ||
        !make_map_bf16_blocks(&mB1, w13, (uint64_t)E * 2 * I / kRowBlock, H) ||
        !make_map_bf16(&mA2, h, (uint64_t)kT + (uint64_t)S * T, I, kBM, I) ||
        !make_map_bf16_blocks(&mB2, w2, (uint64_t)E * H / kRowBlock, I))
        return cudaErrorInvalidValue;
    if (S > 0) {
        if (!make_map_bf16_blocks(&mBs1, a.w13_shared, (uint64_t)S * 2 * I / kRowBlock, H) ||
            !make_map_bf16_blocks(&mBs2, a.w2_shared, (uint64_t)S * H / kRowBlock, I))
            return cudaErrorInvalidValue;
    } else {
        mBs1 = mB1;  // no shared groups in the plan: never read
        mBs2 = mB2;
    }
    const int groups = (k > 0 ? E : 0) + S;
    if (use_pair_gemm((long)kT + (long)S * T, groups)) {
        // B slices of 128 rows (one row block) per CTA
        CUtensorMap pB1, pBs1, pB2, pBs2;
        if (!make_map_bf16_blocks(&pB1, w13, (uint64_t)E * 2 * I / kRowBlock, H, 1) ||
            !make_map_bf16_blocks(&pB2, w2, (uint64_t)E * H / kRowBlock, I, 1))
            return cudaErrorInvalidValue;
        if (S > 0) {
            if (!make_map_bf16_blocks(&pBs1, a.w13_shared, (uint64_t)S * 2 * I / kRowBlock, H, 1) ||
                !make_map_bf16_blocks(&pBs2, a.w2_shared, (uint64_t)S * H / kRowBlock, I, 1))
                return cudaErrorInvalidValue;
        } else {
            pBs1 = pB1;
            pBs2 = pB2;
        }
        const int max_pairs = max_mtiles;  // pair tiles <= m-tiles
        err = launch_gemm_pair(kEpiSwiGLU, mA1, pB1, pBs1, plan1, (2 * I) / kBN, H / kBK, 2 * I, h, I,
                               max_pairs * ((2 * I) / kBN), a.max_ctas, status, st);
        if (err != cudaSuccess) return err;
        err = launch_gemm_pair(kEpiY, mA2, pB2, pBs2, plan2, H / kBN, I / kBK, H, y, H, max_pairs * (H / kBN),
                               a.max_ctas, status, st);
        if (err != cudaSuccess) return err;
    } else {
        err = launch_gemm(kEpiSwiGLU, mA1, mB1, mBs1, plan1, (2 * I) / kBN, H / kBK, 2 * I, h, I,
                          max_mtiles * ((2 * I) / kBN), a.max_ctas, status, st);
        if (err != cudaSuccess) return err;
        err = launch_gemm(kEpiY, mA2, mB2, mBs2, plan2, H / kBN, I / kBK, H, y, H, max_mtiles * (H / kBN), a.max_ctas,
                          status, st);
        if (err != cudaSuccess) return err;
    }
    if (a.peers) {
        const EpPeerLayout L = ep_peer_layout(a.peers->world, a.peers->cap, a.peers->H, a.peers->k);
        ep_partials_kernel<<<T, 160, 0, st>>>(y, wts, dest, k, *a.peers, L.part, L.sig, a.slot_counts, a.slot_fail,
                                              status, a.done);
        return cudaGetLastError();
    }
    prefill_combine_kernel<<<T, std::min(256, (H / 8 + 31) / 32 * 32), 0, st>>>(y, wts, dest, T, H, k, S, a.accumulate,
                                                                                 a.out);
    return cudaGetLastError();
}

}  // namespace uocr
