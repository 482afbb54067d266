// Decode-step MoE sublayer (MoE.decode_rows, unlimited_ocr_max/decoder.py:641-655) for B <= 8
// tokens: three kernels chained by programmatic dependent launch (PDL), each streaming its
// weights from HBM once.
//
//   K1 route   8 CTAs x 8 experts: fp32 router logits in the oracle's order, then the last
//              CTA runs softmax + top-k (bit-exact) and groups the routing by expert
//              ("slots": 0..S-1 the shared experts, S+u the u-th distinct routed expert in
//              ascending id; each slot lists its (pair, token, weight) entries).
//   K2 gate/up persistent: items (slot, rows, token group) -> h[pair][n] = silu(g) * u.
//   K3 down    CTA b owns output rows [b*H/G, (b+1)*H/G); it walks every slot, computes
//              y[slot][token][row] and finishes with the routing-weighted combine
//              out[t][j] = sum over t's slots in order of (w * y or y), no cross-CTA state.
// Pairs: routed (token t, slot s) is pair t*k + s; shared expert q's copy of token t is pair
// k*B + q*B + t. A pair's arithmetic uses only its own token and expert and a token's slots are
// summed in ascending order, so every output row is bitwise independent of the batch.
//
// K2 and K3 are warp-specialised: one producer warp streams each work item's bytes (weight
// rows, int8 scales, and for K3 the pairs' h rows) with cp.async.bulk into a ring of shared-
// memory stages guarded by full/empty mbarriers; each of the 8 consumer warps owns whole
// items, so an SM keeps up to 8 items in flight with no CTA-wide barrier per item. Stage s is
// always consumed by warp s % 8 (the stage count is a multiple of 8), so a warp never waits on
// an mbarrier phase more than one round ahead of the last one it saw.
//
// Every device-side wait is bounded (sm100.cuh, kWaitBudgetNs): on expiry the waiter records a
// status code in the workspace and the kernel winds down without writing its output.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace uocr {

constexpr int kCW = 8;                       // K2 consumer warps
constexpr int kThreads = (kCW + 1) * 32;     // + producer warp
constexpr int kCW3 = 4;                      // K3 consumer warps (two stages each)
constexpr int kThreads3 = (kCW3 + 1) * 32;
constexpr int kMaxB = 8;
constexpr int kGuTok = 4;                    // tokens per K2 item
constexpr int kDnTok = 2;                    // tokens per K3 item
constexpr int kRouteExperts = 8;             // experts per K1 CTA
constexpr int kMaxSlotsSm = 72;              // shared (<= 8) + routed (<= 64)

// Slots of this step in shared memory: rows [0, S) the shared experts, [S, S+U) routed.
struct SlotTable {
    int nslot;
    int pad[3];
    int expert[kMaxSlotsSm];
    int count[kMaxSlotsSm];
    int pair[kMaxSlotsSm][kMaxB];
    int token[kMaxSlotsSm][kMaxB];
    float weight[kMaxSlotsSm][kMaxB];
};

struct ItemMeta {
    int type;    // 0 end marker, 1 work
    int slot, rows0, nrows, q0, nq;
    int sc_off;  // byte offset of the int8 scales inside the stage
    int h_off;   // K3: byte offset of the h rows inside the stage
};

// The shared-expert slots (known from the shape alone).
UOCR_DEV void load_shared_slots(SlotTable* tb, const DecodeArgs& a, int tid, int nthreads) {
    const int kB = a.topk * a.B;
    for (int s = tid; s < a.S; s += nthreads) {
        tb->expert[s] = s;
        tb->count[s] = a.B;
        for (int t = 0; t < kMaxB; ++t) {
            tb->pair[s][t] = kB + s * a.B + t;
            tb->token[s][t] = t;
            tb->weight[s][t] = 1.0f;
        }
    }
    if (tid == 0) tb->nslot = a.S;
}

// The routed slots, from the route kernel's table (call after the dependency wait).
UOCR_DEV void load_routed_slots(SlotTable* tb, const DecodeArgs& a, int lane) {
    const RouteTable* g = a.table;
    const int U = __ldcg(&g->U);
    for (int u = lane; u < U; u += 32) {
        const int row = a.S + u;
        tb->expert[row] = __ldcg(&g->expert[u]);
        tb->count[row] = __ldcg(&g->count[u]);
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) {
            tb->pair[row][q] = __ldcg(&g->pair[u][q]);
            tb->token[row][q] = __ldcg(&g->token[u][q]);
            tb->weight[row][q] = __ldcg(&g->weight[u][q]);
        }
    }
    __syncwarp();
    if (lane == 0) tb->nslot = a.S + U;
    __syncwarp();
}

// Four consecutive weights (bf16 or int8) at element offset k of a staged row -> fp32.
template <bool kI8>
UOCR_DEV void load4(const unsigned char* row, int k, float (&w)[4]) {
    if (kI8) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(row + k) ^ 0x80808080u;
#pragma unroll
        for (int i = 0; i < 4; ++i) w[i] = s8_byte_to_f32(v, i);
    } else {
        const uint2 v = *reinterpret_cast<const uint2*>(row + 2 * k);
        w[0] = bf16lo(v.x); w[1] = bf16hi(v.x); w[2] = bf16lo(v.y); w[3] = bf16hi(v.y);
    }
}

UOCR_DEV float dot4(const float (&w)[4], const float4& x, float acc) {
    acc = __fmaf_rn(w[0], x.x, acc);
    acc = __fmaf_rn(w[1], x.y, acc);
    acc = __fmaf_rn(w[2], x.z, acc);
    acc = __fmaf_rn(w[3], x.w, acc);
    return acc;
}

// Diagnostics timeline: per CTA `items` records of 8 words
// {consumer wait start, data ready, done, slot<<32|rows, producer issue, 0, 0, 0} (global-timer ns).
UOCR_DEV unsigned long long* trace_rec(const DecodeArgs& a, int half, int n) {
    if (!a.trace || n >= a.trace_items / 2) return nullptr;
    return a.trace + ((size_t)blockIdx.x * a.trace_items + (size_t)half * (a.trace_items / 2) + n) * 8;
}

// ======================================================================================
// K1: route
// ======================================================================================
// Thread (token group tg, expert jl, segment s) fma-chains router row jl's segment s against
// tokens tg*TPG..: the oracle's per-segment chain; segments then summed in ascending order.
__global__ void __launch_bounds__(256)
decode_route_kernel(DecodeArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int H = a.H, B = a.B, L = H / 8, E = a.E, k = a.topk;
    const int LW = L + 8;   // padded bf16 segment stride
    const int LX = L + 4;   // padded fp32 segment stride
    uint16_t* ws = reinterpret_cast<uint16_t*>(smem);                          // [8 experts][8 segs][LW]
    float* xs = reinterpret_cast<float*>(smem + sizeof(uint16_t) * 64 * LW);    // [B][8 segs][LX]
    float* part = xs + kMaxB * 8 * LX;                                          // [(jl*8+s)*kMaxB+b]
    int* flag = reinterpret_cast<int*>(part + 64 * kMaxB);                      // [16 + 64 + 64]
    const int tid = threadIdx.x;
    const int j0 = blockIdx.x * kRouteExperts;
    // router rows (weights, independent of the previous kernel) before the dependency wait
    for (int i = tid; i < kRouteExperts * (H / 8); i += blockDim.x) {
        const int jl = i / (H / 8), k8 = (i % (H / 8)) * 8;
        if (j0 + jl < E) {
            const uint4 v = *reinterpret_cast<const uint4*>(a.router + (size_t)(j0 + jl) * H + k8);
            *reinterpret_cast<uint4*>(ws + (jl * 8 + k8 / L) * LW + (k8 % L)) = v;
        }
    }
    pdl_wait_prior_grid();
    pdl_launch_dependents();
    for (int i = tid; i < B * (H / 4); i += blockDim.x) {
        const int b = i / (H / 4), k4 = (i % (H / 4)) * 4;
        const float4 v = *reinterpret_cast<const float4*>(a.x + (size_t)b * H + k4);
        *reinterpret_cast<float4*>(xs + (b * 8 + k4 / L) * LX + (k4 % L)) = v;
    }
    __syncthreads();
    {
        const int tg = tid >> 6, jl = (tid >> 3) & 7, s = tid & 7;
        const int TPG = (B + 3) / 4;
        if (j0 + jl < E && tg * TPG < B) {
            float acc[2] = {0.0f, 0.0f};
            const uint16_t* wr = ws + (jl * 8 + s) * LW;
            for (int kk = 0; kk < L; kk += 8) {
                float wf[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(wr + kk), wf);
#pragma unroll
                for (int bb = 0; bb < 2; ++bb) {
                    const int b = tg * TPG + bb;
                    if (bb < TPG && b < B) {
                        const float* xr = xs + (b * 8 + s) * LX + kk;
                        const float4 xa = *reinterpret_cast<const float4*>(xr);
                        const float4 xb = *reinterpret_cast<const float4*>(xr + 4);
                        float v = acc[bb];
                        v = __fmaf_rn(wf[0], xa.x, v); v = __fmaf_rn(wf[1], xa.y, v);
                        v = __fmaf_rn(wf[2], xa.z, v); v = __fmaf_rn(wf[3], xa.w, v);
                        v = __fmaf_rn(wf[4], xb.x, v); v = __fmaf_rn(wf[5], xb.y, v);
                        v = __fmaf_rn(wf[6], xb.z, v); v = __fmaf_rn(wf[7], xb.w, v);
                        acc[bb] = v;
                    }
                }
            }
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
                const int b = tg * TPG + bb;
                if (bb < TPG && b < B) part[(jl * 8 + s) * kMaxB + b] = acc[bb];
            }
        }
    }
    __syncthreads();
    if (tid < kRouteExperts * B) {
        const int jl = tid / B, b = tid % B, j = j0 + jl;
        if (j < E) {
            float total = part[(jl * 8 + 0) * kMaxB + b];
#pragma unroll
            for (int q = 1; q < 8; ++q) total = __fadd_rn(total, part[(jl * 8 + q) * kMaxB + b]);
            if (a.bias) total = __fadd_rn(total, a.bias[j]);
            a.logits[b * 64 + j] = total;
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        flag[0] = (atomicAdd(&a.ctl->route_done, 1u) == gridDim.x - 1) ? 1 : 0;
    }
    __syncthreads();
    if (!flag[0]) return;
    // the last CTA: softmax + top-k per token (warp b serves token b), then group by expert
    __threadfence();
    int* ids_s = flag + 16;
    float* wts_s = reinterpret_cast<float*>(flag + 16 + 64);
    const int warp = tid >> 5, lane = tid & 31;
    if (warp < B) {
        const int b = warp;
        const bool v0 = lane < E, v1 = lane + 32 < E;
        const float l0 = v0 ? __ldcg(a.logits + b * 64 + lane) : -INFINITY;
        const float l1 = v1 ? __ldcg(a.logits + b * 64 + lane + 32) : -INFINITY;
        float m = fmaxf(l0, l1);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        const float e0 = v0 ? uocr_exp(__fsub_rn(l0, m)) : 0.0f;
        const float e1 = v1 ? uocr_exp(__fsub_rn(l1, m)) : 0.0f;
        float sum = __fadd_rn(e0, e1);
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) sum = __fadd_rn(sum, __shfl_xor_sync(0xffffffffu, sum, off));
        float p0 = v0 ? __fdiv_rn(e0, sum) : -1.0f;
        float p1 = v1 ? __fdiv_rn(e1, sum) : -1.0f;
        for (int rr = 0; rr < k; ++rr) {
            float bp = p0;
            int bi = lane;
            if (p1 > bp) { bp = p1; bi = lane + 32; }
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) {
                const float op = __shfl_xor_sync(0xffffffffu, bp, off);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
                if (op > bp || (op == bp && oi < bi)) { bp = op; bi = oi; }
            }
            if (bi == lane) p0 = -2.0f;
            if (bi == lane + 32) p1 = -2.0f;
            if (lane == 0) {
                a.ids[b * k + rr] = bi;
                a.wts[b * k + rr] = bp;
                ids_s[b * k + rr] = bi;
                wts_s[b * k + rr] = bp;
            }
        }
    }
    __syncthreads();
    const int kB = k * B;
    int c = 0;
    if (tid < 64) {
        for (int q = 0; q < kB; ++q) c += (ids_s[q] == tid);
        const unsigned bal = __ballot_sync(0xffffffffu, c > 0);
        if (lane == 0) flag[8 + warp] = (int)bal;
    }
    __syncthreads();
    if (tid < 64) {
        const unsigned long long used =
            (unsigned long long)(unsigned)flag[8] | ((unsigned long long)(unsigned)flag[9] << 32);
        if (c > 0) {
            const int u = __popcll(used & ((1ull << tid) - 1ull));
            RouteTable* tb = a.table;
            int n = 0;
            for (int q = 0; q < kB; ++q) {
                if (ids_s[q] == tid) {
                    tb->pair[u][n] = q;
                    tb->token[u][n] = q / k;
                    tb->weight[u][n] = wts_s[q];
                    ++n;
                }
            }
            tb->expert[u] = tid;
            tb->count[u] = c;
        }
        if (tid == 0) {
            a.table->U = __popcll(used);
            a.ctl->route_done = 0;  // single-use election counter: leave it zeroed
        }
    }
}

// ======================================================================================
// K2: gate/up + SwiGLU
// ======================================================================================
// Items per slot: (I / RB) row blocks x ceil(count / kGuTok) token groups, RB = 2 row pairs
// for bf16 weights and 4 for int8, so every item is ~10 KB. Items are dealt round-robin over
// the CTAs; shared slots first (they need no routing), then routed slots.
UOCR_DEV int gu_rb(const DecodeArgs& a, int slot) { return (slot >= a.S && a.int8) ? 4 : 2; }

UOCR_DEV int gu_items_of(const DecodeArgs& a, const SlotTable& tb, int slot) {
    return (a.I / gu_rb(a, slot)) * ((tb.count[slot] + kGuTok - 1) / kGuTok);
}

// item index i within slots [first, ...) -> (slot, row block, token group)
UOCR_DEV void gu_decode(const DecodeArgs& a, const SlotTable& tb, int first, int i, int& slot, int& rblk, int& tg) {
    int s = first;
    while (true) {
        const int n = gu_items_of(a, tb, s);
        if (i < n) break;
        i -= n;
        ++s;
    }
    const int ntg = (tb.count[s] + kGuTok - 1) / kGuTok;
    slot = s;
    rblk = i / ntg;
    tg = i % ntg;
}

// One warp, one item: kRB row pairs against up to kGuTok tokens. Lane l owns the 4-element
// chunks k = 4(l + 32j), j < NJ = H/128. A token's chunks sit in registers while every row of the
// item streams past; all rows' partial sums are reduced together (independent butterflies).
// Weight words of one row for chunks j < NJ: int8 -> one u32 (4 weights), bf16 -> two u32.
template <bool kI8, int NJ>
UOCR_DEV void lds_row(uint32_t row, int lane, uint32_t (&w)[NJ][kI8 ? 1 : 2]) {
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        const uint32_t k = 4u * (lane + 32 * j);
        if (kI8) {
            w[j][0] = lds_u32(row + k);
        } else {
            const uint2 v = lds_u64(row + 2 * k);
            w[j][0] = v.x;
            w[j][kI8 ? 0 : 1] = v.y;
        }
    }
}

template <bool kI8>
UOCR_DEV void unpack4(const uint32_t* w, float (&f)[4]) {
    if (kI8) {
        const uint32_t v = w[0] ^ 0x80808080u;
#pragma unroll
        for (int i = 0; i < 4; ++i) f[i] = s8_byte_to_f32(v, i);
    } else {
        f[0] = bf16lo(w[0]); f[1] = bf16hi(w[0]); f[2] = bf16lo(w[1]); f[3] = bf16hi(w[1]);
    }
}

template <bool kI8, int kRB, int NJ>
UOCR_DEV void gu_item_t(const DecodeArgs& a, const SlotTable& tb, const float* __restrict__ xs, int slot, int rows0,
                        int q0, int nq, const unsigned char* __restrict__ stage, int sc_off, int lane) {
    // int8 groups are 128 wide along K and lane l's chunk j is k = 4(l + 32j): group j
    const int H = NJ * 128;
    constexpr int esz = kI8 ? 1 : 2;
    const uint32_t st_s = smem_addr(stage);
    const uint32_t xs_s = smem_addr(xs);
    const uint32_t gsc_s = st_s + sc_off;
    const uint32_t usc_s = gsc_s + kRB * NJ * 4;
    for (int q = 0; q < nq; ++q) {
        const int t = tb.token[slot][q0 + q];
        const int pair = tb.pair[slot][q0 + q];
        float4 xr[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) xr[j] = lds_f128(xs_s + 4u * ((uint32_t)t * H + 4 * (lane + 32 * j)));
#pragma unroll 1
        for (int r = 0; r < kRB; ++r) {
            uint32_t wg[NJ][kI8 ? 1 : 2], wu[NJ][kI8 ? 1 : 2];
            lds_row<kI8, NJ>(st_s + (uint32_t)r * H * esz, lane, wg);
            lds_row<kI8, NJ>(st_s + (uint32_t)(kRB + r) * H * esz, lane, wu);
            float sg[NJ], su[NJ];
            if (kI8) {
#pragma unroll
                for (int j = 0; j < NJ; ++j) {
                    sg[j] = lds_f32(gsc_s + 4u * (r * NJ + j));
                    su[j] = lds_f32(usc_s + 4u * (r * NJ + j));
                }
            }
            float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                float fg[4], fu[4];
                unpack4<kI8>(wg[j], fg);
                unpack4<kI8>(wu[j], fu);
                if (kI8) {
                    acc[0][j & 1] = __fmaf_rn(sg[j], dot4(fg, xr[j], 0.0f), acc[0][j & 1]);
                    acc[1][j & 1] = __fmaf_rn(su[j], dot4(fu, xr[j], 0.0f), acc[1][j & 1]);
                } else {
                    acc[0][j & 1] = dot4(fg, xr[j], acc[0][j & 1]);
                    acc[1][j & 1] = dot4(fu, xr[j], acc[1][j & 1]);
                }
            }
            float g = __fadd_rn(acc[0][0], acc[0][1]);
            float u = __fadd_rn(acc[1][0], acc[1][1]);
#pragma unroll
            for (int off = 16; off >= 1; off >>= 1) {
                g = __fadd_rn(g, __shfl_xor_sync(0xffffffffu, g, off));
                u = __fadd_rn(u, __shfl_xor_sync(0xffffffffu, u, off));
            }
            if (lane == 0) a.h[(size_t)pair * a.I + rows0 + r] = silu(g) * u;
        }
    }
}

// Generic K-length fallback (any H multiple of 128): the same order, runtime trip count.
template <bool kI8, int kRB>
UOCR_DEV void gu_item_any(const DecodeArgs& a, const SlotTable& tb, const float* __restrict__ xs, int slot, int rows0,
                          int q0, int nq, const unsigned char* __restrict__ stage, int sc_off, int lane) {
    const int H = a.H, NJ = H / 128;
    constexpr int esz = kI8 ? 1 : 2;
    const int NG = NJ;  // groups of 128 along K
    const float* gsc = reinterpret_cast<const float*>(stage + sc_off);
    const float* usc = gsc + kRB * NG;
    for (int q = 0; q < nq; ++q) {
        const int t = tb.token[slot][q0 + q];
        const int pair = tb.pair[slot][q0 + q];
        float g[kRB], u[kRB];
#pragma unroll
        for (int r = 0; r < kRB; ++r) {
            const unsigned char* grow = stage + (size_t)r * H * esz;
            const unsigned char* urow = stage + (size_t)(kRB + r) * H * esz;
            float ga = 0.0f, ua = 0.0f;
            for (int j = 0; j < NJ; ++j) {
                const int k = 4 * (lane + 32 * j);
                const float4 xv = *reinterpret_cast<const float4*>(xs + (size_t)t * H + k);
                float wg[4], wu[4];
                load4<kI8>(grow, k, wg);
                load4<kI8>(urow, k, wu);
                if (kI8) {
                    ga = __fmaf_rn(gsc[r * NG + j], dot4(wg, xv, 0.0f), ga);
                    ua = __fmaf_rn(usc[r * NG + j], dot4(wu, xv, 0.0f), ua);
                } else {
                    ga = dot4(wg, xv, ga);
                    ua = dot4(wu, xv, ua);
                }
            }
            g[r] = ga;
            u[r] = ua;
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1) {
#pragma unroll
            for (int r = 0; r < kRB; ++r) {
                g[r] = __fadd_rn(g[r], __shfl_xor_sync(0xffffffffu, g[r], off));
                u[r] = __fadd_rn(u[r], __shfl_xor_sync(0xffffffffu, u[r], off));
            }
        }
        if (lane < kRB) {
            float gv = g[0], uv = u[0];
#pragma unroll
            for (int r = 1; r < kRB; ++r)
                if (lane == r) { gv = g[r]; uv = u[r]; }
            a.h[(size_t)pair * a.I + rows0 + lane] = silu(gv) * uv;
        }
    }
}

UOCR_DEV void gu_item(const DecodeArgs& a, const SlotTable& tb, const float* xs, const ItemMeta& m,
                      const unsigned char* stage, int lane) {
    const int slot = m.slot, rows0 = m.rows0, q0 = m.q0, nq = m.nq, sc = m.sc_off;
    const bool i8 = slot >= a.S && a.int8;
    const int NJ = a.H / 128;
    if (i8) {
        if (NJ == 10) gu_item_t<true, 4, 10>(a, tb, xs, slot, rows0, q0, nq, stage, sc, lane);
        else if (NJ == 2) gu_item_t<true, 4, 2>(a, tb, xs, slot, rows0, q0, nq, stage, sc, lane);
        else gu_item_any<true, 4>(a, tb, xs, slot, rows0, q0, nq, stage, sc, lane);
    } else {
        if (NJ == 10) gu_item_t<false, 2, 10>(a, tb, xs, slot, rows0, q0, nq, stage, sc, lane);
        else if (NJ == 2) gu_item_t<false, 2, 2>(a, tb, xs, slot, rows0, q0, nq, stage, sc, lane);
        else gu_item_any<false, 2>(a, tb, xs, slot, rows0, q0, nq, stage, sc, lane);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
decode_gate_up_kernel(DecodeArgs a, int nst, uint32_t stage_bytes, uint32_t off_tbl, uint32_t off_meta,
                      uint32_t off_xs, uint32_t off_stages) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int abort_flag;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + nst;
    SlotTable* tb = reinterpret_cast<SlotTable*>(smem + off_tbl);
    ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    float* xs = reinterpret_cast<float*>(smem + off_xs);
    unsigned char* stages = smem + off_stages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        abort_flag = 0;
        fence_mbar_init();
        pdl_launch_dependents();  // K3 waits for this grid before it reads h
    }
    // the tokens (complete: the route kernel let this grid launch only after its own wait)
    for (int i = tid; i < a.B * (a.H / 4); i += blockDim.x)
        reinterpret_cast<float4*>(xs)[i] = reinterpret_cast<const float4*>(a.x)[i];
    load_shared_slots(tb, a, tid, blockDim.x);
    __syncthreads();

    if (warp == kCW) {
        // ---------------- producer ----------------
        // Each CTA takes a contiguous range of the phase's items and walks it incrementally
        // (slot, row block, token group), so the per-item work is a handful of instructions.
        int n = 0, st = 0;
        uint32_t round = 0;
        bool ok = true;
        const int NG = a.H / a.G;
        for (int phase = 0; phase < 2 && ok; ++phase) {
            if (phase == 1) {
                pdl_wait_prior_grid();  // the routing table
                load_routed_slots(tb, a, lane);
            }
            const int first = phase == 0 ? 0 : a.S;
            const int last = phase == 0 ? a.S : tb->nslot;
            int total = 0;
            for (int s2 = first; s2 < last; ++s2) total += gu_items_of(a, *tb, s2);
            const int lo = (int)((long)blockIdx.x * total / gridDim.x);
            const int hi = (int)((long)(blockIdx.x + 1) * total / gridDim.x);
            if (lo >= hi) continue;
            int slot = first, base = 0;
            while (lo >= base + gu_items_of(a, *tb, slot)) base += gu_items_of(a, *tb, slot++);
            // per-slot constants
            int count = 0, ntg = 0, RB = 0, nrb = 0, esz = 0;
            bool i8 = false;
            uint32_t blk = 0, scb = 0;
            const unsigned char* wbase = nullptr;
            const unsigned char* sbase = nullptr;
            auto enter_slot = [&](int sl) {
                count = tb->count[sl];
                ntg = (count + kGuTok - 1) / kGuTok;
                i8 = sl >= a.S && a.int8;
                RB = i8 ? 4 : 2;
                nrb = a.I / RB;
                esz = i8 ? 1 : 2;
                blk = (uint32_t)RB * a.H * esz;
                scb = (uint32_t)RB * NG * 4;
                const int e = tb->expert[sl];
                wbase = sl < a.S ? reinterpret_cast<const unsigned char*>(a.w13_shared) + (size_t)e * 2 * a.I * a.H * 2
                                 : reinterpret_cast<const unsigned char*>(a.w13) + (size_t)e * 2 * a.I * a.H * esz;
                sbase = i8 ? reinterpret_cast<const unsigned char*>(a.s13) + (size_t)e * 2 * a.I * NG * 4 : nullptr;
            };
            enter_slot(slot);
            int rblk = (lo - base) / ntg, tg = (lo - base) % ntg;
            for (int i = lo; i < hi; ++i) {
                unsigned long long t_top = 0;
                if (a.trace && lane == 0) t_top = global_timer_ns();
                if (round > 0 && !mbar_wait_warp(&empty[st], (round - 1) & 1, nullptr, &a.ctl->status)) {
                    ok = false;
                    break;
                }
                if (a.trace && lane == 0) {
                    unsigned long long* tr = trace_rec(a, 0, n);
                    if (tr) { tr[6] = t_top; tr[5] = global_timer_ns(); }
                }
                const int n0 = rblk * RB;
                const int pg0 = (n0 / 128) * 256 + (n0 % 128);
                unsigned char* dst = stages + (size_t)st * stage_bytes;
                if (lane == 0) {
                    ItemMeta& m = meta[st];
                    m.type = 1;
                    m.slot = slot;
                    m.rows0 = n0;
                    m.nrows = RB;
                    m.q0 = tg * kGuTok;
                    m.nq = min(kGuTok, count - tg * kGuTok);
                    m.sc_off = (int)(2 * blk);
                    m.h_off = 0;
                    mbar_arrive_expect_tx(&full[st], 2 * blk + (i8 ? 2 * scb : 0));
                }
                __syncwarp();
                // the item's copies, one per lane, issued by a single instruction
                {
                    const int up = lane & 1;                // 0: gate block, 1: up block
                    const bool is_sc = lane >= 2;           // lanes 2, 3: the int8 scales
                    const int prow = pg0 + (up ? 128 : 0);
                    unsigned char* d = dst + (is_sc ? 2 * blk + up * scb : up * blk);
                    const unsigned char* src = is_sc ? sbase + (size_t)prow * NG * 4 : wbase + (size_t)prow * a.H * esz;
                    if (lane < (i8 ? 4 : 2)) bulk_g2s(d, src, is_sc ? scb : blk, &full[st]);
                }
                if (lane == 0) {
                    unsigned long long* tr = trace_rec(a, 0, n);
                    if (tr) tr[4] = global_timer_ns();
                }
                __syncwarp();
                ++n;
                if (++st == nst) { st = 0; ++round; }
                if (++tg == ntg) {
                    tg = 0;
                    if (++rblk == nrb) {
                        rblk = 0;
                        if (++slot < last) enter_slot(slot);
                    }
                }
            }
        }
        if (lane == 0) {
            if (!ok) {
                abort_flag = 1;
                for (int q = max(0, n - nst); q < n; ++q) mbar_wait(&full[q % nst], (q / nst) & 1, nullptr);
            } else {
                // one end marker per consumer warp (stage n belongs to warp n % 8)
                for (int w = 0; w < kCW; ++w, ++n) {
                    if (round > 0 && !mbar_wait(&empty[st], (round - 1) & 1, &a.ctl->status)) {
                        abort_flag = 1;
                        break;
                    }
                    meta[st].type = 0;
                    mbar_arrive(&full[st]);
                    if (++st == nst) { st = 0; ++round; }
                }
            }
        }
        __syncwarp();
    } else {
        // ---------------- consumer warp: ring entries warp, warp + 8, ... ----------------
        int st = warp;
        uint32_t par = 0;
        for (int n = warp;; n += kCW) {
            unsigned long long* tr = trace_rec(a, 0, n);
            if (tr && lane == 0) tr[0] = global_timer_ns();
            if (!mbar_wait_warp(&full[st], par, &abort_flag, &a.ctl->status)) break;
            const ItemMeta& m = meta[st];
            if (m.type == 0) break;
            if (tr && lane == 0) tr[1] = global_timer_ns();
            const unsigned char* stage = stages + (size_t)st * stage_bytes;
            gu_item(a, *tb, xs, m, stage, lane);
            __syncwarp();
            if (tr && lane == 0) {
                tr[2] = global_timer_ns();
                tr[3] = ((unsigned long long)m.slot << 32) | (unsigned)m.rows0;
            }
            if (lane == 0) mbar_arrive(&empty[st]);
            st += kCW;
            if (st >= nst) { st -= nst; par ^= 1; }
        }
    }
}

// ======================================================================================
// K3: down + combine
// ======================================================================================
// One warp, one item: this CTA's nr output rows against up to kDnTok tokens of one slot. Lane l
// owns the chunks k = 4(l + 32j), j < NJ = I/128; the tokens' h chunks stay in registers while
// the rows stream past; all rows' partial sums are reduced together.
constexpr int kMaxRowsCta = 16;

template <bool kI8, int NJ>
UOCR_DEV void down_item_t(const DecodeArgs& a, const SlotTable& tb, int slot, int q0, int nq, int nr,
                          const unsigned char* __restrict__ stage, int sc_off, int h_off, float* ybuf, int lane) {
    // int8 groups are 128 wide along K: lane l's chunk j is group j
    const int I = NJ * 128;
    constexpr int esz = kI8 ? 1 : 2;
    const uint32_t st_s = smem_addr(stage);
    const uint32_t sc_s = st_s + sc_off;
    const uint32_t hs_s = st_s + h_off;
    float4 hr[kDnTok][NJ];
#pragma unroll
    for (int q = 0; q < kDnTok; ++q)
#pragma unroll
        for (int j = 0; j < NJ; ++j)
            hr[q][j] = q < nq ? lds_f128(hs_s + 4u * ((uint32_t)q * I + 4 * (lane + 32 * j)))
                              : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r0 = 0; r0 < nr; r0 += 2) {
        float v[2][kDnTok];
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = min(r0 + rr, nr - 1);
            uint32_t w[NJ][kI8 ? 1 : 2];
            lds_row<kI8, NJ>(st_s + (uint32_t)r * I * esz, lane, w);
            float s[NJ];
            if (kI8) {
#pragma unroll
                for (int j = 0; j < NJ; ++j) s[j] = lds_f32(sc_s + 4u * (r * NJ + j));
            }
            float acc[kDnTok][2];
#pragma unroll
            for (int q = 0; q < kDnTok; ++q) acc[q][0] = acc[q][1] = 0.0f;
#pragma unroll
            for (int j = 0; j < NJ; ++j) {
                float f[4];
                unpack4<kI8>(w[j], f);
#pragma unroll
                for (int q = 0; q < kDnTok; ++q)
                    acc[q][j & 1] = kI8 ? __fmaf_rn(s[j], dot4(f, hr[q][j], 0.0f), acc[q][j & 1])
                                        : dot4(f, hr[q][j], acc[q][j & 1]);
            }
#pragma unroll
            for (int q = 0; q < kDnTok; ++q) v[rr][q] = __fadd_rn(acc[q][0], acc[q][1]);
        }
#pragma unroll
        for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
            for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                for (int q = 0; q < kDnTok; ++q) v[rr][q] = __fadd_rn(v[rr][q], __shfl_xor_sync(0xffffffffu, v[rr][q], off));
        if (lane == 0) {
#pragma unroll
            for (int rr = 0; rr < 2; ++rr)
#pragma unroll
                for (int q = 0; q < kDnTok; ++q)
                    if (r0 + rr < nr && q < nq)
                        ybuf[((size_t)slot * kMaxB + tb.token[slot][q0 + q]) * nr + r0 + rr] = v[rr][q];
        }
    }
}

template <bool kI8>
UOCR_DEV void down_item_any(const DecodeArgs& a, const SlotTable& tb, int slot, int q0, int nq, int nr,
                            const unsigned char* __restrict__ stage, int sc_off, int h_off, float* ybuf, int lane) {
    const int I = a.I, NJ = I / 128;
    constexpr int esz = kI8 ? 1 : 2;
    const int NG = NJ;  // groups of 128 along K
    const float* sc = reinterpret_cast<const float*>(stage + sc_off);
    const float* hs = reinterpret_cast<const float*>(stage + h_off);
    for (int r = 0; r < nr; ++r) {
        const unsigned char* wrow = stage + (size_t)r * I * esz;
        float acc[kDnTok] = {0.0f, 0.0f};
        for (int j = 0; j < NJ; ++j) {
            const int k = 4 * (lane + 32 * j);
            float w[4];
            load4<kI8>(wrow, k, w);
            const float s = kI8 ? sc[r * NG + j] : 1.0f;
#pragma unroll
            for (int q = 0; q < kDnTok; ++q) {
                if (q < nq) {
                    const float4 hv = *reinterpret_cast<const float4*>(hs + (size_t)q * I + k);
                    acc[q] = kI8 ? __fmaf_rn(s, dot4(w, hv, 0.0f), acc[q]) : dot4(w, hv, acc[q]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < kDnTok; ++q) {
            const float y = warp_sum_butterfly(acc[q]);
            if (lane == 0 && q < nq) ybuf[((size_t)slot * kMaxB + tb.token[slot][q0 + q]) * nr + r] = y;
        }
    }
}

UOCR_DEV void down_item(const DecodeArgs& a, const SlotTable& tb, const ItemMeta& m, const unsigned char* stage,
                        float* ybuf, int nr, int lane) {
    const int slot = m.slot, q0 = m.q0, nq = m.nq, sc = m.sc_off, ho = m.h_off;
    const bool i8 = slot >= a.S && a.int8;
    const int NJ = a.I / 128;
    if (i8) {
        if (NJ == 7) down_item_t<true, 7>(a, tb, slot, q0, nq, nr, stage, sc, ho, ybuf, lane);
        else if (NJ == 1) down_item_t<true, 1>(a, tb, slot, q0, nq, nr, stage, sc, ho, ybuf, lane);
        else down_item_any<true>(a, tb, slot, q0, nq, nr, stage, sc, ho, ybuf, lane);
    } else {
        if (NJ == 7) down_item_t<false, 7>(a, tb, slot, q0, nq, nr, stage, sc, ho, ybuf, lane);
        else if (NJ == 1) down_item_t<false, 1>(a, tb, slot, q0, nq, nr, stage, sc, ho, ybuf, lane);
        else down_item_any<false>(a, tb, slot, q0, nq, nr, stage, sc, ho, ybuf, lane);
    }
}

__global__ void __launch_bounds__(kThreads3, 1)
decode_down_kernel(DecodeArgs a, int nst, uint32_t stage_bytes, uint32_t off_tbl, uint32_t off_meta,
                   uint32_t off_ybuf, uint32_t off_stages) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int abort_flag;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + nst;
    SlotTable* tb = reinterpret_cast<SlotTable*>(smem + off_tbl);
    ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    float* ybuf = reinterpret_cast<float*>(smem + off_ybuf);
    unsigned char* stages = smem + off_stages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j0 = (int)((long)blockIdx.x * a.H / gridDim.x);
    const int j1 = (int)((long)(blockIdx.x + 1) * a.H / gridDim.x);
    const int nr = j1 - j0;
    if (tid == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        abort_flag = 0;
        fence_mbar_init();
        pdl_launch_dependents();  // the next layer's route kernel waits for this grid itself
    }
    load_shared_slots(tb, a, tid, blockDim.x);
    __syncthreads();

    if (warp == kCW3) {
        // ---------------- producer ----------------
        int n = 0, st = 0;
        uint32_t round = 0;
        bool ok = true;
        bool waited = false;
        for (int slot = 0; ok; ++slot) {
            if (slot == a.S) {
                // routed slots: their table (K1) and every h (K2) are complete once K2 is
                pdl_wait_prior_grid();
                waited = true;
                load_routed_slots(tb, a, lane);
            }
            if (slot >= tb->nslot) break;
            const bool i8 = slot >= a.S && a.int8;
            const int esz = i8 ? 1 : 2;
            const int e = tb->expert[slot];
            const unsigned char* wbase =
                slot < a.S ? reinterpret_cast<const unsigned char*>(a.w2_shared) + (size_t)e * a.H * a.I * 2
                           : reinterpret_cast<const unsigned char*>(a.w2) + (size_t)e * a.H * a.I * esz;
            const uint32_t wbytes = (uint32_t)nr * a.I * esz;
            const int NG = a.I / a.G;
            // int8 scales of rows [j0, j1): a 16-byte aligned superset of the block
            const size_t sc_off = ((size_t)e * a.H + j0) * NG * 4;
            const size_t sc_a = sc_off & ~size_t(15);
            const uint32_t sc_delta = (uint32_t)(sc_off - sc_a);
            const uint32_t scb = (uint32_t)((sc_delta + (size_t)nr * NG * 4 + 15) & ~size_t(15));
            const uint32_t h_off = (uint32_t)((wbytes + (i8 ? scb : 0u) + 15u) & ~15u);
            const uint32_t hrow = (uint32_t)a.I * 4;
            const int c = tb->count[slot];
            for (int q0 = 0; q0 < c; q0 += kDnTok) {
                const int nq = min(kDnTok, c - q0);
                if (round > 0 && !mbar_wait_warp(&empty[st], (round - 1) & 1, nullptr, &a.ctl->status)) {
                    ok = false;
                    break;
                }
                unsigned char* dst = stages + (size_t)st * stage_bytes;
                if (lane == 0) {
                    ItemMeta& m = meta[st];
                    m.type = 1;
                    m.slot = slot;
                    m.rows0 = j0;
                    m.nrows = nr;
                    m.q0 = q0;
                    m.nq = nq;
                    m.sc_off = (int)(wbytes + sc_delta);
                    m.h_off = (int)h_off;
                    mbar_arrive_expect_tx(&full[st], wbytes + (i8 ? scb : 0u) + (uint32_t)nq * hrow);
                }
                __syncwarp();
                if (!waited) {
                    // h comes from K2; the first item's weight copy is issued before the wait
                    if (lane == 0) bulk_g2s(dst, wbase + (size_t)j0 * a.I * esz, wbytes, &full[st]);
                    if (i8 && lane == 1)
                        bulk_g2s(dst + wbytes, reinterpret_cast<const unsigned char*>(a.s2) + sc_a, scb, &full[st]);
                    pdl_wait_prior_grid();
                    waited = true;
                    __syncwarp();
                    if (lane < nq)
                        bulk_g2s(dst + h_off + (size_t)lane * hrow, a.h + (size_t)tb->pair[slot][q0 + lane] * a.I,
                                 hrow, &full[st]);
                } else {
                    // lane 0 weights, lane 1 int8 scales, lanes 2.. the tokens' h rows: one instruction
                    unsigned char* d;
                    const void* src;
                    uint32_t bytes;
                    bool go;
                    if (lane == 0) {
                        d = dst; src = wbase + (size_t)j0 * a.I * esz; bytes = wbytes; go = true;
                    } else if (lane == 1) {
                        d = dst + wbytes; src = reinterpret_cast<const unsigned char*>(a.s2) + sc_a; bytes = scb; go = i8;
                    } else {
                        const int q = lane - 2;
                        d = dst + h_off + (size_t)q * hrow;
                        src = a.h + (size_t)tb->pair[slot][q0 + min(q, nq - 1)] * a.I;
                        bytes = hrow;
                        go = q < nq;
                    }
                    if (go) bulk_g2s(d, src, bytes, &full[st]);
                }
                if (lane == 0) {
                    unsigned long long* tr = trace_rec(a, 1, n);
                    if (tr) tr[4] = global_timer_ns();
                }
                __syncwarp();
                ++n;
                if (++st == nst) { st = 0; ++round; }
            }
        }
        if (lane == 0) {
            if (!ok) {
                abort_flag = 1;
                for (int q = max(0, n - nst); q < n; ++q) mbar_wait(&full[q % nst], (q / nst) & 1, nullptr);
            } else {
                for (int w = 0; w < kCW3; ++w, ++n) {
                    if (round > 0 && !mbar_wait(&empty[st], (round - 1) & 1, &a.ctl->status)) {
                        abort_flag = 1;
                        break;
                    }
                    meta[st].type = 0;
                    mbar_arrive(&full[st]);
                    if (++st == nst) { st = 0; ++round; }
                }
            }
        }
        __syncwarp();
    } else {
        int st = warp;
        uint32_t par = 0;
        for (int n = warp;; n += kCW3) {
            unsigned long long* tr = trace_rec(a, 1, n);
            if (tr && lane == 0) tr[0] = global_timer_ns();
            if (!mbar_wait_warp(&full[st], par, &abort_flag, &a.ctl->status)) break;
            const ItemMeta& m = meta[st];
            if (m.type == 0) break;
            if (tr && lane == 0) tr[1] = global_timer_ns();
            const unsigned char* stage = stages + (size_t)st * stage_bytes;
            down_item(a, *tb, m, stage, ybuf, nr, lane);
            __syncwarp();
            if (tr && lane == 0) {
                tr[2] = global_timer_ns();
                tr[3] = ((unsigned long long)m.slot << 32) | (unsigned)m.q0;
            }
            if (lane == 0) mbar_arrive(&empty[st]);
            st += kCW3;
            if (st >= nst) { st -= nst; par ^= 1; }
        }
    }
    __syncthreads();
    if (abort_flag) return;
    // combine: a token's slots in ascending order (shared first, then its experts by id)
    const int B = a.B;
    for (int i = tid; i < nr * B; i += blockDim.x) {
        const int r = i % nr, t = i / nr;
        float acc = 0.0f;
        for (int s = 0; s < tb->nslot; ++s) {
            const int c = tb->count[s];
            for (int q = 0; q < c; ++q) {
                if (tb->token[s][q] == t) {
                    const float y = ybuf[((size_t)s * kMaxB + t) * nr + r];
                    acc = s < a.S ? __fadd_rn(acc, y) : __fmaf_rn(tb->weight[s][q], y, acc);
                }
            }
        }
        a.out[(size_t)t * a.H + j0 + r] = acc;
    }
}

// ======================================================================================
// host side
// ======================================================================================
static size_t up(size_t v, size_t a) { return (v + a - 1) / a * a; }

static cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

cudaError_t launch_decode_layer(const DecodeArgs& a_in, cudaStream_t st) {
    DecodeArgs a = a_in;
    int dev = 0, max_smem = 0, sms = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_decode_trace) {
        a.trace = g_decode_trace;
        a.trace_items = (int)(g_decode_trace_bytes / (sizeof(unsigned long long) * 8 * (size_t)sms)) & ~1;
    }

    // ---- K1
    {
        const int L = a.H / 8;
        const size_t smem = sizeof(uint16_t) * 64 * (L + 8) + sizeof(float) * (kMaxB * 8 * (L + 4) + 64 * kMaxB) +
                            sizeof(int) * (16 + 128);
        err = ensure_smem_optin(reinterpret_cast<const void*>(decode_route_kernel), smem);
        if (err != cudaSuccess) return err;
        void* args[] = {&a};
        const int nr = (a.E + kRouteExperts - 1) / kRouteExperts;
        err = launch_pdl(reinterpret_cast<const void*>(decode_route_kernel), dim3(nr), dim3(256), smem, st, args);
        if (err != cudaSuccess) return err;
    }
    // ---- K2
    {
        // a stage holds a bf16 item (2 row pairs) or an int8 item (4 row pairs + scales)
        const uint32_t b16 = 2u * 2 * a.H * 2;
        const uint32_t i8 = 2u * 4 * a.H + 2u * 4 * (a.H / a.G) * 4;
        uint32_t stage_bytes = (uint32_t)up(std::max(b16, a.int8 ? i8 : 0u), 128);
        const size_t off_tbl = up(16 * 16, 128);
        const size_t off_meta = off_tbl + up(sizeof(SlotTable), 128);
        const size_t off_xs = off_meta + up(sizeof(ItemMeta) * 16, 128);
        const size_t off_stages = up(off_xs + sizeof(float) * a.B * a.H, 1024);
        int nst = (int)std::min<size_t>(16, ((size_t)max_smem - off_stages) / stage_bytes);
        nst = nst / kCW * kCW;
        if (nst < kCW) return cudaErrorInvalidConfiguration;
        const size_t smem = off_stages + (size_t)nst * stage_bytes;
        err = ensure_smem_optin(reinterpret_cast<const void*>(decode_gate_up_kernel), smem);
        if (err != cudaSuccess) return err;
        uint32_t ot = (uint32_t)off_tbl, om = (uint32_t)off_meta, ox = (uint32_t)off_xs, os = (uint32_t)off_stages;
        void* args[] = {&a, &nst, &stage_bytes, &ot, &om, &ox, &os};
        err = launch_pdl(reinterpret_cast<const void*>(decode_gate_up_kernel), dim3(sms), dim3(kThreads), smem, st,
                         args);
        if (err != cudaSuccess) return err;
    }
    // ---- K3
    {
        const int grid = std::min(sms, a.H);
        const int nr_max = (a.H + grid - 1) / grid;
        const uint32_t w16 = (uint32_t)nr_max * a.I * 2;
        const uint32_t w8 = (uint32_t)nr_max * a.I + (uint32_t)up((size_t)nr_max * (a.I / a.G) * 4 + 16, 16);
        uint32_t stage_bytes =
            (uint32_t)up(up(std::max(w16, a.int8 ? w8 : 0u), 16) + (size_t)kDnTok * a.I * 4, 128);
        const int slots = a.S + std::min(a.E, a.topk * a.B);
        const size_t off_tbl = up(16 * 16, 128);
        const size_t off_meta = off_tbl + up(sizeof(SlotTable), 128);
        const size_t off_ybuf = off_meta + up(sizeof(ItemMeta) * 16, 128);
        const size_t off_stages = up(off_ybuf + sizeof(float) * (size_t)slots * kMaxB * nr_max, 1024);
        int nst = (int)std::min<size_t>(16, ((size_t)max_smem - off_stages) / stage_bytes);
        nst = nst / kCW3 * kCW3;
        if (nst < kCW3) return cudaErrorInvalidConfiguration;
        const size_t smem = off_stages + (size_t)nst * stage_bytes;
        err = ensure_smem_optin(reinterpret_cast<const void*>(decode_down_kernel), smem);
        if (err != cudaSuccess) return err;
        uint32_t ot = (uint32_t)off_tbl, om = (uint32_t)off_meta, oy = (uint32_t)off_ybuf, os = (uint32_t)off_stages;
        void* args[] = {&a, &nst, &stage_bytes, &ot, &om, &oy, &os};
        err = launch_pdl(reinterpret_cast<const void*>(decode_down_kernel), dim3(grid), dim3(kThreads3), smem, st, args);
        if (err != cudaSuccess) return err;
    }
    return cudaGetLastError();
}

}  // namespace uocr
