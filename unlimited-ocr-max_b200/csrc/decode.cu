// Decode-step MoE sublayer (MoE.decode_rows, unlimited_ocr_max/decoder.py:641-655) for B <= 8
// tokens: two persistent kernels chained by programmatic dependent launch (PDL), each
// streaming its weights from HBM once.
//
//   K2 route + gate/up   every CTA routes the step itself (fp32 logits in the oracle's order,
//              softmax, top-k: bit-exact and identical in every CTA, so no grid-wide exchange)
//              while its producer already streams shared-expert blocks; the routing groups the
//              step by expert ("slots": 0..S-1 the shared experts, S+u the u-th distinct routed
//              expert in ascending id), each slot owning contiguous rows of the h and y scratch.
//              Items (slot, block of 8 or 16 row pairs) -> h[slot row][n] = silu(g) * u.
//   K3 down + combine    items (slot, 32 output rows) -> y[slot row][j]; a publisher warp counts
//              finished 4-row groups (a self-resetting counter per group) and the one that
//              completes a group sums it over each token's slots in a fixed order: out[t][j].
// A slot's arithmetic uses only its own token rows, and each output sums a token's slots in
// ascending order, so every output row is bitwise independent of the batch.
//
// One producer warp copies each item with a single cp.async.bulk (the weights are repacked so
// an item is one contiguous block, layout.h; K3 adds one copy of the slot's h rows) into
// shared memory; all 8 consumer warps work on the same item, each on its own rows, with the
// tokens' activations held in registers. A bulk copy costs ~0.2 us to issue, so blocks of
// 28-58 KB are what keeps 100+ KB in flight per SM. Work is split over the CTAs by a static
// partition weighted by each item's cost (bytes and tokens).
//
// Every device-side wait is bounded (sm100.cuh, kWaitBudgetNs): on expiry the waiter records a
// status code in the workspace and the kernel winds down without writing its output.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "layout.h"
#include "sm100.cuh"

namespace uocr {

constexpr int kCW = 8;                       // consumer warps (K2 and K3)
constexpr int kThreads = (kCW + 1) * 32;     // + producer warp
constexpr int kMaxB = 8;
constexpr int kMaxSlotsSm = 72;              // shared (<= 8) + routed (<= 64)
constexpr int kK3Desc = 8;                   // K3 items in flight (descriptor ring)
constexpr int kThreads3 = kThreads + 32;     // K3: + publisher warp
constexpr uint32_t kBarConsumers = 1;        // named barrier of the 8 consumer warps

// Slots of this step in shared memory: rows [0, S) the shared experts, [S, S+U) routed.
struct SlotTable {
    int nslot;
    int pad[3];
    int expert[kMaxSlotsSm];
    int count[kMaxSlotsSm];
    int base[kMaxSlotsSm];
    int token[kMaxSlotsSm][kMaxB];
    float weight[kMaxSlotsSm][kMaxB];
};

struct ItemMeta {
    int slot;  // < 0: end of the work
    int blk;
    uint32_t off;  // K3: byte offset of the item in the ring
    uint32_t hoff; // K3: offset of the h rows from `off`
};

// The shared-expert slots (known from the shape alone).
UOCR_DEV void load_shared_slots(SlotTable* tb, const DecodeArgs& a, int tid, int nthreads) {
    for (int s = tid; s < a.S; s += nthreads) {
        tb->expert[s] = s;
        tb->count[s] = a.B;
        tb->base[s] = s * a.B;
        for (int t = 0; t < kMaxB; ++t) {
            tb->token[s][t] = t;
            tb->weight[s][t] = 1.0f;
        }
    }
    if (tid == 0) tb->nslot = a.S;
}

// The routed slots, from K2's table in global memory (K3, after the dependency wait; one warp).
UOCR_DEV void load_routed_slots(SlotTable* tb, const DecodeArgs& a, int lane) {
    const RouteTable* g = a.table;
    const int U = __ldcg(&g->U);
    for (int u = lane; u < U; u += 32) {
        const int row = a.S + u;
        tb->expert[row] = __ldcg(&g->expert[u]);
        tb->count[row] = __ldcg(&g->count[u]);
        tb->base[row] = __ldcg(&g->base[u]);
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) {
            tb->token[row][q] = __ldcg(&g->token[u][q]);
            tb->weight[row][q] = __ldcg(&g->weight[u][q]);
        }
    }
    __syncwarp();
    if (lane == 0) tb->nslot = a.S + U;
    __syncwarp();
}

// Diagnostics timeline: per CTA `items` records of 8 words
// {consumer wait start, data ready, done, slot<<32|block, producer issue, 0, 0, 0} (global-timer ns).
UOCR_DEV unsigned long long* trace_rec(const DecodeArgs& a, int half, int n) {
    if (!a.trace || n >= a.trace_items / 2) return nullptr;
    return a.trace + ((size_t)blockIdx.x * a.trace_items + (size_t)half * (a.trace_items / 2) + n) * 8;
}

// Weight words of one staged row for lane l's chunks k = 4(l + 32j), j < NJ:
// int8 -> one u32 (4 weights), bf16 -> two u32.
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

UOCR_DEV float dot4(const float (&w)[4], const float4& x, float acc) {
    acc = __fmaf_rn(w[0], x.x, acc);
    acc = __fmaf_rn(w[1], x.y, acc);
    acc = __fmaf_rn(w[2], x.z, acc);
    acc = __fmaf_rn(w[3], x.w, acc);
    return acc;
}

// Sum each of the N values over the warp (every lane gets every total).
template <int N>
UOCR_DEV void warp_sum_n(float (&v)[N]) {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = __fadd_rn(v[i], __shfl_xor_sync(0xffffffffu, v[i], off));
}


// ======================================================================================
// routing inside a CTA (the 8 consumer warps of K2)
// ======================================================================================
// Scratch of the step's routing in shared memory.
struct RouteSmem {
    float logits[kMaxB][64];
    int ids[kMaxB * kDecodeMaxTopk];
    float wts[kMaxB * kDecodeMaxTopk];
    int cnt[64];
    int rowof[kMaxB * kDecodeMaxTopk];
    unsigned used[2];
};

// MoEGate (decoder.py:500-514) for the B tokens of xs, in the oracle's fp32 order: logit =
// 8 segments of H/8, each an fma chain in ascending k from +0, summed in ascending order, +
// bias; softmax with this build's exponential and a fixed butterfly sum; top-k by (p desc,
// index asc). Warp w computes segment w of every expert for every token (lane: experts lane
// and lane + 32). `part` is >= 8 * kMaxB * 64 floats of scratch. Then the slot table: routed
// slot u is the u-th used expert; its rows start after the shared experts' S * B rows.
// CTA 0 also writes ids / wts and the global RouteTable (read by K3).
UOCR_DEV void cta_route(const DecodeArgs& a, const float* xs, float* part, RouteSmem* rs, SlotTable* tb, int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    const int H = a.H, L = H / 8, B = a.B, E = a.E, k = a.topk;
    {
        const int s = warp;
        float acc[2][kMaxB];
#pragma unroll
        for (int t = 0; t < kMaxB; ++t) acc[0][t] = acc[1][t] = 0.0f;
        const bool v0 = lane < E, v1 = lane + 32 < E;
        const uint16_t* w0 = a.router + (size_t)(v0 ? lane : 0) * H + s * L;
        const uint16_t* w1 = a.router + (size_t)(v1 ? lane + 32 : 0) * H + s * L;
        const uint32_t xs_s = smem_addr(xs) + 4u * (uint32_t)(s * L);
        for (int kk = 0; kk < L; kk += 8) {
            float f0[8], f1[8];
            unpack_bf16x8(ldg_nc_v4(w0 + kk), f0);
            unpack_bf16x8(ldg_nc_v4(w1 + kk), f1);
#pragma unroll
            for (int t = 0; t < kMaxB; ++t) {
                if (t < B) {
                    const uint32_t xr = xs_s + 4u * (uint32_t)(t * H + kk);
                    const float4 xa = lds_f128(xr), xb = lds_f128(xr + 16);
                    const float x8[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                    float u0 = acc[0][t], u1 = acc[1][t];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        u0 = __fmaf_rn(f0[i], x8[i], u0);
                        u1 = __fmaf_rn(f1[i], x8[i], u1);
                    }
                    acc[0][t] = u0;
                    acc[1][t] = u1;
                }
            }
        }
#pragma unroll
        for (int t = 0; t < kMaxB; ++t) {
            if (t < B) {
                part[(s * kMaxB + t) * 64 + lane] = acc[0][t];
                part[(s * kMaxB + t) * 64 + lane + 32] = acc[1][t];
            }
        }
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    for (int i = tid; i < B * 64; i += kCW * 32) {
        const int t = i >> 6, e = i & 63;
        if (e < E) {
            float total = part[t * 64 + e];
#pragma unroll
            for (int s = 1; s < 8; ++s) total = __fadd_rn(total, part[(s * kMaxB + t) * 64 + e]);
            if (a.bias) total = __fadd_rn(total, a.bias[e]);
            rs->logits[t][e] = total;
        }
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    // softmax + top-k: warp b serves token b
    if (warp < B) {
        const int b = warp;
        const bool v0 = lane < E, v1 = lane + 32 < E;
        const float l0 = v0 ? rs->logits[b][lane] : -INFINITY;
        const float l1 = v1 ? rs->logits[b][lane + 32] : -INFINITY;
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
                rs->ids[b * k + rr] = bi;
                rs->wts[b * k + rr] = bp;
                if (blockIdx.x == 0) {
                    a.ids[b * k + rr] = bi;
                    a.wts[b * k + rr] = bp;
                }
            }
        }
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    // group by expert (threads 0..63 = experts)
    const int kB = k * B;
    int c = 0;
    if (tid < 64) {
        for (int q = 0; q < kB; ++q) c += (rs->ids[q] == tid);
        rs->cnt[tid] = c;
        const unsigned bal = __ballot_sync(0xffffffffu, c > 0);
        if (lane == 0) rs->used[warp] = bal;
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    const unsigned long long used = (unsigned long long)rs->used[0] | ((unsigned long long)rs->used[1] << 32);
    RouteTable* g = a.table;
    const bool pub = blockIdx.x == 0;  // CTA 0 publishes the table for K3
    if (tid < 64 && c > 0) {
        const int u = __popcll(used & ((1ull << tid) - 1ull));
        const int row = a.S + u;
        int base = a.S * B;
        for (int e = 0; e < tid; ++e) base += rs->cnt[e];
        int n = 0;
        for (int q = 0; q < kB; ++q) {
            if (rs->ids[q] == tid) {
                tb->token[row][n] = q / k;
                tb->weight[row][n] = rs->wts[q];
                rs->rowof[q] = base + n;
                if (pub) {
                    g->token[u][n] = q / k;
                    g->weight[u][n] = rs->wts[q];
                }
                ++n;
            }
        }
        tb->expert[row] = tid;
        tb->count[row] = c;
        tb->base[row] = base;
        if (pub) {
            g->expert[u] = tid;
            g->count[u] = c;
            g->base[u] = base;
        }
    }
    if (tid == 0) {
        tb->nslot = a.S + __popcll(used);
        if (pub) g->U = __popcll(used);
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    if (pub && tid < B) {
        // token tid's routed rows in ascending expert id (the combine's order)
        int ord[kDecodeMaxTopk];
        for (int s = 0; s < k; ++s) {
            int i = s;
            while (i > 0 && rs->ids[tid * k + ord[i - 1]] > rs->ids[tid * k + s]) {
                ord[i] = ord[i - 1];
                --i;
            }
            ord[i] = s;
        }
        for (int s = 0; s < k; ++s) {
            g->tok_row[tid][s] = rs->rowof[tid * k + ord[s]];
            g->tok_w[tid][s] = rs->wts[tid * k + ord[s]];
        }
    }
    // `part` lives in a stage buffer the producer fills next with the async proxy
    fence_proxy_async_smem();
    named_bar_sync(kBarConsumers, kCW * 32);
}

// Weighted static partition: the items of slots [first, last) in order, item cost c(slot);
// this CTA takes the items whose cost prefix starts in [lo, hi) of the total.
struct Partition {
    long long lo, hi;
};
template <class CostFn, class ItemsFn>
UOCR_DEV Partition cta_share(int first, int last, CostFn cost, ItemsFn items) {
    long long total = 0;
    for (int s = first; s < last; ++s) total += (long long)items(s) * cost(s);
    Partition p;
    p.lo = total * blockIdx.x / gridDim.x;
    p.hi = total * (blockIdx.x + 1) / gridDim.x;
    return p;
}
// Items j of slot s (cost prefix before the slot `pre`, cost c) that start in [lo, hi).
UOCR_DEV void slot_range(long long pre, long long c, int n, const Partition& p, int& j0, int& j1) {
    long long a = p.lo - pre, b = p.hi - pre;
    long long s0 = a <= 0 ? 0 : (a + c - 1) / c;
    long long s1 = b <= 0 ? 0 : (b + c - 1) / c;
    j0 = (int)(s0 < n ? s0 : n);
    j1 = (int)(s1 < n ? s1 : n);
}

// ======================================================================================
// K2: route + gate/up + SwiGLU
// ======================================================================================
// Items: (slot, block) with I / P blocks per slot, P = 16 row pairs for int8 stacks and 8 for
// bf16 (one packed block, layout.h). Shared slots first (streamed while the CTA routes), then
// routed slots.
UOCR_DEV int gu_pairs(const DecodeArgs& a, int slot) { return (slot >= a.S && a.int8) ? 16 : 8; }
// relative cost of one item: weight bytes plus per-token work
UOCR_DEV long long gu_cost(const SlotTable& tb, int slot) { return 6 + tb.count[slot]; }

// One warp's share of an item for tokens [q0, q0 + NQ) of the slot: row pairs
// [warp * PW, warp * PW + PW). Lane l owns the chunks k = 4(l + 32j), j < NJ = H/128 (for int8,
// chunk j lies in scale group j); the tokens' chunks stay in registers while the rows stream.
template <bool kI8, int NJ, int NQ>
UOCR_DEV void gu_rows_t(const DecodeArgs& a, const SlotTable& tb, uint32_t xs_s, int slot, int blk, int q0,
                        uint32_t stage_s, int lane, int warp) {
    constexpr int P = kI8 ? 16 : 8;
    constexpr int PW = P / kCW;
    constexpr int H = NJ * 128;
    constexpr uint32_t rowb = kI8 ? H : 2 * H;
    const uint32_t gsc_s = stage_s + 2u * P * rowb;  // int8 gate scales [P][NJ], then up scales
    const uint32_t usc_s = gsc_s + 4u * P * NJ;
    const int base = tb.base[slot];
    float4 xr[NQ][NJ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const int t = tb.token[slot][q0 + q];
#pragma unroll
        for (int j = 0; j < NJ; ++j) xr[q][j] = lds_f128(xs_s + 4u * ((uint32_t)t * H + 4 * (lane + 32 * j)));
    }
#pragma unroll 1
    for (int pp = 0; pp < PW; ++pp) {
        const int p = warp * PW + pp;
        uint32_t wg[NJ][kI8 ? 1 : 2], wu[NJ][kI8 ? 1 : 2];
        lds_row<kI8, NJ>(stage_s + (uint32_t)p * rowb, lane, wg);
        lds_row<kI8, NJ>(stage_s + (uint32_t)(P + p) * rowb, lane, wu);
        float acc[2 * NQ][2];
#pragma unroll
        for (int i = 0; i < 2 * NQ; ++i) acc[i][0] = acc[i][1] = 0.0f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            float fg[4], fu[4];
            unpack4<kI8>(wg[j], fg);
            unpack4<kI8>(wu[j], fu);
            if (kI8) {
                const float sg = lds_f32(gsc_s + 4u * (p * NJ + j));
                const float su = lds_f32(usc_s + 4u * (p * NJ + j));
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    acc[2 * q][j & 1] = __fmaf_rn(sg, dot4(fg, xr[q][j], 0.0f), acc[2 * q][j & 1]);
                    acc[2 * q + 1][j & 1] = __fmaf_rn(su, dot4(fu, xr[q][j], 0.0f), acc[2 * q + 1][j & 1]);
                }
            } else {
#pragma unroll
                for (int q = 0; q < NQ; ++q) {
                    acc[2 * q][j & 1] = dot4(fg, xr[q][j], acc[2 * q][j & 1]);
                    acc[2 * q + 1][j & 1] = dot4(fu, xr[q][j], acc[2 * q + 1][j & 1]);
                }
            }
        }
        float v[2 * NQ];
#pragma unroll
        for (int i = 0; i < 2 * NQ; ++i) v[i] = __fadd_rn(acc[i][0], acc[i][1]);
        warp_sum_n<2 * NQ>(v);
        if (lane < NQ) {
            float g = v[0], u = v[1];
#pragma unroll
            for (int q = 1; q < NQ; ++q)
                if (lane == q) { g = v[2 * q]; u = v[2 * q + 1]; }
            a.h[(size_t)(base + q0 + lane) * a.I + blk * P + p] = silu(g) * u;
        }
    }
}

template <bool kI8, int NJ>
UOCR_DEV void gu_item_t(const DecodeArgs& a, const SlotTable& tb, uint32_t xs_s, int slot, int blk, uint32_t stage_s,
                        int lane, int warp) {
    const int cnt = tb.count[slot];
    int q0 = 0;
    for (; q0 + 2 <= cnt; q0 += 2) gu_rows_t<kI8, NJ, 2>(a, tb, xs_s, slot, blk, q0, stage_s, lane, warp);
    if (q0 < cnt) gu_rows_t<kI8, NJ, 1>(a, tb, xs_s, slot, blk, q0, stage_s, lane, warp);
}

// Any H multiple of 128 (activations re-read from shared memory per chunk).
template <bool kI8>
UOCR_DEV void gu_item_any(const DecodeArgs& a, const SlotTable& tb, const float* xs, int slot, int blk,
                          const unsigned char* stage, int lane, int warp) {
    const int P = kI8 ? 16 : 8, PW = P / kCW, H = a.H, NJ = H / 128;
    const size_t rowb = kI8 ? H : 2 * (size_t)H;
    const float* gsc = reinterpret_cast<const float*>(stage + 2 * P * rowb);
    const float* usc = gsc + P * NJ;
    const int cnt = tb.count[slot], base = tb.base[slot];
    for (int q = 0; q < cnt; ++q) {
        const float* xt = xs + (size_t)tb.token[slot][q] * H;
        for (int pp = 0; pp < PW; ++pp) {
            const int p = warp * PW + pp;
            const unsigned char* gr = stage + p * rowb;
            const unsigned char* ur = stage + (P + p) * rowb;
            float g = 0.0f, u = 0.0f;
            for (int j = 0; j < NJ; ++j) {
                const int k = 4 * (lane + 32 * j);
                const float4 xv = *reinterpret_cast<const float4*>(xt + k);
                uint32_t wg[2], wu[2];
                if (kI8) {
                    wg[0] = *reinterpret_cast<const uint32_t*>(gr + k);
                    wu[0] = *reinterpret_cast<const uint32_t*>(ur + k);
                } else {
                    const uint2 g2 = *reinterpret_cast<const uint2*>(gr + 2 * k);
                    const uint2 u2 = *reinterpret_cast<const uint2*>(ur + 2 * k);
                    wg[0] = g2.x; wg[1] = g2.y; wu[0] = u2.x; wu[1] = u2.y;
                }
                float fg[4], fu[4];
                unpack4<kI8>(wg, fg);
                unpack4<kI8>(wu, fu);
                if (kI8) {
                    g = __fmaf_rn(gsc[p * NJ + j], dot4(fg, xv, 0.0f), g);
                    u = __fmaf_rn(usc[p * NJ + j], dot4(fu, xv, 0.0f), u);
                } else {
                    g = dot4(fg, xv, g);
                    u = dot4(fu, xv, u);
                }
            }
            float v[2] = {g, u};
            warp_sum_n<2>(v);
            if (lane == 0) a.h[(size_t)(base + q) * a.I + blk * P + p] = silu(v[0]) * v[1];
        }
    }
}

UOCR_DEV void gu_item(const DecodeArgs& a, const SlotTable& tb, const float* xs, int slot, int blk,
                      const unsigned char* stage, int lane, int warp) {
    const bool i8 = slot >= a.S && a.int8;
    const int NJ = a.H / 128;
    const uint32_t xs_s = smem_addr(xs), st_s = smem_addr(stage);
    if (i8) {
        if (NJ == 10) gu_item_t<true, 10>(a, tb, xs_s, slot, blk, st_s, lane, warp);
        else if (NJ == 2) gu_item_t<true, 2>(a, tb, xs_s, slot, blk, st_s, lane, warp);
        else gu_item_any<true>(a, tb, xs, slot, blk, stage, lane, warp);
    } else {
        if (NJ == 10) gu_item_t<false, 10>(a, tb, xs_s, slot, blk, st_s, lane, warp);
        else if (NJ == 2) gu_item_t<false, 2>(a, tb, xs_s, slot, blk, st_s, lane, warp);
        else gu_item_any<false>(a, tb, xs, slot, blk, stage, lane, warp);
    }
}

__global__ void __launch_bounds__(kThreads, 1)
decode_gate_up_kernel(DecodeArgs a, int nst, uint32_t stage_bytes, uint32_t off_tbl, uint32_t off_route,
                      uint32_t off_meta, uint32_t off_xs, uint32_t off_stages) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int abort_flag;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + nst;
    uint64_t* table_ready = empty + nst;
    SlotTable* tb = reinterpret_cast<SlotTable*>(smem + off_tbl);
    RouteSmem* rs = reinterpret_cast<RouteSmem*>(smem + off_route);
    ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    float* xs = reinterpret_cast<float*>(smem + off_xs);
    unsigned char* stages = smem + off_stages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        mbar_init(table_ready, 1);
        abort_flag = 0;
        fence_mbar_init();
        pdl_launch_dependents();  // K3 launches early; it waits for this grid before it reads h
    }
    load_shared_slots(tb, a, tid, blockDim.x);
    __syncthreads();

    if (warp == kCW) {
        // ---------------- producer: one bulk copy per item ----------------
        int n = 0, st = 0;
        uint32_t round = 0;
        bool ok = true, routed = false;
        auto wait_table = [&]() {
            if (!routed) {
                ok = mbar_wait_warp(table_ready, 0, &abort_flag, &a.ctl->status);
                routed = true;
            }
        };
        auto issue = [&](int slot, int blk) {
            // the last stage doubles as the routing scratch until the table is ready
            if (round == 0 && st == nst - 1) wait_table();
            if (ok && round > 0 && !mbar_wait_warp(&empty[st], (round - 1) & 1, &abort_flag, &a.ctl->status))
                ok = false;
            if (!ok) return;
            if (lane == 0) {
                const bool i8 = slot >= a.S && a.int8;
                const uint32_t bytes = (uint32_t)w13_block_bytes(a.H, a.G, i8);
                const unsigned char* src =
                    slot < a.S ? reinterpret_cast<const unsigned char*>(a.w13_shared) +
                                     (size_t)tb->expert[slot] * w13_expert_bytes(a.I, a.H, a.G, false)
                               : reinterpret_cast<const unsigned char*>(a.w13) +
                                     (size_t)tb->expert[slot] * w13_expert_bytes(a.I, a.H, a.G, i8);
                src += (size_t)blk * bytes;
                meta[st].slot = slot;
                meta[st].blk = blk;
                mbar_arrive_expect_tx(&full[st], bytes);
                bulk_g2s(stages + (size_t)st * stage_bytes, src, bytes, &full[st]);
                unsigned long long* tr = trace_rec(a, 0, n);
                if (tr) tr[4] = global_timer_ns();
            }
            __syncwarp();
            ++n;
            if (++st == nst) { st = 0; ++round; }
        };
        for (int phase = 0; phase < 2 && ok; ++phase) {
            if (phase == 1) wait_table();
            if (!ok) break;
            const int first = phase == 0 ? 0 : a.S;
            const int last = phase == 0 ? a.S : tb->nslot;
            auto items = [&](int s) { return a.I / gu_pairs(a, s); };
            auto cost = [&](int s) { return gu_cost(*tb, s); };
            const Partition p = cta_share(first, last, cost, items);
            long long pre = 0;
            for (int s = first; s < last && ok; ++s) {
                const long long c = cost(s);
                int j0, j1;
                slot_range(pre, c, items(s), p, j0, j1);
                for (int j = j0; j < j1 && ok; ++j) issue(s, j);
                pre += (long long)items(s) * c;
            }
        }
        if (lane == 0) {
            if (!ok) {
                abort_flag = 1;
                for (int q = max(0, n - nst); q < n; ++q) mbar_wait(&full[q % nst], (q / nst) & 1, nullptr);
            } else if (round == 0 || mbar_wait(&empty[st], (round - 1) & 1, &a.ctl->status)) {
                meta[st].slot = -1;  // end marker
                mbar_arrive(&full[st]);
            } else {
                abort_flag = 1;
            }
        }
        __syncwarp();
    } else {
        // ---------------- consumers: route, then every warp takes its rows of every item ----------------
        // the tokens (complete once the previous layer's grid is)
        pdl_wait_prior_grid();
        for (int i = tid; i < a.B * (a.H / 4); i += kCW * 32)
            reinterpret_cast<float4*>(xs)[i] = __ldcg(reinterpret_cast<const float4*>(a.x) + i);
        named_bar_sync(kBarConsumers, kCW * 32);
        cta_route(a, xs, reinterpret_cast<float*>(stages + (size_t)(nst - 1) * stage_bytes), rs, tb, tid);
        if (tid == 0) mbar_arrive(table_ready);
        for (int n = 0;; ++n) {
            const int st = n % nst;
            unsigned long long* tr = warp == 0 ? trace_rec(a, 0, n) : nullptr;
            if (tr && lane == 0) tr[0] = global_timer_ns();
            if (!mbar_wait_warp(&full[st], (n / nst) & 1, &abort_flag, &a.ctl->status)) break;
            const int slot = meta[st].slot, blk = meta[st].blk;
            if (slot < 0) break;
            if (tr && lane == 0) tr[1] = global_timer_ns();
            gu_item(a, *tb, xs, slot, blk, stages + (size_t)st * stage_bytes, lane, warp);
            __syncwarp();
            if (tr && lane == 0) {
                tr[2] = global_timer_ns();
                tr[3] = ((unsigned long long)slot << 32) | (unsigned)blk;
            }
            if (lane == 0) mbar_arrive(&empty[st]);
        }
    }
}

// ======================================================================================
// K3: down + combine
// ======================================================================================
// Items: (slot, 32-row block) with H / 32 blocks per slot; an item is its weight block (one
// copy) and the slot's h rows (one copy), placed back to back in a byte ring. Warp w computes
// rows [4w, 4w + 4) of the block for all the slot's tokens.
UOCR_DEV long long dn_cost(const DecodeArgs& a, const SlotTable& tb, int slot) {
    return ((slot >= a.S && a.int8) ? 4 : 8) + tb.count[slot];
}

template <bool kI8, int NJ, int NQ>
UOCR_DEV void dn_rows_t(const DecodeArgs& a, const SlotTable& tb, int slot, int blk, int q0, uint32_t item_s,
                        uint32_t hoff, int lane, int warp) {
    constexpr int I = NJ * 128;
    constexpr uint32_t rowb = kI8 ? I : 2 * I;
    constexpr int RW = kW2Rows / kCW;  // rows per warp
    const uint32_t sc_s = item_s + (uint32_t)kW2Rows * rowb;  // int8 scales [32][NJ]
    const uint32_t h_s = item_s + hoff;
    const int base = tb.base[slot];
    float4 hr[NQ][NJ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
        const uint32_t hrow = h_s + 4u * (uint32_t)(q0 + q) * I;
#pragma unroll
        for (int j = 0; j < NJ; ++j) hr[q][j] = lds_f128(hrow + 16u * (lane + 32 * j));
    }
    float v[RW * NQ];
#pragma unroll
    for (int rr = 0; rr < RW; ++rr) {
        const int r = warp * RW + rr;
        uint32_t w[NJ][kI8 ? 1 : 2];
        lds_row<kI8, NJ>(item_s + (uint32_t)r * rowb, lane, w);
        float acc[NQ][2];
#pragma unroll
        for (int q = 0; q < NQ; ++q) acc[q][0] = acc[q][1] = 0.0f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            float f[4];
            unpack4<kI8>(w[j], f);
            if (kI8) {
                const float s = lds_f32(sc_s + 4u * (r * NJ + j));
#pragma unroll
                for (int q = 0; q < NQ; ++q) acc[q][j & 1] = __fmaf_rn(s, dot4(f, hr[q][j], 0.0f), acc[q][j & 1]);
            } else {
#pragma unroll
                for (int q = 0; q < NQ; ++q) acc[q][j & 1] = dot4(f, hr[q][j], acc[q][j & 1]);
            }
        }
#pragma unroll
        for (int q = 0; q < NQ; ++q) v[rr * NQ + q] = __fadd_rn(acc[q][0], acc[q][1]);
    }
    warp_sum_n<RW * NQ>(v);
    // lane (rr * NQ + q) stores row rr of token q
    if (lane < RW * NQ) {
        float y = v[0];
#pragma unroll
        for (int i = 1; i < RW * NQ; ++i)
            if (lane == i) y = v[i];
        const int rr = lane / NQ, q = lane % NQ;
        a.y[(size_t)(base + q0 + q) * a.H + blk * kW2Rows + warp * RW + rr] = y;
    }
}

template <bool kI8, int NJ>
UOCR_DEV void dn_item_t(const DecodeArgs& a, const SlotTable& tb, int slot, int blk, uint32_t item_s, uint32_t hoff,
                        int lane, int warp) {
    const int cnt = tb.count[slot];
    int q0 = 0;
    for (; q0 + 2 <= cnt; q0 += 2) dn_rows_t<kI8, NJ, 2>(a, tb, slot, blk, q0, item_s, hoff, lane, warp);
    if (q0 < cnt) dn_rows_t<kI8, NJ, 1>(a, tb, slot, blk, q0, item_s, hoff, lane, warp);
}

// Any I multiple of 128 (h re-read from shared memory per chunk).
template <bool kI8>
UOCR_DEV void dn_item_any(const DecodeArgs& a, const SlotTable& tb, int slot, int blk, const unsigned char* item,
                          uint32_t hoff, int lane, int warp) {
    const int I = a.I, NJ = I / 128, RW = kW2Rows / kCW;
    const size_t rowb = kI8 ? I : 2 * (size_t)I;
    const float* sc = reinterpret_cast<const float*>(item + kW2Rows * rowb);
    const float* hs = reinterpret_cast<const float*>(item + hoff);
    const int cnt = tb.count[slot], base = tb.base[slot];
    for (int q = 0; q < cnt; ++q) {
        for (int rr = 0; rr < RW; ++rr) {
            const int r = warp * RW + rr;
            const unsigned char* wr = item + r * rowb;
            float acc = 0.0f;
            for (int j = 0; j < NJ; ++j) {
                const int k = 4 * (lane + 32 * j);
                const float4 hv = *reinterpret_cast<const float4*>(hs + (size_t)q * I + k);
                uint32_t w[2];
                if (kI8) {
                    w[0] = *reinterpret_cast<const uint32_t*>(wr + k);
                } else {
                    const uint2 w2 = *reinterpret_cast<const uint2*>(wr + 2 * k);
                    w[0] = w2.x; w[1] = w2.y;
                }
                float f[4];
                unpack4<kI8>(w, f);
                acc = kI8 ? __fmaf_rn(sc[r * NJ + j], dot4(f, hv, 0.0f), acc) : dot4(f, hv, acc);
            }
            float v[1] = {acc};
            warp_sum_n<1>(v);
            if (lane == 0) a.y[(size_t)(base + q) * a.H + blk * kW2Rows + r] = v[0];
        }
    }
}

UOCR_DEV void dn_item(const DecodeArgs& a, const SlotTable& tb, int slot, int blk, const unsigned char* item,
                      uint32_t hoff, int lane, int warp) {
    const bool i8 = slot >= a.S && a.int8;
    const int NJ = a.I / 128;
    const uint32_t it_s = smem_addr(item);
    if (i8) {
        if (NJ == 7) dn_item_t<true, 7>(a, tb, slot, blk, it_s, hoff, lane, warp);
        else if (NJ == 1) dn_item_t<true, 1>(a, tb, slot, blk, it_s, hoff, lane, warp);
        else dn_item_any<true>(a, tb, slot, blk, item, hoff, lane, warp);
    } else {
        if (NJ == 7) dn_item_t<false, 7>(a, tb, slot, blk, it_s, hoff, lane, warp);
        else if (NJ == 1) dn_item_t<false, 1>(a, tb, slot, blk, it_s, hoff, lane, warp);
        else dn_item_any<false>(a, tb, slot, blk, item, hoff, lane, warp);
    }
}

// Rows [r0, r0 + 4) are complete over all slots: lane (t, r) sums token t's shared rows, then its
// routed rows in ascending expert id (w * y). (The token lists come from the global table.)
UOCR_DEV void combine_rows(const DecodeArgs& a, int r0, int lane) {
    const int t = lane >> 2, r = r0 + (lane & 3);
    if (t >= a.B) return;
    float acc = 0.0f;
    for (int q = 0; q < a.S; ++q) acc = __fadd_rn(acc, __ldcg(a.y + (size_t)(q * a.B + t) * a.H + r));
    for (int s = 0; s < a.topk; ++s) {
        const int row = __ldcg(&a.table->tok_row[t][s]);
        acc = __fmaf_rn(__ldcg(&a.table->tok_w[t][s]), __ldcg(a.y + (size_t)row * a.H + r), acc);
    }
    a.out[(size_t)t * a.H + r] = acc;
}

__global__ void __launch_bounds__(kThreads3, 1)
decode_down_kernel(DecodeArgs a, uint32_t ring_bytes, uint32_t off_tbl, uint32_t off_meta, uint32_t off_ring) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int abort_flag;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* done = full + kK3Desc;
    uint64_t* empty = done + kK3Desc;
    SlotTable* tb = reinterpret_cast<SlotTable*>(smem + off_tbl);
    ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    unsigned char* ring = smem + off_ring;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblk = a.H / kW2Rows;
    if (tid == 0) {
        for (int s = 0; s < kK3Desc; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&done[s], kCW);
            mbar_init(&empty[s], 1);
        }
        abort_flag = 0;
        fence_mbar_init();
        pdl_launch_dependents();  // the next layer's kernel waits for this grid itself
    }
    load_shared_slots(tb, a, tid, blockDim.x);
    __syncthreads();

    if (warp == kCW) {
        // ---------------- producer ----------------
        // Items are placed back to back in the ring (wrapping to 0 when one does not fit) and
        // retire in order; an item may be placed once the descriptor it reuses is free and no
        // in-flight item overlaps its bytes.
        uint32_t lo_b[kK3Desc], hi_b[kK3Desc];  // byte range of descriptor d's item
        int n = 0, oldest = 0;
        uint32_t head = 0;
        bool ok = true;
        pdl_wait_prior_grid();  // h and the routing table come from K2
        load_routed_slots(tb, a, lane);
        auto items = [&](int) { return nblk; };
        auto cost = [&](int s) { return dn_cost(a, *tb, s); };
        const Partition p = cta_share(0, tb->nslot, cost, items);
        long long pre = 0;
        for (int slot = 0; slot < tb->nslot && ok; ++slot) {
            const long long c = cost(slot);
            int j0, j1;
            slot_range(pre, c, nblk, p, j0, j1);
            pre += (long long)nblk * c;
            const bool i8 = slot >= a.S && a.int8;
            const uint32_t wbytes = (uint32_t)w2_block_bytes(a.I, a.G, i8);
            const uint32_t hoff = (wbytes + 15u) & ~15u;
            const uint32_t hbytes = (uint32_t)tb->count[slot] * a.I * 4;
            const uint32_t need = hoff + hbytes;
            for (int blk = j0; blk < j1 && ok; ++blk) {
                if (head + need > ring_bytes) head = 0;
                // retire items until this one's descriptor is free and its bytes do not overlap
                while (oldest < n) {
                    bool clash = n - oldest >= kK3Desc;
                    for (int m = oldest; m < n && !clash; ++m) {
                        const int d = m % kK3Desc;
                        clash = head < hi_b[d] && lo_b[d] < head + need;
                    }
                    if (!clash) break;
                    if (!mbar_wait_warp(&empty[oldest % kK3Desc], (oldest / kK3Desc) & 1, &abort_flag,
                                        &a.ctl->status)) {
                        ok = false;
                        break;
                    }
                    ++oldest;
                }
                if (!ok) break;
                const int d = n % kK3Desc;
                lo_b[d] = head;
                hi_b[d] = head + need;
                if (lane == 0) {
                    const unsigned char* wsrc =
                        slot < a.S ? reinterpret_cast<const unsigned char*>(a.w2_shared) +
                                         (size_t)tb->expert[slot] * w2_expert_bytes(a.H, a.I, a.G, false)
                                   : reinterpret_cast<const unsigned char*>(a.w2) +
                                         (size_t)tb->expert[slot] * w2_expert_bytes(a.H, a.I, a.G, i8);
                    wsrc += (size_t)blk * wbytes;
                    meta[d].slot = slot;
                    meta[d].blk = blk;
                    meta[d].off = head;
                    meta[d].hoff = hoff;
                    mbar_arrive_expect_tx(&full[d], wbytes + hbytes);
                    bulk_g2s(ring + head, wsrc, wbytes, &full[d]);
                    bulk_g2s(ring + head + hoff, a.h + (size_t)tb->base[slot] * a.I, hbytes, &full[d]);
                    unsigned long long* tr = trace_rec(a, 1, n);
                    if (tr) tr[4] = global_timer_ns();
                }
                __syncwarp();
                head += need;
                ++n;
            }
        }
        if (lane == 0) {
            if (ok) {
                // end marker in the next descriptor once it is free
                if (n >= kK3Desc && !mbar_wait(&empty[n % kK3Desc], ((n / kK3Desc) - 1) & 1, &a.ctl->status)) {
                    ok = false;
                } else {
                    meta[n % kK3Desc].slot = -1;
                    mbar_arrive(&full[n % kK3Desc]);
                }
            }
            if (!ok) {
                abort_flag = 1;
                for (int m = max(0, n - kK3Desc); m < n; ++m) mbar_wait(&full[m % kK3Desc], (m / kK3Desc) & 1, nullptr);
            }
        }
        __syncwarp();
    } else if (warp == kCW + 1) {
        // ---------------- publisher: count finished row groups, combine completed ones ----------------
        // One fence per item publishes the consumers' y rows (ordered before it by the done
        // barrier) device-wide before they are counted.
        pdl_wait_prior_grid();
        const unsigned nslot_all = (unsigned)(a.S + __ldcg(&a.table->U));
        for (int m = 0;; ++m) {
            const int d = m % kK3Desc;
            if (!mbar_wait_warp(&done[d], (m / kK3Desc) & 1, &abort_flag, &a.ctl->status)) break;
            const int slot = meta[d].slot, blk = meta[d].blk;
            if (slot < 0) break;
            __threadfence();
            const bool last = lane < kCW && atomicAdd(&a.row_done[blk * kCW + lane], 1u) == nslot_all - 1;
            unsigned mask = __ballot_sync(0xffffffffu, last);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[d]);
            if (mask) __threadfence();
            while (mask) {
                const int w = __ffs(mask) - 1;
                mask &= mask - 1;
                const int g = blk * kCW + w;
                combine_rows(a, g * 4, lane);
                __syncwarp();
                if (lane == 0) a.row_done[g] = 0;  // counters are left zeroed for the next launch
            }
        }
    } else {
        // ---------------- consumers ----------------
        for (int n = 0;; ++n) {
            const int d = n % kK3Desc;
            unsigned long long* tr = warp == 0 ? trace_rec(a, 1, n) : nullptr;
            if (tr && lane == 0) tr[0] = global_timer_ns();
            if (!mbar_wait_warp(&full[d], (n / kK3Desc) & 1, &abort_flag, &a.ctl->status)) break;
            const int slot = meta[d].slot, blk = meta[d].blk;
            if (slot >= 0) {
                if (tr && lane == 0) tr[1] = global_timer_ns();
                dn_item(a, *tb, slot, blk, ring + meta[d].off, meta[d].hoff, lane, warp);
                __syncwarp();
                if (tr && lane == 0) {
                    tr[2] = global_timer_ns();
                    tr[3] = ((unsigned long long)slot << 32) | (unsigned)blk;
                }
            }
            if (lane == 0) mbar_arrive(&done[d]);
            if (slot < 0) break;
        }
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
    max_smem -= 1024;  // the kernels' static shared memory (a few words) comes out of the same budget
    if (g_decode_trace) {
        a.trace = g_decode_trace;
        a.trace_items = (int)(g_decode_trace_bytes / (sizeof(unsigned long long) * 8 * (size_t)sms)) & ~1;
    }

    // ---- K2: route + gate/up; a stage holds one w13 block (the last one also the routing scratch)
    {
        uint32_t stage_bytes = (uint32_t)up(
            std::max({w13_block_bytes(a.H, a.G, false), a.int8 ? w13_block_bytes(a.H, a.G, true) : size_t(0),
                      sizeof(float) * 8 * kMaxB * 64}),
            128);
        const size_t off_tbl = 256;
        const size_t off_route = off_tbl + up(sizeof(SlotTable), 128);
        const size_t off_meta = off_route + up(sizeof(RouteSmem), 128);
        const size_t off_xs = off_meta + up(sizeof(ItemMeta) * 8, 128);
        const size_t off_stages = up(off_xs + sizeof(float) * a.B * a.H, 128);
        if ((size_t)max_smem < off_stages + 2 * (size_t)stage_bytes) return cudaErrorInvalidConfiguration;
        int nst = (int)std::min<size_t>(8, ((size_t)max_smem - off_stages) / stage_bytes);
        const size_t smem = off_stages + (size_t)nst * stage_bytes;
        err = ensure_smem_optin(reinterpret_cast<const void*>(decode_gate_up_kernel), smem);
        if (err != cudaSuccess) return err;
        uint32_t ot = (uint32_t)off_tbl, orr = (uint32_t)off_route, om = (uint32_t)off_meta, ox = (uint32_t)off_xs,
                 os = (uint32_t)off_stages;
        void* args[] = {&a, &nst, &stage_bytes, &ot, &orr, &om, &ox, &os};
        err = launch_pdl(reinterpret_cast<const void*>(decode_gate_up_kernel), dim3(sms), dim3(kThreads), smem, st,
                         args);
        if (err != cudaSuccess) return err;
    }
    // ---- K3: the rest of shared memory is the item ring
    {
        const size_t off_tbl = 256;
        const size_t off_meta = off_tbl + up(sizeof(SlotTable), 128);
        const size_t off_ring = off_meta + up(sizeof(ItemMeta) * kK3Desc, 128);
        const size_t max_item =
            up(std::max(w2_block_bytes(a.I, a.G, false), a.int8 ? w2_block_bytes(a.I, a.G, true) : size_t(0)), 16) +
            (size_t)kMaxB * a.I * 4;
        if ((size_t)max_smem < off_ring + 2 * max_item) return cudaErrorInvalidConfiguration;
        uint32_t ring_bytes = (uint32_t)(((size_t)max_smem - off_ring) & ~size_t(127));
        const size_t smem = off_ring + ring_bytes;
        err = ensure_smem_optin(reinterpret_cast<const void*>(decode_down_kernel), smem);
        if (err != cudaSuccess) return err;
        uint32_t ot = (uint32_t)off_tbl, om = (uint32_t)off_meta, orr = (uint32_t)off_ring;
        void* args[] = {&a, &ring_bytes, &ot, &om, &orr};
        err = launch_pdl(reinterpret_cast<const void*>(decode_down_kernel), dim3(sms), dim3(kThreads3), smem, st, args);
        if (err != cudaSuccess) return err;
    }
    return cudaGetLastError();
}

}  // namespace uocr
