// Decode-step MoE sublayer (MoE.decode_rows, unlimited_ocr_max/decoder.py:641-655) for B <= 8
// tokens, as ONE persistent kernel per layer. HBM-bound: the job is to stream the touched
// experts' weights at full bandwidth, once each.
//
// Pairs. Routed (token t, slot s) is pair t*k + s; shared expert q's copy of token t is pair
// k*B + q*B + t. Expert slots: 0..S-1 are the shared experts, S+u is the u-th distinct routed
// expert in ascending id (the reference's rows-grouped-by-expert, kernels/moe_routing.mojo).
//
// Work items, claimed in this order from an atomic queue (so an item only ever waits for
// items claimed before it, which are already running: no deadlock at any grid size):
//   ROUTE r   logits of experts [8r, 8r+8) for all B tokens; the last ROUTE item runs the
//             softmax + top-k (bit-exact with the oracle) and publishes the routing table;
//   GU        (slot, 8 intermediate rows): gate and up rows of the slot's expert, SwiGLU,
//             h[pair][n] for every pair on that expert -- each weight row read once;
//   DOWN      (slot, 16 output rows): y[pair][j] = Wd[e][j] . h[pair]; the last DOWN item of
//             an output block (all S + U slots done) combines
//             out[t][j] = sum_s w[t,s] y[t*k+s][j] + sum_q y_shared[q][t][j]   (fixed order).
// A warp-specialised CTA: one producer warp claims items and streams each item's weight rows
// with cp.async.bulk into a ring of shared-memory stages (mbarrier full/empty pairs); eight
// consumer warps compute from shared memory. A pair's arithmetic uses only its own token and
// expert, so every output row is bitwise independent of the batch it rides in.
//
// Every device-side wait is bounded (sm100.cuh: kWaitBudgetNs): on expiry it records a
// status code in the workspace and the kernel winds down. The control counters reset
// themselves at the end of each launch (the last CTA to finish clears them), so a
// zero-filled workspace stays valid across calls.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace uocr {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;       // 256
constexpr int kThreads = kConsumers + 32;              // + producer warp
constexpr int kRB = 8;                                 // intermediate rows per GU item
constexpr int kRJ = 16;                                // output rows per DOWN item
constexpr int kUnit = 64;                              // K elements per compute unit
constexpr int kPad = 68;                               // padded floats per 64-element slice
constexpr int kMaxB = 8;
constexpr int kRouteExperts = 8;                       // experts per ROUTE item
constexpr int kClaim = 4;                              // items claimed per queue atomic
constexpr int kMaxSlotsSm = 72;                        // shared (<= 8) + routed (<= 64) slots

enum ItemType : int { kDone = 0, kRoute = 1, kGateUp = 2, kDown = 3 };

struct ItemMeta {
    int type, slot, block, pad;
};

// Slots of this step: rows [0, S) the shared experts, [S, S+U) the routed experts.
struct SlotTable {
    int nslot;
    int pad[3];
    int expert[kMaxSlotsSm];
    int count[kMaxSlotsSm];
    int pair[kMaxSlotsSm][kMaxB];
    int token[kMaxSlotsSm][kMaxB];
    float weight[kMaxSlotsSm][kMaxB];
};

struct Smem {
    uint64_t* full;
    uint64_t* empty;
    ItemMeta* meta;
    SlotTable* tbl;
    float* xs;     // [B][H/64][68]
    float* hs;     // [8][I/64][68]
    float* part;   // partial sums
    unsigned char* stages;
    int* flag;     // small scratch ints
};

UOCR_DEV unsigned char* stage_ptr(const Smem& s, int st, uint32_t stage_bytes) {
    return s.stages + (size_t)st * stage_bytes;
}

// ---- item enumeration -------------------------------------------------------------------
struct Plan {
    int NR, NGB, NDB, MR, S;
    uint32_t total;
};

UOCR_DEV Plan make_plan(const DecodeArgs& a) {
    Plan p;
    p.NR = (a.E + kRouteExperts - 1) / kRouteExperts;
    p.NGB = a.I / kRB;
    p.NDB = a.H / kRJ;
    p.MR = min(a.E, a.topk * a.B);
    p.S = a.S;
    p.total = (uint32_t)((p.S + p.MR) * (p.NGB + p.NDB));
    return p;
}

// Main-queue item i (the ROUTE items have their own counter, one per claim).
UOCR_DEV void decode_item(const Plan& p, uint32_t i, int& type, int& slot, int& block) {
    const uint32_t gu = (uint32_t)(p.S + p.MR) * p.NGB;
    if (i < gu) { type = kGateUp; slot = (int)(i / p.NGB); block = (int)(i % p.NGB); return; }
    i -= gu;
    type = kDown; slot = (int)(i / p.NDB); block = (int)(i % p.NDB);
}

// ---- ROUTE -----------------------------------------------------------------------------------
// Thread (expert j, segment s) fma-chains router row j's segment s against every token (the
// oracle's order); segments summed in ascending order; bias added; logits to global. The last
// ROUTE item to finish runs softmax + top-k and publishes the routing grouped by expert.
UOCR_DEV void do_route(const DecodeArgs& a, const Smem& sm, const Plan& p, int r, const unsigned char* stage,
                      uint32_t row_stride, int ctid) {
    const int H = a.H, B = a.B, L = H / 8, NKX = H / kUnit;
    // thread (token group tg, expert jl, segment s): router row jl (staged) segment s against
    // tokens tg*TPG .. tg*TPG+TPG-1
    const int tg = ctid >> 6, jl = (ctid >> 3) & 7, s = ctid & 7;
    const int TPG = (B + 3) / 4;
    const int j = r * kRouteExperts + jl;
    if (j < a.E && tg * TPG < B) {
        float acc[2] = {0.0f, 0.0f};
        const uint16_t* wrow = reinterpret_cast<const uint16_t*>(stage + (size_t)jl * row_stride) + s * L;
        for (int kk = 0; kk < L; kk += 8) {
            float wf[8];
            unpack_bf16x8(*reinterpret_cast<const uint4*>(wrow + kk), wf);
            const int k0 = s * L + kk;
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
                const int b = tg * TPG + bb;
                if (bb < TPG && b < B) {
                    const float* xr = sm.xs + (b * NKX + k0 / kUnit) * kPad + (k0 % kUnit);  // 8 | 64: no straddle
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
            if (bb < TPG && b < B) sm.part[(jl * 8 + s) * kMaxB + b] = acc[bb];
        }
    }
    named_bar_sync(1, kConsumers);
    if (ctid < kRouteExperts * B) {
        const int jj = ctid / B, b = ctid % B, jg = r * kRouteExperts + jj;
        if (jg < a.E) {
            float total = sm.part[(jj * 8 + 0) * kMaxB + b];
#pragma unroll
            for (int q = 1; q < 8; ++q) total = __fadd_rn(total, sm.part[(jj * 8 + q) * kMaxB + b]);
            if (a.bias) total = __fadd_rn(total, a.bias[jg]);
            a.logits[b * 64 + jg] = total;
        }
    }
    named_bar_sync(1, kConsumers);
    if (ctid == 0) {
        __threadfence();
        sm.flag[0] = (atomicAdd(&a.ctl->route_done, 1u) == (uint32_t)p.NR - 1) ? 1 : 0;
    }
    named_bar_sync(1, kConsumers);
    if (!sm.flag[0]) return;
    __threadfence();
    int* ids_s = sm.flag + 16;                               // [kB]
    float* wts_s = reinterpret_cast<float*>(sm.flag + 16 + 64);  // [kB]
    const int warp = ctid >> 5, lane = ctid & 31, k = a.topk, E = a.E;
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
    named_bar_sync(1, kConsumers);
    // group by expert: thread e (< 64) owns expert e; its row is the number of used experts below it
    const int kB = k * B;
    int c = 0;
    if (ctid < 64) {
        for (int q = 0; q < kB; ++q) c += (ids_s[q] == ctid);
        const unsigned bal = __ballot_sync(0xffffffffu, c > 0);
        if (lane == 0) sm.flag[8 + warp] = (int)bal;
    }
    named_bar_sync(1, kConsumers);
    if (ctid < 64) {
        const unsigned long long used =
            (unsigned long long)(unsigned)sm.flag[8] | ((unsigned long long)(unsigned)sm.flag[9] << 32);
        if (c > 0) {
            const int u = __popcll(used & ((1ull << ctid) - 1ull));
            RouteTable* tb = a.table;
            int n = 0;
            for (int q = 0; q < kB; ++q) {
                if (ids_s[q] == ctid) {
                    tb->pair[u][n] = q;
                    tb->token[u][n] = q / k;
                    tb->weight[u][n] = wts_s[q];
                    ++n;
                }
            }
            tb->expert[u] = ctid;
            tb->count[u] = c;
        }
        if (ctid == 0) a.table->U = __popcll(used);
    }
    named_bar_sync(1, kConsumers);
    if (ctid == 0) {
        __threadfence();
        st_release_gpu(&a.ctl->route_ready, 1u);
    }
}

// ---- GU -----------------------------------------------------------------------------------------
template <bool kI8>
UOCR_DEV void gu_units(const DecodeArgs& a, const Smem& sm, int slot, int block, const unsigned char* stage,
                       uint32_t row_stride, int ctid) {
    const SlotTable& tb = *sm.tbl;
    const int H = a.H, NKX = H / kUnit, c = tb.count[slot];
    const int units = kRB * NKX;
    for (int u = ctid; u < units; u += kConsumers) {
        const int r = u % kRB, ks = u / kRB;
        const unsigned char* grow = stage + (size_t)r * row_stride;
        const unsigned char* urow = stage + (size_t)(kRB + r) * row_stride;
        float ag[kMaxB], au[kMaxB];
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) ag[q] = au[q] = 0.0f;
        if (!kI8) {
#pragma unroll 2
            for (int j = 0; j < kUnit / 8; ++j) {
                float fg[8], fu[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(grow + ks * kUnit * 2 + j * 16), fg);
                unpack_bf16x8(*reinterpret_cast<const uint4*>(urow + ks * kUnit * 2 + j * 16), fu);
#pragma unroll
                for (int q = 0; q < kMaxB; ++q) {
                    if (q < c) {
                        const float* xr = sm.xs + (tb.token[slot][q] * NKX + ks) * kPad + j * 8;
                        const float4 xa = *reinterpret_cast<const float4*>(xr);
                        const float4 xb = *reinterpret_cast<const float4*>(xr + 4);
                        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                        float g = ag[q], v = au[q];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            g = __fmaf_rn(fg[e], xv[e], g);
                            v = __fmaf_rn(fu[e], xv[e], v);
                        }
                        ag[q] = g;
                        au[q] = v;
                    }
                }
            }
        } else {
#pragma unroll 1
            for (int j = 0; j < kUnit / 16; ++j) {
                const uint4 wg = *reinterpret_cast<const uint4*>(grow + ks * kUnit + j * 16);
                const uint4 wu = *reinterpret_cast<const uint4*>(urow + ks * kUnit + j * 16);
                float fg[16], fu[16];
                unpack_s8x8(wg.x, wg.y, *reinterpret_cast<float(*)[8]>(fg));
                unpack_s8x8(wg.z, wg.w, *reinterpret_cast<float(*)[8]>(fg + 8));
                unpack_s8x8(wu.x, wu.y, *reinterpret_cast<float(*)[8]>(fu));
                unpack_s8x8(wu.z, wu.w, *reinterpret_cast<float(*)[8]>(fu + 8));
#pragma unroll
                for (int q = 0; q < kMaxB; ++q) {
                    if (q < c) {
                        const float* xr = sm.xs + (tb.token[slot][q] * NKX + ks) * kPad + j * 16;
                        float g = ag[q], v = au[q];
#pragma unroll
                        for (int h4 = 0; h4 < 4; ++h4) {
                            const float4 xv = *reinterpret_cast<const float4*>(xr + 4 * h4);
                            g = __fmaf_rn(fg[4 * h4 + 0], xv.x, g); v = __fmaf_rn(fu[4 * h4 + 0], xv.x, v);
                            g = __fmaf_rn(fg[4 * h4 + 1], xv.y, g); v = __fmaf_rn(fu[4 * h4 + 1], xv.y, v);
                            g = __fmaf_rn(fg[4 * h4 + 2], xv.z, g); v = __fmaf_rn(fu[4 * h4 + 2], xv.z, v);
                            g = __fmaf_rn(fg[4 * h4 + 3], xv.w, g); v = __fmaf_rn(fu[4 * h4 + 3], xv.w, v);
                        }
                        ag[q] = g;
                        au[q] = v;
                    }
                }
            }
            // the unit lies in one quantisation group: scale its partial sums (group sum, then scale)
            const int n = block * kRB + r;
            const int pg = (n / 128) * 256 + (n % 128);
            const size_t groups = (size_t)H / a.G;
            const float* sb = a.s13 + (size_t)tb.expert[slot] * 2 * a.I * groups;
            const float sg = __ldg(sb + (size_t)pg * groups + (ks * kUnit) / a.G);
            const float su = __ldg(sb + (size_t)(pg + 128) * groups + (ks * kUnit) / a.G);
#pragma unroll
            for (int q = 0; q < kMaxB; ++q) { ag[q] = __fmul_rn(ag[q], sg); au[q] = __fmul_rn(au[q], su); }
        }
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) {
            if (q < c) {
                sm.part[((r * NKX + ks) * kMaxB + q) * 2 + 0] = ag[q];
                sm.part[((r * NKX + ks) * kMaxB + q) * 2 + 1] = au[q];
            }
        }
    }
}

// ---- DOWN -------------------------------------------------------------------------------------
template <bool kI8>
UOCR_DEV void down_units(const DecodeArgs& a, const Smem& sm, int slot, int block, const unsigned char* stage,
                         uint32_t row_stride, int ctid) {
    const SlotTable& tb = *sm.tbl;
    const int I = a.I, NKI = I / kUnit, c = tb.count[slot];
    const int units = kRJ * NKI;
    for (int u = ctid; u < units; u += kConsumers) {
        const int r = u % kRJ, ks = u / kRJ;
        const unsigned char* wrow = stage + (size_t)r * row_stride;
        float acc[kMaxB];
#pragma unroll
        for (int q = 0; q < kMaxB; ++q) acc[q] = 0.0f;
        if (!kI8) {
#pragma unroll 2
            for (int j = 0; j < kUnit / 8; ++j) {
                float f[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(wrow + ks * kUnit * 2 + j * 16), f);
#pragma unroll
                for (int q = 0; q < kMaxB; ++q) {
                    if (q < c) {
                        const float* hr = sm.hs + (q * NKI + ks) * kPad + j * 8;
                        const float4 ha = *reinterpret_cast<const float4*>(hr);
                        const float4 hb = *reinterpret_cast<const float4*>(hr + 4);
                        float v = acc[q];
                        v = __fmaf_rn(f[0], ha.x, v); v = __fmaf_rn(f[1], ha.y, v);
                        v = __fmaf_rn(f[2], ha.z, v); v = __fmaf_rn(f[3], ha.w, v);
                        v = __fmaf_rn(f[4], hb.x, v); v = __fmaf_rn(f[5], hb.y, v);
                        v = __fmaf_rn(f[6], hb.z, v); v = __fmaf_rn(f[7], hb.w, v);
                        acc[q] = v;
                    }
                }
            }
        } else {
#pragma unroll 1
            for (int j = 0; j < kUnit / 16; ++j) {
                const uint4 w = *reinterpret_cast<const uint4*>(wrow + ks * kUnit + j * 16);
                float f[16];
                unpack_s8x8(w.x, w.y, *reinterpret_cast<float(*)[8]>(f));
                unpack_s8x8(w.z, w.w, *reinterpret_cast<float(*)[8]>(f + 8));
#pragma unroll
                for (int q = 0; q < kMaxB; ++q) {
                    if (q < c) {
                        const float* hr = sm.hs + (q * NKI + ks) * kPad + j * 16;
                        float v = acc[q];
#pragma unroll
                        for (int h4 = 0; h4 < 4; ++h4) {
                            const float4 hv = *reinterpret_cast<const float4*>(hr + 4 * h4);
                            v = __fmaf_rn(f[4 * h4 + 0], hv.x, v);
                            v = __fmaf_rn(f[4 * h4 + 1], hv.y, v);
                            v = __fmaf_rn(f[4 * h4 + 2], hv.z, v);
                            v = __fmaf_rn(f[4 * h4 + 3], hv.w, v);
                        }
                        acc[q] = v;
                    }
                }
            }
            const int jrow = block * kRJ + r;
            const size_t groups = (size_t)I / a.G;
            const float sc = __ldg(a.s2 + ((size_t)tb.expert[slot] * a.H + jrow) * groups + (ks * kUnit) / a.G);
#pragma unroll
            for (int q = 0; q < kMaxB; ++q) acc[q] = __fmul_rn(acc[q], sc);
        }
#pragma unroll
        for (int q = 0; q < kMaxB; ++q)
            if (q < c) sm.part[(r * NKI + ks) * kMaxB + q] = acc[q];
    }
}

// ---- producer warp --------------------------------------------------------------------------
// Lane 0 claims items kClaim at a time and drives the mbarriers; the whole warp copies the
// routing table into shared memory once and issues the bulk copies (one weight row per lane).
UOCR_DEV void producer_warp(const DecodeArgs& a, const Smem& sm, const Plan& p, int nst, uint32_t stage_bytes,
                            uint32_t gu_b16, uint32_t gu_i8, uint32_t dn_b16, uint32_t dn_i8, volatile int* abort_flag) {
    const int lane = threadIdx.x & 31;
    bool have_table = false;
    int n = 0;
    bool ok = true;
    uint32_t next = 0, left = 0;
    bool routes_left = true;
    while (true) {
        int type = kRoute, slot = 0, block = 0;
        if (routes_left) {
            uint32_t r = 0;
            if (lane == 0) r = atomicAdd(&a.ctl->route_q, 1u);
            r = __shfl_sync(0xffffffffu, r, 0);
            if (r < (uint32_t)p.NR) {
                block = (int)r;
            } else {
                routes_left = false;
            }
        }
        if (!routes_left) {
            if (left == 0) {
                uint32_t base = 0;
                if (lane == 0) base = atomicAdd(&a.ctl->queue, (uint32_t)kClaim);
                next = __shfl_sync(0xffffffffu, base, 0);
                left = kClaim;
            }
            const uint32_t i = next++;
            --left;
            if (i >= p.total) break;
            decode_item(p, i, type, slot, block);
        }
        if (type != kRoute && slot >= p.S) {
            if (!have_table) {
                int got = 1;
                if (lane == 0) got = wait_counter_geq(&a.ctl->route_ready, 1u, &a.ctl->status) ? 1 : 0;
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) { ok = false; break; }
                __syncwarp();
                const RouteTable* g = a.table;
                const int U = __ldcg(&g->U);
                for (int u = lane; u < U; u += 32) {
                    const int row = p.S + u;
                    sm.tbl->expert[row] = __ldcg(&g->expert[u]);
                    sm.tbl->count[row] = __ldcg(&g->count[u]);
#pragma unroll
                    for (int q = 0; q < kMaxB; ++q) {
                        sm.tbl->pair[row][q] = __ldcg(&g->pair[u][q]);
                        sm.tbl->token[row][q] = __ldcg(&g->token[u][q]);
                        sm.tbl->weight[row][q] = __ldcg(&g->weight[u][q]);
                    }
                }
                if (lane == 0) sm.tbl->nslot = p.S + U;
                __syncwarp();
                have_table = true;
            }
            if (slot >= sm.tbl->nslot) continue;  // no such routed expert this step
        }
        const int st = n % nst, round = n / nst;
        int got = 1;
        if (lane == 0 && round > 0) got = mbar_wait(&sm.empty[st], (round - 1) & 1, &a.ctl->status) ? 1 : 0;
        got = __shfl_sync(0xffffffffu, got, 0);
        if (!got) { ok = false; break; }
        if (lane == 0) {
            sm.meta[st].type = type;
            sm.meta[st].slot = slot;
            sm.meta[st].block = block;
        }
        unsigned char* dst = stage_ptr(sm, st, stage_bytes);
        if (type == kRoute) {
            // the ROUTE item's router rows
            const uint32_t rb = (uint32_t)a.H * 2;
            const int j0 = block * kRouteExperts;
            const int nrow = min(kRouteExperts, a.E - j0);
            if (lane == 0) mbar_arrive_expect_tx(&sm.full[st], (uint32_t)nrow * rb);
            __syncwarp();
            if (lane < nrow)
                bulk_g2s(dst + (size_t)lane * gu_b16, reinterpret_cast<const unsigned char*>(a.router) + (size_t)(j0 + lane) * rb,
                         rb, &sm.full[st]);
        } else {
            const bool shared = slot < p.S;
            const bool i8 = !shared && a.int8;
            const int expert = sm.tbl->expert[slot];
            if (type == kGateUp) {
                const uint32_t rb = (uint32_t)a.H * (i8 ? 1 : 2);
                const uint32_t stride = i8 ? gu_i8 : gu_b16;
                const unsigned char* base =
                    shared ? reinterpret_cast<const unsigned char*>(a.w13_shared) + (size_t)expert * 2 * a.I * rb
                           : reinterpret_cast<const unsigned char*>(a.w13) + (size_t)expert * 2 * a.I * rb;
                if (lane == 0) mbar_arrive_expect_tx(&sm.full[st], 2u * kRB * rb);
                __syncwarp();
                const int n0 = block * kRB;
                const int pg0 = (n0 / 128) * 256 + (n0 % 128);
                if (lane < 2 * kRB) {
                    const int r = lane % kRB;
                    const int prow = pg0 + r + (lane >= kRB ? 128 : 0);
                    bulk_g2s(dst + (size_t)lane * stride, base + (size_t)prow * rb, rb, &sm.full[st]);
                }
            } else {
                const uint32_t rb = (uint32_t)a.I * (i8 ? 1 : 2);
                const uint32_t stride = i8 ? dn_i8 : dn_b16;
                const unsigned char* base =
                    shared ? reinterpret_cast<const unsigned char*>(a.w2_shared) + (size_t)expert * a.H * rb
                           : reinterpret_cast<const unsigned char*>(a.w2) + (size_t)expert * a.H * rb;
                if (lane == 0) mbar_arrive_expect_tx(&sm.full[st], (uint32_t)kRJ * rb);
                __syncwarp();
                if (lane < kRJ)
                    bulk_g2s(dst + (size_t)lane * stride, base + (size_t)(block * kRJ + lane) * rb, rb, &sm.full[st]);
            }
        }
        __syncwarp();
        ++n;
    }
    if (!ok) {
        if (lane == 0) {
            *abort_flag = 1;
            // wait (bounded) for the copies already issued into stages the consumers may not drain
            for (int q = max(0, n - nst); q < n; ++q) mbar_wait(&sm.full[q % nst], (q / nst) & 1, nullptr);
        }
        __syncwarp();
        return;
    }
    if (lane == 0) {
        const int st = n % nst, round = n / nst;
        if (round > 0 && !mbar_wait(&sm.empty[st], (round - 1) & 1, &a.ctl->status)) {
            *abort_flag = 1;
        } else {
            sm.meta[st].type = kDone;
            mbar_arrive(&sm.full[st]);
        }
    }
    __syncwarp();
}

// ---- consumers ---------------------------------------------------------------------------------
UOCR_DEV void consumers(const DecodeArgs& a, const Smem& sm, const Plan& p, int nst, uint32_t stage_bytes,
                        uint32_t gu_b16, uint32_t gu_i8, uint32_t dn_b16, uint32_t dn_i8, volatile int* abort_flag,
                        int ctid) {
    const int NKX = a.H / kUnit, NKI = a.I / kUnit, B = a.B, k = a.topk, kB = k * B;
    const SlotTable& tb = *sm.tbl;
    int n = 0;
    int staged_slot = -1;
    unsigned long long* tr = a.trace ? a.trace + (size_t)blockIdx.x * a.trace_items * 4 : nullptr;
    while (true) {
        const int st = n % nst;
        const uint32_t parity = (n / nst) & 1;
        if (ctid == 0) {
            int ok = 1;
            const uint64_t t0 = global_timer_ns();
            if (tr && n < a.trace_items) tr[n * 4 + 0] = t0;
            while (!mbar_try_wait(&sm.full[st], parity)) {
                if (*abort_flag || global_timer_ns() - t0 > kWaitBudgetNs) {
                    set_status(&a.ctl->status, kStatusWaitTimeout);
                    ok = 0;
                    break;
                }
            }
            sm.flag[3] = ok;
            if (tr && n < a.trace_items) {
                tr[n * 4 + 1] = global_timer_ns();
                tr[n * 4 + 3] = ((unsigned long long)sm.meta[st].type << 48) | ((unsigned long long)sm.meta[st].slot << 24) |
                                (unsigned long long)sm.meta[st].block;
            }
        }
        named_bar_sync(1, kConsumers);
        if (!sm.flag[3]) break;
        const int type = sm.meta[st].type, slot = sm.meta[st].slot, block = sm.meta[st].block;
        if (type == kDone) break;
        const unsigned char* stage = stage_ptr(sm, st, stage_bytes);
        if (type == kRoute) {
            do_route(a, sm, p, block, stage, gu_b16, ctid);
            named_bar_sync(1, kConsumers);
            if (ctid == 0) mbar_arrive(&sm.empty[st]);
        } else if (type == kGateUp) {
            const bool i8 = slot >= p.S && a.int8;
            if (i8)
                gu_units<true>(a, sm, slot, block, stage, gu_i8, ctid);
            else
                gu_units<false>(a, sm, slot, block, stage, gu_b16, ctid);
            named_bar_sync(1, kConsumers);
            if (ctid == 0) mbar_arrive(&sm.empty[st]);  // stage consumed
            const int c = tb.count[slot];
            for (int t = ctid; t < kRB * c; t += kConsumers) {
                const int r = t / c, q = t % c;
                float g = sm.part[((r * NKX + 0) * kMaxB + q) * 2 + 0];
                float u = sm.part[((r * NKX + 0) * kMaxB + q) * 2 + 1];
                for (int ks = 1; ks < NKX; ++ks) {
                    g = __fadd_rn(g, sm.part[((r * NKX + ks) * kMaxB + q) * 2 + 0]);
                    u = __fadd_rn(u, sm.part[((r * NKX + ks) * kMaxB + q) * 2 + 1]);
                }
                a.h[(size_t)tb.pair[slot][q] * a.I + block * kRB + r] = silu(g) * u;
            }
            named_bar_sync(1, kConsumers);
            if (ctid == 0) {
                __threadfence();
                atomicAdd(&a.ctl->gu_done[slot], 1u);
            }
        } else {
            const int c = tb.count[slot];
            if (slot != staged_slot) {
                // the slot's gate/up must be complete before its h is read (one waiter per warp)
                if (ctid == 0) {
                    if (!wait_counter_geq(&a.ctl->gu_done[slot], (uint32_t)p.NGB, &a.ctl->status)) *abort_flag = 1;
                }
                named_bar_sync(1, kConsumers);
                for (int i = ctid; i < c * (a.I / 4); i += kConsumers) {
                    const int q = i / (a.I / 4), kk = (i % (a.I / 4)) * 4;
                    const float4 v = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)tb.pair[slot][q] * a.I + kk));
                    *reinterpret_cast<float4*>(sm.hs + (q * NKI + kk / kUnit) * kPad + (kk % kUnit)) = v;
                }
                named_bar_sync(1, kConsumers);
                staged_slot = slot;
            }
            const bool i8 = slot >= p.S && a.int8;
            if (i8)
                down_units<true>(a, sm, slot, block, stage, dn_i8, ctid);
            else
                down_units<false>(a, sm, slot, block, stage, dn_b16, ctid);
            named_bar_sync(1, kConsumers);
            if (ctid == 0) mbar_arrive(&sm.empty[st]);
            for (int t = ctid; t < kRJ * c; t += kConsumers) {
                const int r = t / c, q = t % c;
                float y = sm.part[(r * NKI + 0) * kMaxB + q];
                for (int ks = 1; ks < NKI; ++ks) y = __fadd_rn(y, sm.part[(r * NKI + ks) * kMaxB + q]);
                a.y[(size_t)tb.pair[slot][q] * a.H + block * kRJ + r] = y;
            }
            named_bar_sync(1, kConsumers);
            if (ctid == 0) {
                __threadfence();
                const uint32_t done = atomicAdd(&a.ctl->j_done[block], 1u) + 1u;
                int fin = 0;
                if (wait_counter_geq(&a.ctl->route_ready, 1u, &a.ctl->status))
                    fin = (done == (uint32_t)(p.S + __ldcg(&a.table->U))) ? 1 : 0;
                sm.flag[2] = fin;
                if (fin) __threadfence();
            }
            named_bar_sync(1, kConsumers);
            if (sm.flag[2]) {
                // the last DOWN item of this output block: out = sum_s w y_routed + sum_q y_shared
                for (int t = ctid; t < kRJ * B; t += kConsumers) {
                    const int r = t % kRJ, b = t / kRJ;
                    const int j = block * kRJ + r;
                    float acc = 0.0f;
                    for (int s = 0; s < k; ++s) {
                        const int pr = b * k + s;
                        acc = __fmaf_rn(__ldcg(a.wts + pr), __ldcg(a.y + (size_t)pr * a.H + j), acc);
                    }
                    for (int q = 0; q < a.S; ++q) acc = __fadd_rn(acc, __ldcg(a.y + (size_t)(kB + q * B + b) * a.H + j));
                    a.out[(size_t)b * a.H + j] = acc;
                }
            }
        }
        if (ctid == 0 && tr && n < a.trace_items) tr[n * 4 + 2] = global_timer_ns();
        ++n;
    }
}

// ---- the kernel ---------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
decode_layer_kernel(DecodeArgs a, int nst, uint32_t stage_bytes, uint32_t off_meta, uint32_t off_tbl, uint32_t off_xs,
                    uint32_t off_hs, uint32_t off_part, uint32_t off_flag, uint32_t off_stages) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ int abort_flag;
    Smem sm;
    sm.full = reinterpret_cast<uint64_t*>(smem);
    sm.empty = sm.full + nst;
    sm.meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    sm.tbl = reinterpret_cast<SlotTable*>(smem + off_tbl);
    sm.xs = reinterpret_cast<float*>(smem + off_xs);
    sm.hs = reinterpret_cast<float*>(smem + off_hs);
    sm.part = reinterpret_cast<float*>(smem + off_part);
    sm.flag = reinterpret_cast<int*>(smem + off_flag);
    sm.stages = smem + off_stages;
    const Plan p = make_plan(a);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        abort_flag = 0;
        fence_mbar_init();
    }
    // shared-expert slots are known before routing
    if (tid < a.S) {
        sm.tbl->expert[tid] = tid;
        sm.tbl->count[tid] = a.B;
        for (int t = 0; t < kMaxB; ++t) {
            sm.tbl->pair[tid][t] = a.topk * a.B + tid * a.B + t;
            sm.tbl->token[tid][t] = t;
            sm.tbl->weight[tid][t] = 1.0f;
        }
    }
    // stage the tokens: xs[b][k/64][k%64]
    const int NKX = a.H / kUnit;
    for (int i = tid; i < a.B * (a.H / 4); i += kThreads) {
        const int b = i / (a.H / 4), k = (i % (a.H / 4)) * 4;
        const float4 v = *reinterpret_cast<const float4*>(a.x + (size_t)b * a.H + k);
        *reinterpret_cast<float4*>(sm.xs + (b * NKX + k / kUnit) * kPad + (k % kUnit)) = v;
    }
    __syncthreads();

    const uint32_t gu_b16 = (uint32_t)a.H * 2 + 16, gu_i8 = (uint32_t)a.H + 16;
    const uint32_t dn_b16 = (uint32_t)a.I * 2 + 16, dn_i8 = (uint32_t)a.I + 16;
    if (tid >= kConsumers)
        producer_warp(a, sm, p, nst, stage_bytes, gu_b16, gu_i8, dn_b16, dn_i8, &abort_flag);
    else
        consumers(a, sm, p, nst, stage_bytes, gu_b16, gu_i8, dn_b16, dn_i8, &abort_flag, tid);
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&a.ctl->cta_done, 1u) == gridDim.x - 1) {
            // last CTA: leave the control block zeroed for the next launch (status stays)
            __threadfence();
            a.ctl->queue = 0;
            a.ctl->route_done = 0;
            a.ctl->route_ready = 0;
            a.ctl->route_q = 0;
            for (int s = 0; s < p.S + p.MR; ++s) a.ctl->gu_done[s] = 0;
            for (int j = 0; j < p.NDB; ++j) a.ctl->j_done[j] = 0;
            __threadfence();
            a.ctl->cta_done = 0;
        }
    }
}

// ---- host side ------------------------------------------------------------------------------------
static size_t up(size_t v, size_t a) { return (v + a - 1) / a * a; }

cudaError_t launch_decode_layer(const DecodeArgs& a, cudaStream_t st) {
    const int NKX = a.H / kUnit, NKI = a.I / kUnit;
    const uint32_t gu_stage_b16 = 2u * kRB * ((uint32_t)a.H * 2 + 16);
    const uint32_t dn_stage_b16 = (uint32_t)kRJ * ((uint32_t)a.I * 2 + 16);
    // shared experts are always bf16, so a stage must hold a bf16 item
    const uint32_t stage_bytes = (uint32_t)up(std::max(gu_stage_b16, dn_stage_b16), 128);
    const size_t xs_bytes = sizeof(float) * (size_t)a.B * NKX * kPad;
    const size_t hs_bytes = sizeof(float) * (size_t)a.B * NKI * kPad;
    const size_t part_bytes = sizeof(float) * std::max((size_t)kRB * NKX * kMaxB * 2,
                                                       std::max((size_t)kRJ * NKI * kMaxB, (size_t)64 * 8 * kMaxB));
    const size_t flag_bytes = sizeof(int) * (16 + 64 + 64);
    int dev = 0, max_smem = 0, sms = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int kMaxStages = 8;
    const size_t fixed = up(16 * kMaxStages, 128) + up(sizeof(ItemMeta) * kMaxStages, 128) + up(sizeof(SlotTable), 128) +
                         up(xs_bytes, 128) + up(hs_bytes, 128) + up(part_bytes, 128) + up(flag_bytes, 128) + 2048;
    const int nst = (int)std::min<size_t>(kMaxStages, ((size_t)max_smem - fixed) / stage_bytes);
    if (nst < 2) return cudaErrorInvalidConfiguration;
    size_t off = up(16 * (size_t)nst, 128);
    const size_t off_meta = off; off += up(sizeof(ItemMeta) * nst, 128);
    const size_t off_tbl = off; off += up(sizeof(SlotTable), 128);
    const size_t off_xs = off; off += up(xs_bytes, 128);
    const size_t off_hs = off; off += up(hs_bytes, 128);
    const size_t off_part = off; off += up(part_bytes, 128);
    const size_t off_flag = off; off += up(flag_bytes, 128);
    const size_t off_stages = up(off, 1024);
    const size_t smem = off_stages + (size_t)nst * stage_bytes;
    err = ensure_smem_optin(reinterpret_cast<const void*>(decode_layer_kernel), smem);
    if (err != cudaSuccess) return err;
    const int NR = (a.E + kRouteExperts - 1) / kRouteExperts;
    const int MR = std::min(a.E, a.topk * a.B);
    const long total = (long)(a.S + MR) * (a.I / kRB + a.H / kRJ);
    const int grid = (int)std::min<long>(NR + (total + kClaim - 1) / kClaim, (long)sms);
    DecodeArgs args = a;
    if (g_decode_trace) {
        args.trace = g_decode_trace;
        args.trace_items = (int)(g_decode_trace_bytes / (sizeof(unsigned long long) * 4 * (size_t)grid));
    }
    decode_layer_kernel<<<grid, kThreads, smem, st>>>(args, nst, stage_bytes, (uint32_t)off_meta, (uint32_t)off_tbl,
                                                     (uint32_t)off_xs, (uint32_t)off_hs, (uint32_t)off_part,
                                                     (uint32_t)off_flag, (uint32_t)off_stages);
    return cudaGetLastError();
}

}  // namespace uocr
