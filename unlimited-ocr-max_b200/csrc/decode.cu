// Decode-step MoE sublayer (MoE.decode_rows, unlimited_ocr_max/decoder.py:641-655) for B <= 8
// tokens: three kernels chained by programmatic dependent launch (PDL); K2 and K3 are persistent
// and stream their weights from HBM once.
//
//   K1 logits            one small CTA per routed expert: the fp32 router logits of the B tokens
//              in the oracle's order (router row fetched before the dependency wait).
//   K2 route + gate/up   every CTA finishes the routing itself from K1's logits (softmax, top-k:
//              bit-exact and identical in every CTA, so no grid-wide exchange) while its
//              producer already streams shared-expert blocks; the routing groups the step by
//              expert ("slots": 0..S-1 the shared experts, S+u the u-th distinct routed expert in
//              ascending id), each slot owning contiguous rows of the h and y scratch.
//              Items (slot, block of 8 or 16 row pairs) -> h[slot row][n] = silu(g) * u.
//   K3 down + combine    items (slot, 32 output rows) -> y[slot row][j]; then a grid barrier
//              (K3's CTAs, one per SM, are all resident) and every CTA sums its 1/grid slice of
//              the B x H outputs over each token's slots in a fixed order: out[t][j].
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
#include "mma.cuh"
#include "sm100.cuh"

namespace uocr {

constexpr int kCW = 8;                       // consumer warps (K2 and K3)
constexpr int kThreads = (kCW + 1) * 32;     // + producer warp
constexpr int kMaxB = 8;
constexpr int kMaxSlotsSm = 72;              // shared (<= 8) + routed (<= 64)
constexpr int kK3Desc = 8;                   // K3 items in flight (descriptor ring)
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
    signed char pos[kMaxSlotsSm][kMaxB];  // pos[slot][t]: entry of token t in the slot, -1 if none
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
            tb->pos[s][t] = t < a.B ? (signed char)t : (signed char)-1;
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

// ---- tensor-core tile products (mma.cuh) -------------------------------------------------
// Rows live in shared memory with a stride of `rowb` bytes; a k-step is 32 bytes of a row.
// Lane (g, t) loads 8 bytes at 8t of rows g and g + 8 of the 16-row tile starting at `rows_s`.
//
// s8 weights, int8-digit activations: k-steps [s0, s1) of the tile; digits `xd_s` in fragment
// order ([k-step][digit][lane] x 8 bytes), their scales sig[col * NG + group]; per-row weight
// scales at sc_s + 4 * (row * NG + group) for the tile's rows row0 + g, row0 + g + 8. Adds the
// fp32 products to acc (C layout: (g, 2t), (g, 2t + 1), (g + 8, 2t), (g + 8, 2t + 1)).
UOCR_DEV void mma_tile_s8(uint32_t rows_s, uint32_t rowb, int row0, uint32_t sc_s, int NG, int s0, int s1,
                          uint32_t xd_s, const float* sig, int lane, float (&acc)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t ra = rows_s + (uint32_t)g * rowb + 8u * t, rb = ra + 8u * rowb;
    for (int s = s0; s < s1;) {
        const int grp = s >> 2;
        const int se = min(s1, (grp + 1) << 2);
        int c[3][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}, {0, 0, 0, 0}};
        for (; s < se; ++s) {
            const uint2 A0 = lds_u64(ra + 32u * s), A1 = lds_u64(rb + 32u * s);
#pragma unroll
            for (int d = 0; d < 3; ++d) {
                const uint2 Bd = lds_u64(xd_s + 8u * ((s * 3 + d) * 32 + lane));
                mma_s8(c[d], A0.x, A1.x, A0.y, A1.y, Bd.x, Bd.y);
            }
        }
        const float slo = lds_f32(sc_s + 4u * ((row0 + g) * NG + grp));
        const float shi = lds_f32(sc_s + 4u * ((row0 + g + 8) * NG + grp));
        const float sg0 = sig[2 * t * NG + grp], sg1 = sig[(2 * t + 1) * NG + grp];
        acc[0] = __fmaf_rn(undigit(c[0][0], c[1][0], c[2][0]), slo * sg0, acc[0]);
        acc[1] = __fmaf_rn(undigit(c[0][1], c[1][1], c[2][1]), slo * sg1, acc[1]);
        acc[2] = __fmaf_rn(undigit(c[0][2], c[1][2], c[2][2]), shi * sg0, acc[2]);
        acc[3] = __fmaf_rn(undigit(c[0][3], c[1][3], c[2][3]), shi * sg1, acc[3]);
    }
}

// bf16 weights, fp32 activations xf (column n = row n of xf, stride ldx floats) split into
// three bf16 terms on the fly: k-steps [s0, s1) (16 values each).
UOCR_DEV void mma_tile_bf16(uint32_t rows_s, uint32_t rowb, int s0, int s1, uint32_t xf_s, int ldx, int lane,
                            float (&acc)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t ra = rows_s + (uint32_t)g * rowb + 8u * t, rb = ra + 8u * rowb;
    const uint32_t xa = xf_s + 4u * ((uint32_t)g * ldx + 4 * t);
    for (int s = s0; s < s1; ++s) {
        const uint2 A0 = lds_u64(ra + 32u * s), A1 = lds_u64(rb + 32u * s);
        const float4 v = lds_f128(xa + 64u * s);
        uint32_t b0[3], b1[3];
        bf16_terms(v.x, v.y, b0[0], b0[1], b0[2]);
        bf16_terms(v.z, v.w, b1[0], b1[1], b1[2]);
#pragma unroll
        for (int q = 0; q < 3; ++q) mma_bf16(acc, A0.x, A1.x, A0.y, A1.y, b0[q], b1[q]);
    }
}

// Digits of one 128-value group of one column: lane L holds values [4L, 4L + 4) of the group.
// Returns the group's scale (warp-uniform) and the lane's three digit words.
UOCR_DEV float group_digits(float4 v, uint32_t (&w)[3]) {
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float sg, inv;
    digit_scale(m, sg, inv);
    int d[4][3];
    to_digits(v.x, inv, d[0][0], d[0][1], d[0][2]);
    to_digits(v.y, inv, d[1][0], d[1][1], d[1][2]);
    to_digits(v.z, inv, d[2][0], d[2][1], d[2][2]);
    to_digits(v.w, inv, d[3][0], d[3][1], d[3][2]);
#pragma unroll
    for (int q = 0; q < 3; ++q) w[q] = pack_s8x4(d[0][q], d[1][q], d[2][q], d[3][q]);
    return sg;
}
// Index (in 32-bit words) of digit q of values k..k+3 (k a multiple of 4) of column col in the
// fragment-ordered digit buffer: k-step k / 32, fragment lane 4 col + (k % 32) / 8, half (k % 8) / 4.
UOCR_DEV int digit_word(int k, int col, int q) {
    return (((k >> 5) * 3 + q) * 32 + 4 * col + ((k & 31) >> 3)) * 2 + ((k & 7) >> 2);
}

// Activations of 8 columns (rows of xf, stride ldx; rows >= valid are zero) as int8 digits in
// fragment order, one power-of-two scale per column and 128-group (sig[col * K/128 + g]):
// warp w converts column w (kCW >= 8 warps).
UOCR_DEV void stage_digits(const float* xf, int ldx, int K, int valid, uint32_t* xd, float* sig, int warp, int lane) {
    if (warp >= kMaxB) return;
    const int col = warp, NG = K / 128;
    const float* row = xf + (size_t)col * ldx;
    const bool live = col < valid;
    for (int g = 0; g < NG; ++g) {
        const int k = 128 * g + 4 * lane;
        const float4 v = live ? *reinterpret_cast<const float4*>(row + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t w[3];
        const float sg = group_digits(v, w);
        if (lane == 0) sig[col * NG + g] = sg;
#pragma unroll
        for (int q = 0; q < 3; ++q) xd[digit_word(k, col, q)] = w[q];
    }
}

// ======================================================================================
// routing inside a CTA (the 8 consumer warps of K2)
// ======================================================================================
// Scratch of the step's routing in shared memory.
struct RouteSmem {
    float logits[kMaxB][64];
    float bias[64];
    unsigned long long mask[64];  // entries (token * k + r) routed to expert e
    int ids[kMaxB * kDecodeMaxTopk];
    float wts[kMaxB * kDecodeMaxTopk];
    int rowof[kMaxB * kDecodeMaxTopk];
    unsigned used[2];
    int wsum[2];
};

// The rest of MoEGate (decoder.py:500-514) for the B tokens, from K1's partials: logit = the 8
// segment partials added in ascending order, + bias; softmax with this build's exponential and
// a fixed butterfly sum; top-k by (p desc, index asc) — identical in every CTA. Then the slot
// table: routed slot u is the u-th used expert; its rows start after the shared experts' S * B
// rows, its entries in token order. CTA 0 also writes ids / wts and the global RouteTable (read
// by K3). The inputs arrive by bulk copies on `inb`: the partials into `part` (the last stage
// buffer, which the producer fills only after the table is ready), the digits and their scales
// (int8 layers), and the token rows into xs (rows B..7 zero).
UOCR_DEV void cta_route(const DecodeArgs& a, float* xs, int ldx, uint32_t* xd, float* xsig, float* part,
                        uint64_t* inb, volatile int* abort_flag, RouteSmem* rs, SlotTable* tb, int tid,
                        unsigned long long* ev) {
    const int warp = tid >> 5, lane = tid & 31;
    const int H = a.H, B = a.B, E = a.E, k = a.topk, kB = k * B;
    unsigned long long* rv = a.trace ? trace_rec(a, 0, a.trace_items / 2 - 2) : nullptr;  // diagnostics
    // before the wait: this call's inputs that no kernel of the step writes, and scratch resets
    if (tid < 64) {
        rs->bias[tid] = a.bias && tid < E ? a.bias[tid] : 0.0f;
        rs->mask[tid] = 0ull;
    }
    for (int i = tid; i < 64 * kMaxB; i += kCW * 32) tb->pos[a.S + i / kMaxB][i % kMaxB] = -1;
    pdl_wait_prior_grid();  // K1's partials and digits; through K1, the previous layer's output x
    if (ev && tid == 0) ev[1] = global_timer_ns();
    if (warp == 0) {
        const uint32_t pbytes = (uint32_t)B * 64 * 8 * 4;
        const uint32_t dbytes = a.int8 ? (uint32_t)H * 24 : 0u, sbytes = a.int8 ? 8u * (H / 128) * 4 : 0u;
        if (lane == 0) mbar_arrive_expect_tx(inb, pbytes + dbytes + sbytes + (uint32_t)B * H * 4);
        __syncwarp();
        if (lane == 0) bulk_g2s(part, a.logits, pbytes, inb);
        if (lane == 1 && dbytes) bulk_g2s(xd, a.xdig, dbytes, inb);
        if (lane == 2 && sbytes) bulk_g2s(xsig, a.xsig, sbytes, inb);
        if (lane >= 8 && lane < 8 + B) bulk_g2s(xs + (size_t)(lane - 8) * ldx, a.x + (size_t)(lane - 8) * H, H * 4, inb);
    }
    for (int i = B * (H / 4) + tid; i < kMaxB * (H / 4); i += kCW * 32)
        *reinterpret_cast<float4*>(xs + (size_t)(i / (H / 4)) * ldx + 4 * (i % (H / 4))) = make_float4(0.f, 0.f, 0.f, 0.f);
    if (!mbar_wait_warp(inb, 0, abort_flag, &a.ctl->status)) *abort_flag = 1;
    if (rv && tid == 0) rv[0] = global_timer_ns();
    for (int i = tid; i < B * 64; i += kCW * 32) {
        const float4 p0 = *reinterpret_cast<const float4*>(part + 8 * i);
        const float4 p1 = *reinterpret_cast<const float4*>(part + 8 * i + 4);
        float total = __fadd_rn(__fadd_rn(__fadd_rn(p0.x, p0.y), p0.z), p0.w);
        total = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(total, p1.x), p1.y), p1.z), p1.w);
        if (a.bias) total = __fadd_rn(total, rs->bias[i & 63]);
        rs->logits[i >> 6][i & 63] = total;
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    if (rv && tid == 0) rv[3] = global_timer_ns();
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
        // keys: bits of p + 1 (p >= 0, so the order of the keys is the order of p); 0 = no candidate
        uint32_t k0 = v0 ? __float_as_uint(__fdiv_rn(e0, sum)) + 1u : 0u;
        uint32_t k1 = v1 ? __float_as_uint(__fdiv_rn(e1, sum)) + 1u : 0u;
        for (int rr = 0; rr < k; ++rr) {
            const uint32_t mk = __reduce_max_sync(0xffffffffu, max(k0, k1));
            const unsigned b0 = __ballot_sync(0xffffffffu, k0 == mk), b1 = __ballot_sync(0xffffffffu, k1 == mk);
            const int bi = b0 ? __ffs(b0) - 1 : 31 + __ffs(b1);  // the lowest index of the largest p
            if (bi == lane) k0 = 0u;
            if (bi == lane + 32) k1 = 0u;
            if (lane == 0) {
                const float bp = __uint_as_float(mk - 1u);
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
    if (rv && tid == 0) rv[4] = global_timer_ns();
    // group by expert: entry q = token * k + r sets bit q of its expert's mask
    if (tid < kB) atomicOr(&rs->mask[rs->ids[tid]], 1ull << tid);
    named_bar_sync(kBarConsumers, kCW * 32);
    unsigned long long m = 0ull;
    int c = 0, incl = 0;
    if (tid < 64) {  // warps 0, 1: expert tid
        m = rs->mask[tid];
        c = __popcll(m);
        incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, off);
            if (lane >= off) incl += v;
        }
        const unsigned bal = __ballot_sync(0xffffffffu, c > 0);
        if (lane == 0) rs->used[warp] = bal;
        if (lane == 31) rs->wsum[warp] = incl;
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    const unsigned long long used = (unsigned long long)rs->used[0] | ((unsigned long long)rs->used[1] << 32);
    RouteTable* g = a.table;
    const bool pub = blockIdx.x == 0;  // CTA 0 publishes the table for K3
    if (tid < 64 && c > 0) {
        const int u = __popcll(used & ((1ull << tid) - 1ull));
        const int row = a.S + u;
        const int base = a.S * B + (incl - c) + (warp == 1 ? rs->wsum[0] : 0);
        tb->expert[row] = tid;
        tb->count[row] = c;
        tb->base[row] = base;
        if (pub) {
            g->expert[u] = tid;
            g->count[u] = c;
            g->base[u] = base;
        }
        int n = 0;
        for (unsigned long long mm = m; mm; mm &= mm - 1ull, ++n) {
            const int q = __ffsll((long long)mm) - 1, t = q / k;
            tb->pos[row][t] = (signed char)n;
            tb->token[row][n] = t;
            tb->weight[row][n] = rs->wts[q];
            rs->rowof[q] = base + n;
            if (pub) {
                g->token[u][n] = t;
                g->weight[u][n] = rs->wts[q];
            }
        }
    }
    if (tid == 0) {
        tb->nslot = a.S + __popcll(used);
        if (pub) g->U = __popcll(used);
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    if (rv && tid == 0) rv[5] = global_timer_ns();
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
    if (rv && tid == 0) rv[6] = global_timer_ns();
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
// K1: router logit partials and the activation digits
// ======================================================================================
// One warp per CTA. CTAs [0, 8E): expert e = c / 8, segment s = c % 8; lane t < B runs the
// oracle's chain for token t over segment s (fma in ascending k from +0) and writes the
// partial sum part[t][e][s]; K2 adds the 8 partials in ascending order plus the bias. The
// router segment is fetched before the dependency wait. CTAs [8E, 8E + 8 H/128): column
// t = d / (H/128), group g = d % (H/128): the int8 digits of x[t][128g, 128g + 128) in K2's
// fragment order plus the group's scale (zero digits for t >= B). Small CTAs (no shared
// memory) so several start beside the previous layer's K3 on every SM.
constexpr int kLogitSteps = 20;  // 8-element steps per segment held in registers (H <= 1280)

__global__ void __launch_bounds__(32)
decode_logits_kernel(DecodeArgs a) {
    const int c = blockIdx.x, lane = threadIdx.x;
    const int H = a.H;
    // diagnostics: start, past the dependency wait, done
    unsigned long long* ev = a.trace && c < 64 ? trace_rec(a, 1, a.trace_items / 2 - 2) : nullptr;
    if (ev && lane == 0) ev[0] = global_timer_ns();
    if (c < a.E * 8) {
        const int e = c >> 3, s = c & 7, L = H / 8, nit = L / 8;
        const uint16_t* w = a.router + (size_t)e * H + s * L;
        uint4 r[kLogitSteps];
        if (lane < a.B) {
#pragma unroll
            for (int i = 0; i < kLogitSteps; ++i)
                if (i < nit) r[i] = ldg_nc_v4(w + 8 * i);
        }
        pdl_launch_dependents();  // K2 launches now; it waits for this grid before it reads the partials
        pdl_wait_prior_grid();    // x is the previous layer's output
        if (ev && lane == 0) ev[1] = global_timer_ns();
        float acc = 0.0f;
        if (lane < a.B) {
            const float* x = a.x + (size_t)lane * H + s * L;
            if (nit <= kLogitSteps) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    constexpr int kHalf = kLogitSteps / 2;
                    float4 xv[2 * kHalf];  // this half's 8-element steps of x, all loads issued first
#pragma unroll
                    for (int i = 0; i < kHalf; ++i) {
                        const int q = half * kHalf + i;
                        if (q < nit) {
                            xv[2 * i] = __ldcg(reinterpret_cast<const float4*>(x + 8 * q));
                            xv[2 * i + 1] = __ldcg(reinterpret_cast<const float4*>(x + 8 * q + 4));
                        }
                    }
#pragma unroll
                    for (int i = 0; i < kHalf; ++i) {
                        const int q = half * kHalf + i;
                        if (q < nit) {
                            float f[8];
                            unpack_bf16x8(r[q], f);
                            const float x8[8] = {xv[2 * i].x,     xv[2 * i].y,     xv[2 * i].z,     xv[2 * i].w,
                                                 xv[2 * i + 1].x, xv[2 * i + 1].y, xv[2 * i + 1].z, xv[2 * i + 1].w};
#pragma unroll
                            for (int j = 0; j < 8; ++j) acc = __fmaf_rn(f[j], x8[j], acc);
                        }
                    }
                }
            } else {
                for (int kk = 0; kk < L; kk += 8) {
                    float f[8];
                    unpack_bf16x8(ldg_nc_v4(w + kk), f);
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc = __fmaf_rn(f[j], __ldcg(x + kk + j), acc);
                }
            }
            a.logits[((size_t)lane * 64 + e) * 8 + s] = acc;
        }
    } else {
        const int d = c - a.E * 8, NG = H / 128, t = d / NG, g = d % NG;
        pdl_launch_dependents();
        pdl_wait_prior_grid();
        const int k = 128 * g + 4 * lane;
        const float4 v = t < a.B ? __ldcg(reinterpret_cast<const float4*>(a.x + (size_t)t * H + k))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        uint32_t w[3];
        const float sg = group_digits(v, w);
        if (lane == 0) a.xsig[t * NG + g] = sg;
#pragma unroll
        for (int q = 0; q < 3; ++q) a.xdig[digit_word(k, t, q)] = w[q];
    }
    if (ev && lane == 0) ev[2] = global_timer_ns();
}

// ======================================================================================
// K2: route + gate/up + SwiGLU
// ======================================================================================
// Items: (slot, block) with I / P blocks per slot, P = 16 row pairs for int8 stacks and 8 for
// bf16 (one packed block, layout.h). Shared slots first (streamed while the CTA routes), then
// routed slots. In an item all 8 consumer warps split the block's K range: int8 blocks are two
// 16-row tiles (gate, up) x 4 K quarters, bf16 blocks one tile [8 gate | 8 up rows] x 8 K
// eighths; the partial sums meet in shared memory and the SwiGLU is applied per (pair, token).
UOCR_DEV int gu_pairs(const DecodeArgs& a, int slot) { return (slot >= a.S && a.int8) ? 16 : 8; }
// relative cost of one item (its bytes dominate; tokens ride along in the tensor-core product)
UOCR_DEV long long gu_cost(const DecodeArgs& a, const SlotTable&, int) { return 1; }

// Partial tiles of items n, n-1, n-2: item n's finish runs after item n+1's products, and a
// warp releases item n's buffer only after that finish.
constexpr int kRedBufs = 3;
struct GuSmem {
    float red[kRedBufs][kCW][16][8];
};

// The warp's partial tile of one item. int8 blocks: tile warp / 4 (gate, up), K quarter
// warp % 4 (H / 128 k-steps of 32); bf16 blocks: K eighth `warp` (H / 128 k-steps of 16).
// The activation fragments are read from shared memory in the loop: a compact loop runs
// faster here than one unrolled over register-held fragments (instruction fetch dominates).
UOCR_DEV void gu_partial(const DecodeArgs& a, bool i8, uint32_t stage_s, uint32_t xf_s, int ldx, uint32_t xd_s,
                         const float* xsig, int lane, int warp, float (&acc)[4]) {
    acc[0] = acc[1] = acc[2] = acc[3] = 0.0f;
    const int n = a.H / 128;  // k-steps per warp, both kinds
    if (i8) {
        const uint32_t rowb = (uint32_t)packed_row_bytes(a.H, true);
        const int tile = warp >> 2, s0 = (warp & 3) * n;
        const uint32_t rows = stage_s + (uint32_t)tile * 16 * rowb, sc = stage_s + 32 * rowb;
        mma_tile_s8(rows, rowb, tile * 16, sc, n, s0, s0 + n, xd_s, xsig, lane, acc);
    } else {
        const uint32_t rowb = (uint32_t)packed_row_bytes(a.H, false);
        mma_tile_bf16(stage_s, rowb, warp * n, warp * n + n, xf_s, ldx, lane, acc);
    }
}

UOCR_DEV void store_partial(float (&red)[kCW][16][8], int warp, int lane, const float (&acc)[4]) {
    const int g = lane >> 2, t = lane & 3;
    *reinterpret_cast<float2*>(&red[warp][g][2 * t]) = make_float2(acc[0], acc[1]);
    *reinterpret_cast<float2*>(&red[warp][g + 8][2 * t]) = make_float2(acc[2], acc[3]);
}

// h[slot row][blk * P + p] = silu(g) * u for the slot's tokens, from the partial tiles.
UOCR_DEV void gu_finish(const DecodeArgs& a, const SlotTable& tb, bool i8, int slot, int blk,
                        const float (&red)[kCW][16][8], int tid) {
    const int p = tid >> 3, n = tid & 7;
    float g = 0.0f, u = 0.0f;
    int P;
    if (i8) {
        P = 16;
        if (p >= 16) return;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            g += red[q][p][n];
            u += red[4 + q][p][n];
        }
    } else {
        P = 8;
        if (p >= 8) return;
#pragma unroll
        for (int w = 0; w < kCW; ++w) {
            g += red[w][p][n];
            u += red[w][8 + p][n];
        }
    }
    const int pos = tb.pos[slot][n];
    if (pos >= 0) a.h[(size_t)(tb.base[slot] + pos) * a.I + blk * P + p] = silu(g) * u;
}

__global__ void __launch_bounds__(kThreads, 1)
decode_gate_up_kernel(DecodeArgs a, int nst, uint32_t stage_bytes, uint32_t off_tbl, uint32_t off_route,
                      uint32_t off_meta, uint32_t off_gu, uint32_t off_xf, uint32_t off_xd, uint32_t off_sig,
                      uint32_t off_stages) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int abort_flag;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + nst;
    uint64_t* table_ready = empty + nst;
    uint64_t* redbar = table_ready + 1;  // [kRedBufs]: all warps' partial tiles of an item are stored
    uint64_t* inb = redbar + kRedBufs;   // the routing's inputs have arrived
    SlotTable* tb = reinterpret_cast<SlotTable*>(smem + off_tbl);
    RouteSmem* rs = reinterpret_cast<RouteSmem*>(smem + off_route);
    ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    GuSmem* gs = reinterpret_cast<GuSmem*>(smem + off_gu);
    float* xf = reinterpret_cast<float*>(smem + off_xf);
    uint32_t* xd = reinterpret_cast<uint32_t*>(smem + off_xd);
    float* xsig = reinterpret_cast<float*>(smem + off_sig);
    unsigned char* stages = smem + off_stages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ldx = a.H + 4;
    // diagnostics: kernel-level events of this CTA (start, consumers past the dependency wait,
    // routed, fragments loaded, consumers done)
    unsigned long long* ev = a.trace ? trace_rec(a, 0, a.trace_items / 2 - 1) : nullptr;
    if (ev && tid == 0) ev[0] = global_timer_ns();
    if (tid == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        mbar_init(table_ready, 1);
        for (int b = 0; b < kRedBufs; ++b) mbar_init(&redbar[b], kCW);
        mbar_init(inb, 1);
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
            // the last stage holds the routing's logit partials until the table is ready
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
            auto cost = [&](int s) { return gu_cost(a, *tb, s); };
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
        // ---------------- consumers: route, stage the digits, then the items ----------------
        cta_route(a, xf, ldx, xd, xsig, reinterpret_cast<float*>(stages + (size_t)(nst - 1) * stage_bytes), inb,
                  &abort_flag, rs, tb, tid, ev);
        if (tid == 0) mbar_arrive(table_ready);
        if (ev && tid == 0) ev[2] = ev[5] = global_timer_ns();
        const uint32_t xf_s = smem_addr(xf), xd_s = smem_addr(xd);
        // this warp's activation fragments, fixed for the CTA
        if (ev && tid == 0) ev[3] = global_timer_ns();
        // Item n: products, stage release, partial tile stored; then item n-1 is finished (its
        // partial tiles are complete once every warp has arrived) and item n's buffer released.
        int pend_slot = -1, pend_blk = 0, pend_n = 0;
        bool pend_i8 = false, ok = true;
        auto finish_pending = [&]() {
            const int b = pend_n % kRedBufs;
            ok = mbar_wait_warp(&redbar[b], (pend_n / kRedBufs) & 1, &abort_flag, &a.ctl->status);
            if (ok) gu_finish(a, *tb, pend_i8, pend_slot, pend_blk, gs->red[b], tid);
        };
        for (int n = 0;; ++n) {
            const int st = n % nst;
            unsigned long long* tr = warp == 0 ? trace_rec(a, 0, n) : nullptr;
            if (tr && lane == 0) tr[0] = global_timer_ns();
            if (!mbar_wait_warp(&full[st], (n / nst) & 1, &abort_flag, &a.ctl->status)) {
                ok = false;
                break;
            }
            const int slot = meta[st].slot, blk = meta[st].blk;
            if (slot < 0) break;
            if (tr && lane == 0) tr[1] = global_timer_ns();
            const bool i8 = slot >= a.S && a.int8;
            const uint32_t stage_s = launder(smem_addr(stages + (size_t)st * stage_bytes));
            float acc[4];
            gu_partial(a, i8, stage_s, xf_s, ldx, xd_s, xsig, lane, warp, acc);
            fence_regs(acc);
            __syncwarp();
            if (tr && lane == 0) tr[5] = global_timer_ns();
            if (lane == 0) mbar_arrive(&empty[st]);  // the stage is free once the warp's products are done
            store_partial(gs->red[n % kRedBufs], warp, lane, acc);
            if (pend_slot >= 0) {
                finish_pending();
                if (!ok) break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&redbar[n % kRedBufs]);
            if (tr && lane == 0) {
                tr[6] = global_timer_ns();
                tr[2] = global_timer_ns();
                tr[3] = ((unsigned long long)slot << 32) | (unsigned)blk;
            }
            pend_slot = slot;
            pend_blk = blk;
            pend_i8 = i8;
            pend_n = n;
        }
        if (ok && pend_slot >= 0) finish_pending();
        if (ev && tid == 0) ev[4] = global_timer_ns();
    }
}

// ======================================================================================
// K3: down + combine
// ======================================================================================
// Items: (slot, 32-row block) with H / 32 blocks per slot, each one bulk copy of its weight
// block; the first item of each run of a slot in this CTA also carries the slot's h rows. At a
// run's start the consumers stage those rows (fp32, padded) and, for int8 weights, their digits.
// All 8 warps split each item: two 16-row tiles x 4 K quarters.
UOCR_DEV long long dn_cost(const DecodeArgs& a, const SlotTable&, int slot) {
    return (slot >= a.S && a.int8) ? 1 : 2;  // bf16 blocks are twice the bytes
}

struct DnSmem {
    float red[kRedBufs][kCW][16][8];
};

// y[slot row][blk * 32 + row] for the slot's tokens, from the partial tiles.
UOCR_DEV void dn_finish(const DecodeArgs& a, const SlotTable& tb, int slot, int blk, const float (&red)[kCW][16][8],
                        int tid) {
    const int row = tid >> 3, n = tid & 7;
    if (n >= tb.count[slot]) return;
    const int tile = row >> 4, r16 = row & 15;
    float y = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) y += red[tile * 4 + q][r16][n];
    a.y[(size_t)(tb.base[slot] + n) * a.H + blk * kW2Rows + row] = y;
}

// This CTA's share of the outputs, after every CTA's items (grid barrier): out[t][j] for the
// flat indices [lo, hi) of the B x H output, one per thread: token t's shared rows in order,
// then its routed rows in ascending expert id (w * y), from the slot table's row lists.
UOCR_DEV void combine_slice(const DecodeArgs& a, const int (&trow)[kMaxB][kDecodeMaxTopk],
                            const float (&tw)[kMaxB][kDecodeMaxTopk], int tid) {
    const int total = a.B * a.H;
    const int lo = (int)((long long)total * blockIdx.x / gridDim.x);
    const int hi = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
    for (int o = lo + tid; o < hi; o += blockDim.x) {
        const int t = o / a.H, j = o - t * a.H;
        float ys[kDecodeMaxShared], yr[kDecodeMaxTopk];
#pragma unroll
        for (int q = 0; q < kDecodeMaxShared; ++q)
            if (q < a.S) ys[q] = __ldcg(a.y + (size_t)(q * a.B + t) * a.H + j);
#pragma unroll
        for (int s = 0; s < kDecodeMaxTopk; ++s)
            if (s < a.topk) yr[s] = __ldcg(a.y + (size_t)trow[t][s] * a.H + j);
        float acc = 0.0f;
#pragma unroll
        for (int q = 0; q < kDecodeMaxShared; ++q)
            if (q < a.S) acc = __fadd_rn(acc, ys[q]);
#pragma unroll
        for (int s = 0; s < kDecodeMaxTopk; ++s)
            if (s < a.topk) acc = __fmaf_rn(tw[t][s], yr[s], acc);
        a.out[o] = acc;
    }
}

__global__ void __launch_bounds__(kThreads, 1)
decode_down_kernel(DecodeArgs a, uint32_t ring_bytes, uint32_t off_tbl, uint32_t off_meta, uint32_t off_dn,
                   uint32_t off_hf, uint32_t off_hd, uint32_t off_sig, uint32_t off_ring) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int abort_flag, bar_ok;
    __shared__ int trow[kMaxB][kDecodeMaxTopk];
    __shared__ float tw[kMaxB][kDecodeMaxTopk];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* freed = full + kK3Desc;    // consumers: the item's ring bytes are no longer read
    uint64_t* empty = freed + kK3Desc;   // consumers: the item is finished, its descriptor free
    uint64_t* redbar = empty + kK3Desc;     // [kRedBufs]
    uint64_t* hbar = redbar + kRedBufs;     // [2]: the run's h staged by all warps
    SlotTable* tb = reinterpret_cast<SlotTable*>(smem + off_tbl);
    ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    DnSmem* ds = reinterpret_cast<DnSmem*>(smem + off_dn);
    float* hf = reinterpret_cast<float*>(smem + off_hf);
    uint32_t* hd = reinterpret_cast<uint32_t*>(smem + off_hd);
    float* hsig = reinterpret_cast<float*>(smem + off_sig);
    unsigned char* ring = smem + off_ring;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nblk = a.H / kW2Rows, ldh = a.I + 4;
    unsigned long long* ev = a.trace ? trace_rec(a, 1, a.trace_items / 2 - 1) : nullptr;
    if (ev && tid == 0) ev[0] = global_timer_ns();
    if (tid == 0) {
        for (int s = 0; s < kK3Desc; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&freed[s], kCW);
            mbar_init(&empty[s], kCW);
        }
        for (int s = 0; s < kRedBufs; ++s) mbar_init(&redbar[s], kCW);
        for (int s = 0; s < 2; ++s) mbar_init(&hbar[s], kCW);
        abort_flag = 0;
        fence_mbar_init();
        pdl_launch_dependents();  // the next layer's kernel waits for this grid itself
    }
    load_shared_slots(tb, a, tid, blockDim.x);
    __syncthreads();

    if (warp == kCW) {
        // ---------------- producer ----------------
        // Items are placed back to back in the ring (wrapping to 0 when one does not fit). Ring
        // bytes retire in order as the consumers finish their products (`freed`); descriptors
        // retire in order as the consumers finish the items (`empty`). An item may be placed
        // once its descriptor is free and no item still being read overlaps its bytes.
        uint32_t lo_b[kK3Desc], hi_b[kK3Desc];  // byte range of descriptor d's item
        int n = 0, oldest = 0, oldest_desc = 0;
        uint32_t head = 0;
        bool ok = true;
        pdl_wait_prior_grid();  // h and the routing table come from K2
        if (ev && lane == 0) ev[1] = global_timer_ns();
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
            for (int blk = j0; blk < j1 && ok; ++blk) {
                const uint32_t hbytes = blk == j0 ? (uint32_t)tb->count[slot] * a.I * 4 : 0u;  // run start
                const uint32_t need = hoff + hbytes;
                if (head + need > ring_bytes) head = 0;
                // retire ring bytes until this item's do not overlap any still being read
                while (oldest < n) {
                    bool clash = false;
                    for (int m = oldest; m < n && !clash; ++m) {
                        const int d = m % kK3Desc;
                        clash = head < hi_b[d] && lo_b[d] < head + need;
                    }
                    if (!clash) break;
                    if (!mbar_wait_warp(&freed[oldest % kK3Desc], (oldest / kK3Desc) & 1, &abort_flag,
                                        &a.ctl->status)) {
                        ok = false;
                        break;
                    }
                    ++oldest;
                }
                // and the descriptor: item n reuses item n - kK3Desc's
                while (ok && n - oldest_desc >= kK3Desc) {
                    if (!mbar_wait_warp(&empty[oldest_desc % kK3Desc], (oldest_desc / kK3Desc) & 1, &abort_flag,
                                        &a.ctl->status))
                        ok = false;
                    ++oldest_desc;
                }
                // a retired descriptor's bytes were freed before it: never wait on that `freed`
                // phase again (its barrier may complete again for a later item)
                oldest = max(oldest, oldest_desc);
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
                    meta[d].hoff = hbytes ? hoff : 0u;  // 0: no h with this item
                    mbar_arrive_expect_tx(&full[d], wbytes + hbytes);
                    bulk_g2s(ring + head, wsrc, wbytes, &full[d]);
                    if (hbytes) bulk_g2s(ring + head + hoff, a.h + (size_t)tb->base[slot] * a.I, hbytes, &full[d]);
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
    } else {
        // ---------------- consumers ----------------
        const uint32_t hf_s = smem_addr(hf), hd_s = smem_addr(hd);
        int runs = 0;
        const int tile = warp >> 2, q = warp & 3;
        const int n8 = a.I / 128, n16 = a.I / 64;  // k-steps per warp (s8 32-wide, bf16 16-wide)
        // As in K2: item n's products, then item n-1 is finished (y rows written, its descriptor
        // released), then item n's partial tile buffer is released.
        int pend_slot = -1, pend_blk = 0, pend_n = 0, pend_d = 0;
        bool ok = true;
        auto finish_pending = [&]() {
            const int b = pend_n % kRedBufs;
            ok = mbar_wait_warp(&redbar[b], (pend_n / kRedBufs) & 1, &abort_flag, &a.ctl->status);
            if (!ok) return;
            dn_finish(a, *tb, pend_slot, pend_blk, ds->red[b], tid);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[pend_d]);
        };
        for (int n = 0;; ++n) {
            const int d = n % kK3Desc;
            unsigned long long* tr = warp == 0 ? trace_rec(a, 1, n) : nullptr;
            if (tr && lane == 0) tr[0] = global_timer_ns();
            if (!mbar_wait_warp(&full[d], (n / kK3Desc) & 1, &abort_flag, &a.ctl->status)) {
                ok = false;
                break;
            }
            const int slot = meta[d].slot, blk = meta[d].blk;
            if (slot < 0) {
                if (pend_slot >= 0) finish_pending();
                pend_slot = -1;
                break;
            }
            if (tr && lane == 0) tr[1] = global_timer_ns();
            const bool i8 = slot >= a.S && a.int8;
            const uint32_t item_s = launder(smem_addr(ring + meta[d].off));
            if (meta[d].hoff) {
                // a run of this slot starts: every warp's products of the previous item must be
                // done before the caches change (their partial tiles are all stored)
                if (pend_slot >= 0 && !mbar_wait_warp(&redbar[pend_n % kRedBufs], (pend_n / kRedBufs) & 1,
                                                      &abort_flag, &a.ctl->status)) {
                    ok = false;
                    break;
                }
                // stage its h rows (fp32, padded; rows >= count zero) and, for int8 weights, their digits
                const float* hsrc = reinterpret_cast<const float*>(ring + meta[d].off + meta[d].hoff);
                const int cnt = tb->count[slot];
                for (int i = tid; i < kMaxB * (a.I / 4); i += kCW * 32) {
                    const int qq = i / (a.I / 4), c4 = i % (a.I / 4);
                    const float4 v = qq < cnt ? *reinterpret_cast<const float4*>(hsrc + (size_t)qq * a.I + 4 * c4)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
                    *reinterpret_cast<float4*>(hf + (size_t)qq * ldh + 4 * c4) = v;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&hbar[runs & 1]);
                if (!mbar_wait_warp(&hbar[runs & 1], (runs >> 1) & 1, &abort_flag, &a.ctl->status)) {
                    ok = false;
                    break;
                }
                ++runs;
                if (i8) {
                    stage_digits(hf, ldh, a.I, cnt, hd, hsig, warp, lane);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&hbar[runs & 1]);
                    if (!mbar_wait_warp(&hbar[runs & 1], (runs >> 1) & 1, &abort_flag, &a.ctl->status)) {
                        ok = false;
                        break;
                    }
                    ++runs;
                }
            }
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            if (i8) {
                const uint32_t rowb = (uint32_t)packed_row_bytes(a.I, true);
                const int NG = a.I / 128;
                const uint32_t rows = item_s + (uint32_t)tile * 16 * rowb, sc = item_s + kW2Rows * rowb;
                mma_tile_s8(rows, rowb, tile * 16, sc, NG, q * n8, q * n8 + n8, hd_s, hsig, lane, acc);
            } else {
                const uint32_t rowb = (uint32_t)packed_row_bytes(a.I, false);
                const uint32_t rows = item_s + (uint32_t)tile * 16 * rowb;
                mma_tile_bf16(rows, rowb, q * n16, q * n16 + n16, hf_s, ldh, lane, acc);
            }
            fence_regs(acc);
            __syncwarp();
            if (tr && lane == 0) tr[5] = global_timer_ns();
            if (lane == 0) mbar_arrive(&freed[d]);  // the item's ring bytes are no longer read
            store_partial(ds->red[n % kRedBufs], warp, lane, acc);
            if (pend_slot >= 0) {
                finish_pending();
                if (!ok) break;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&redbar[n % kRedBufs]);
            if (tr && lane == 0) {
                tr[6] = global_timer_ns();
                tr[2] = global_timer_ns();
                tr[3] = ((unsigned long long)slot << 32) | (unsigned)blk;
            }
            pend_slot = slot;
            pend_blk = blk;
            pend_n = n;
            pend_d = d;
        }
        if (ev && tid == 0) ev[2] = global_timer_ns();
    }

    // ---------------- combine: every CTA's y rows are written (grid barrier) ----------------
    pdl_wait_prior_grid();  // the routing table (K2); already complete for the producer
    const int tk = tid / kDecodeMaxTopk, ts = tid % kDecodeMaxTopk;
    if (tk < kMaxB) {
        const bool v = tk < a.B && ts < a.topk;
        trow[tk][ts] = v ? __ldcg(&a.table->tok_row[tk][ts]) : 0;
        tw[tk][ts] = v ? __ldcg(&a.table->tok_w[tk][ts]) : 0.0f;
    }
    const bool ok = grid_barrier(&a.ctl->bar_count, &a.ctl->bar_epoch, &a.ctl->status, &bar_ok);
    if (ev && tid == 0) ev[3] = global_timer_ns();
    if (ok && !abort_flag && __ldcg(&a.ctl->status) == 0) combine_slice(a, trow, tw, tid);
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
    int sm_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&sm_smem, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // K2 / K3 leave room on their SM for their own static shared memory (< 1 KB) and their
    // reservation, and for K1's CTAs (no shared memory, 1 KB reservation each), so K1 can start
    // beside them
    const int k1_ctas = a.E * 8 + kMaxB * (a.H / 128);
    const int k1_per_sm = (k1_ctas + sms - 1) / sms;
    max_smem = std::min(max_smem - 1024, sm_smem - 1024 - 1024 - 1024 * k1_per_sm);
    if (g_decode_trace) {
        a.trace = g_decode_trace;
        a.trace_items = (int)(g_decode_trace_bytes / (sizeof(unsigned long long) * 8 * (size_t)sms)) & ~1;
    }

    // ---- K1: logit partials (one CTA per expert and segment) and the activation digits
    {
        void* args[] = {&a};
        err = launch_pdl(reinterpret_cast<const void*>(decode_logits_kernel), dim3(k1_ctas), dim3(32), 0, st, args);
        if (err != cudaSuccess) return err;
    }
    // ---- K2: route + gate/up; a stage holds one w13 block
    {
        uint32_t stage_bytes = (uint32_t)up(
            std::max({w13_block_bytes(a.H, a.G, false), a.int8 ? w13_block_bytes(a.H, a.G, true) : size_t(0),
                      sizeof(float) * kMaxB * 64 * 8}),  // the last stage first holds the logit partials
            128);
        const size_t off_tbl = 256;
        const size_t off_route = off_tbl + up(sizeof(SlotTable), 128);
        const size_t off_meta = off_route + up(sizeof(RouteSmem), 128);
        const size_t off_gu = off_meta + up(sizeof(ItemMeta) * 8, 128);
        const size_t off_xf = off_gu + up(sizeof(GuSmem), 128);
        const size_t off_xd = off_xf + up(sizeof(float) * kMaxB * (a.H + 4), 128);
        const size_t xd_bytes = a.int8 ? (size_t)(a.H / 32) * 3 * 32 * 8 : 0;
        const size_t off_sig = off_xd + up(xd_bytes, 128);
        const size_t off_stages = up(off_sig + sizeof(float) * kMaxB * (a.H / 128), 128);
        if ((size_t)max_smem < off_stages + 2 * (size_t)stage_bytes) return cudaErrorInvalidConfiguration;
        int nst = (int)std::min<size_t>(8, ((size_t)max_smem - off_stages) / stage_bytes);
        const size_t smem = off_stages + (size_t)nst * stage_bytes;
        const void* k2 = reinterpret_cast<const void*>(decode_gate_up_kernel);
        err = ensure_smem_optin(k2, smem);
        if (err != cudaSuccess) return err;
        uint32_t o[8] = {(uint32_t)off_tbl, (uint32_t)off_route, (uint32_t)off_meta, (uint32_t)off_gu,
                         (uint32_t)off_xf,  (uint32_t)off_xd,    (uint32_t)off_sig,  (uint32_t)off_stages};
        void* args[] = {&a, &nst, &stage_bytes, &o[0], &o[1], &o[2], &o[3], &o[4], &o[5], &o[6], &o[7]};
        err = launch_pdl(k2, dim3(sms), dim3(kThreads), smem, st, args);
        if (err != cudaSuccess) return err;
    }
    // ---- K3: the rest of shared memory is the item ring
    {
        const size_t off_tbl = 512;  // 3 x kK3Desc + kRedBufs + 2 mbarriers before it
        const size_t off_meta = off_tbl + up(sizeof(SlotTable), 128);
        const size_t off_dn = off_meta + up(sizeof(ItemMeta) * kK3Desc, 128);
        const size_t off_hf = off_dn + up(sizeof(DnSmem), 128);
        const size_t off_hd = off_hf + up(sizeof(float) * kMaxB * (a.I + 4), 128);
        const size_t hd_bytes = a.int8 ? (size_t)(a.I / 32) * 3 * 32 * 8 : 0;
        const size_t off_sig = off_hd + up(hd_bytes, 128);
        const size_t off_ring = up(off_sig + sizeof(float) * kMaxB * (a.I / 128), 128);
        const size_t max_item =
            up(std::max(w2_block_bytes(a.I, a.G, false), a.int8 ? w2_block_bytes(a.I, a.G, true) : size_t(0)), 16) +
            (size_t)kMaxB * a.I * 4;
        if ((size_t)max_smem < off_ring + max_item) return cudaErrorInvalidConfiguration;
        uint32_t ring_bytes = (uint32_t)(((size_t)max_smem - off_ring) & ~size_t(127));
        const size_t smem = off_ring + ring_bytes;
        const void* k3 = reinterpret_cast<const void*>(decode_down_kernel);
        err = ensure_smem_optin(k3, smem);
        if (err != cudaSuccess) return err;
        uint32_t o[7] = {(uint32_t)off_tbl, (uint32_t)off_meta, (uint32_t)off_dn, (uint32_t)off_hf,
                         (uint32_t)off_hd,  (uint32_t)off_sig,  (uint32_t)off_ring};
        void* args[] = {&a, &ring_bytes, &o[0], &o[1], &o[2], &o[3], &o[4], &o[5], &o[6]};
        err = launch_pdl(k3, dim3(sms), dim3(kThreads), smem, st, args);
        if (err != cudaSuccess) return err;
    }
    return cudaGetLastError();
}

}  // namespace uocr
