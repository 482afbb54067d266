// Decode-step MoE sublayer (MoE.decode_rows, unlimited_ocr_max/decoder.py:641-655) for B <= 8
// tokens: two kernels chained by programmatic dependent launch (PDL). The experts kernel is
// persistent (one CTA per SM) and streams every weight byte of the step from HBM once, through
// the tcgen05 tensor cores.
//
//   K1 logits + operands   one warp per CTA: the fp32 router logit partials of (expert,
//              segment) in the oracle's order, and the tokens as tensor-core B operands
//              (int8 digits, bf16 terms) in the swizzled shared-memory image.
//   experts    every CTA finishes the routing itself from K1's partials (softmax, top-k:
//              bit-exact and identical in every CTA, so no grid-wide exchange) while its producer
//              already streams shared-expert items; the routing groups the step by expert
//              ("slots": 0..S-1 the shared experts, S+u the u-th distinct routed expert in
//              ascending id), each slot owning contiguous rows of the h and y scratch.
//              Phase A, units (slot, 64 gate|up pairs) -> h[slot row][pair] = silu(g) * u, each
//              unit counted on its slot's counter. Phase B, units (slot, 128 output rows) ->
//              y[slot row][j]; a slot's h rows become the B operand once its counter is full.
//              Each down unit is counted on its column block's counter; the arrival that
//              completes a block has its CTA sum the block's B x 128 outputs over each token's
//              slots in a fixed order: out[t][j]. No grid-wide barrier.
//
// Inside the experts kernel (9 warps): warp 8 copies each item (a row block's weights over one K
// range, layout.h) with one cp.async.bulk into a ring of shared-memory stages; warps 0 and 1
// issue the tcgen05.mma of alternate accumulator groups (M = 128 weight rows, N = 32: three int8
// digit planes x 8 tokens, or N = 16: two bf16 terms x 8 tokens; accumulators in TMEM); warps 4-7
// read the accumulators back (tcgen05.ld: one TMEM lane per weight row), apply the int8 group
// scales and finish the units; warps 2-3 convert each slot's h rows into the phase-B operand.
// Work is split over the CTAs by a static partition of the units weighted by their bytes.
//
// Exact activations: an fp32 value v is given to the int8 MMA as three int8 digits with a
// power-of-two scale per (token, 128-group), v = sigma (d0 + d1/128 + d2/128^2), |d| <= 64, the
// int32 sums recombined in fp32 per group before the weight scale (error < 2^-21 of the group's
// largest value); to the bf16 MMA as two bf16 terms v = t0 + t1 (t0 = bf16(v), t1 = bf16(v - t0)).
// Every output element is its own dot product, so every output row is bitwise independent of
// the batch it rides in.
//
// Every device-side wait is bounded (sm100.cuh, kWaitBudgetNs): on expiry the waiter records a
// status code, the kernel winds down, and the call writes NaN over its output (DecodeCtl in
// kernels.h); the sticky status word tells the host (uocr_moe_device_status), and until it is
// read every later call on the workspace writes NaN too.
#include <algorithm>

#include <cuda_bf16.h>

#include "common.cuh"
#include "kernels.h"
#include "layout.h"
#include "digits.cuh"
#include "sm100.cuh"

namespace uocr {

constexpr int kThreads = 9 * 32;             // MMA warps 0-1, stagers 2-3, epilogue 4-7, producer 8
constexpr int kCW = 8;                       // warps 0-7 (the routing)
constexpr int kMaxB = 8;
constexpr int kMaxSlotsSm = 72;              // shared (<= 8) + routed (<= 64)
constexpr uint32_t kBarConsumers = 1;        // named barrier of warps 0-7
constexpr int kAccSlots = 4;                 // TMEM accumulators of 64 columns
constexpr int kMaxJobs = 64;                 // group-image jobs of one CTA (<= its gate/up units)
constexpr uint32_t kAccCols = 64;
constexpr uint32_t kTmemCols = kAccSlots * kAccCols;
constexpr int kDigitAtomBytes = 24 * 128;    // int8 B operand group: 3 digit planes x 8 tokens (24 rows)
constexpr int kDigitPadBytes = 8 * 128;      // an N = 32 MMA reads 8 rows past a group (ignored columns)
constexpr int kTermAtomBytes = 16 * 128;     // bf16 B operand atom: 2 terms x 8 tokens
constexpr uint32_t kIdescS8 = umma_idesc_s8(128, 32);
constexpr uint32_t kIdescBf16 = umma_idesc_bf16(128, 16);

// Slots of this step in shared memory: rows [0, S) the shared experts, [S, S+U) routed.
struct SlotTable {
    int nslot;
    int pad[3];
    int expert[kMaxSlotsSm];
    int count[kMaxSlotsSm];
    int base[kMaxSlotsSm];
    signed char pos[kMaxSlotsSm][kMaxB];  // pos[slot][t]: entry of token t in the slot, -1 if none
};

struct ItemMeta {
    int slot;   // < 0: end of the work
    int rb;     // row block (gate/up: 64 pairs; down: 128 output rows)
    int ki;     // item (K range) within the row block
    int phase;  // 0: gate/up, 1: down
    int run;    // down: the slot run this item starts (its operand image), -1 for none
    int grp;    // accumulator group: an int8 item, or a bf16 unit's even or odd items (MMA warp grp % 2 issues it)
    int pad[2];
};

// One TMEM accumulator's description, written by the MMA warp, read by the epilogue. An
// accumulator is 64 TMEM columns: int8 = up to two 128-groups (columns 0-31, 32-63; column 3t + p
// = digit plane p of token t, 8 unused each), bf16 = two terms x 8 tokens (column 2t + q, 0-15).
struct AccMeta {
    int slot;   // < 0: end of the work
    int rb;
    int gi;     // int8: the 128-group of columns 0-31 (columns 32-63: gi + 1)
    int flags;  // bit 0: int8, bit 1: the unit's last accumulator, bit 2: int8 with two groups, bit 3: down
    float sig[2][kMaxB];       // down, int8: digit scales of the slot's entries for each group
    float scl[2][kRowBlock];   // int8: weight scales of the 128 rows for each group
};

// The shared-expert slots (known from the shape alone).
UOCR_DEV void load_shared_slots(SlotTable* tb, const DecodeArgs& a, int tid, int nthreads) {
    for (int s = tid; s < a.S; s += nthreads) {
        tb->expert[s] = s;
        tb->count[s] = a.B;
        tb->base[s] = s * a.B;
        for (int t = 0; t < kMaxB; ++t) {
            tb->pos[s][t] = t < a.B ? (signed char)t : (signed char)-1;
        }
    }
    if (tid == 0) tb->nslot = a.S;
}

// Diagnostics timeline: per CTA `items` records of 8 words (global-timer ns); item n of the gate/up
// (half 0) or down (half 1) phase: {MMA warp wait start, data ready, MMAs issued and committed,
// slot<<32|rb<<16|ki, producer issue, accumulator acquired (int8), MMAs issued, 0}.
UOCR_DEV unsigned long long* trace_rec(const DecodeArgs& a, int half, int n) {
    if (!a.trace || n >= a.trace_items / 2) return nullptr;
    return a.trace + ((size_t)blockIdx.x * a.trace_items + (size_t)half * (a.trace_items / 2) + n) * 8;
}

// ---- B operands ----------------------------------------------------------------------------
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
// int8 operand image [group][24 rows][128 B] (swizzled, groups `stride` bytes apart: 3 KB in shared
// memory): digit plane p of column t is row 3t + p, so a column's rows are contiguous and the
// first c columns are the group's first 3c rows. The N = 32 MMA of a group also reads the next 8
// rows (the next group's, or padding after the last): their accumulator columns 24-31 are never
// read. Lane L's words of group g, column t.
UOCR_DEV void put_digits(unsigned char* img, size_t stride, int g, int t, int lane, const uint32_t (&w)[3]) {
#pragma unroll
    for (int p = 0; p < 3; ++p)
        *reinterpret_cast<uint32_t*>(img + (size_t)g * stride + atom_offset(3 * t + p, 4 * lane)) = w[p];
}
// bf16 operand image [64-element atom][16 rows][128 B] (swizzled, atoms `stride` bytes apart: 2 KB in
// shared memory): term q of column t is row 2t + q. Lane L's values [4L, 4L + 4) of 128-element
// chunk g of column t (atom 2g + L / 16).
UOCR_DEV void put_terms(unsigned char* img, size_t stride, int g, int t, int lane, float4 v) {
    const __nv_bfloat162 a0 = __floats2bfloat162_rn(v.x, v.y), a1 = __floats2bfloat162_rn(v.z, v.w);
    const __nv_bfloat162 b0 = __floats2bfloat162_rn(v.x - __low2float(a0), v.y - __high2float(a0));
    const __nv_bfloat162 b1 = __floats2bfloat162_rn(v.z - __low2float(a1), v.w - __high2float(a1));
    unsigned char* atom = img + (size_t)(2 * g + (lane >> 4)) * stride;
    const int c = 8 * (lane & 15);
    *reinterpret_cast<uint2*>(atom + atom_offset(2 * t, c)) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&a0), *reinterpret_cast<const uint32_t*>(&a1));
    *reinterpret_cast<uint2*>(atom + atom_offset(2 * t + 1, c)) =
        make_uint2(*reinterpret_cast<const uint32_t*>(&b0), *reinterpret_cast<const uint32_t*>(&b1));
}

// Static partition of the work units over the CTAs, in levels. The units of a phase, in global
// order (the shared experts' units, then the routed slots' in ascending slot, each slot's row
// blocks in order), are dealt like list scheduling by cost: a shared unit costs r quanta, a routed
// unit one (r = 2 for int8 routed experts beside the bf16 shared ones, else 1). Shared unit i goes
// to CTA i % G; CTAs [m, G) (m = shared units % G) carry one shared unit less, so the first
// r (G - m) routed units go to them, one per CTA per level, and every later level deals G routed
// units to all CTAs. A CTA works through its units level by level, so every slot's gate/up units
// are finished by the level that holds them, early slots first: a CTA's first down units belong to
// slots that were complete long before its own gate/up units run out (no wait at the phase
// change), and the costs per CTA differ by at most one quantum.
struct Units {
    int ca, cb;  // this CTA's shared units in each phase (indices c, c + G, ...)
    int ma, mb;  // m of each phase
    int ra, rb;  // r of each phase
    int na, nb;  // this CTA's units in each phase (shared first, then routed by level)
};
// The routed index of this CTA's k-th routed unit (increasing in k).
UOCR_DEV int routed_index(int k, int m, int r) {
    const int G = gridDim.x, c = blockIdx.x;
    if (c >= m) return k < r ? k * (G - m) + (c - m) : r * (G - m) + (k - r) * G + c;
    return r * (G - m) + k * G + c;
}
// How many of n routed units this CTA takes.
UOCR_DEV int routed_count(int n, int m, int r) {
    int k = 0;
    while (routed_index(k, m, r) < n) ++k;
    return k;
}
// A phase's shared-unit split and cost ratio (n_s shared units of `shared_bytes`, routed units of
// `routed_bytes`).
UOCR_DEV void shared_split(int n_s, size_t shared_bytes, size_t routed_bytes, int& cnt, int& m, int& r) {
    const int G = gridDim.x, c = blockIdx.x;
    cnt = c < n_s ? (n_s - 1 - c) / G + 1 : 0;
    m = n_s % G;
    r = max(1, (int)((2 * shared_bytes + routed_bytes) / (2 * routed_bytes)));
}
UOCR_DEV void unit_a(const Units& u, const DecodeArgs& a, int i, int& slot, int& rb) {
    const int per = a.I / 64;
    if (i < u.ca) {
        const int j = blockIdx.x + i * gridDim.x;
        slot = j / per;
        rb = j % per;
    } else {
        const int j = routed_index(i - u.ca, u.ma, u.ra);
        slot = a.S + j / per;
        rb = j % per;
    }
}
UOCR_DEV void unit_b(const Units& u, const DecodeArgs& a, int i, int& slot, int& rb) {
    const int nrb = a.H / kRowBlock;
    if (i < u.cb) {
        const int j = blockIdx.x + i * gridDim.x;
        slot = j / nrb;
        rb = j % nrb;
    } else {
        const int j = routed_index(i - u.cb, u.mb, u.rb);
        slot = a.S + j / nrb;
        rb = j % nrb;
    }
}

// ======================================================================================
// routing inside a CTA (warps 0-7 of the experts kernel)
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

// Per token, its routed y rows in ascending expert id and their weights (the combine's order).
struct CombineSmem {
    int trow[kMaxB][kDecodeMaxTopk];
    float tw[kMaxB][kDecodeMaxTopk];
    int req[2];  // a column block this CTA's epilogue completed: (down unit end << 8) | (block + 1)
};

// The rest of MoEGate (decoder.py:500-514) for the B tokens, from K1's partials: logit = the 8
// segment partials added in ascending order, + bias; softmax with this build's exponential and
// a fixed butterfly sum; top-k by (p desc, index asc) — identical in every CTA. Then the slot
// table: routed slot u is the u-th used expert; its rows start after the shared experts' S * B
// rows, its entries in token order; each token's rows for the combine; and this CTA's routed
// units (`units`, from a table of every possible routed-slot count built before the dependency
// wait). CTA 0 also writes ids / wts. The partials are read straight from L2 into registers;
// K1's operand images arrive by bulk copies on `imb` (the MMA warps wait for them), the digit
// scales are copied into `xsig` by plain loads. Returns false (nothing routed) if the workspace
// holds an unread failure (`stale`).
UOCR_DEV bool cta_route(const DecodeArgs& a, unsigned char* xd, unsigned char* xb, float* xsig, uint64_t* imb,
                        RouteSmem* rs, SlotTable* tb, CombineSmem* cs, Units* units, int* stale, int tid,
                        unsigned long long* ev) {
    const int warp = tid >> 5, lane = tid & 31;
    const int H = a.H, B = a.B, E = a.E, k = a.topk, kB = k * B, nrb = H / kRowBlock;
    unsigned long long* rv = a.trace ? trace_rec(a, 0, a.trace_items / 2 - 2) : nullptr;  // diagnostics
    // before the wait: this call's inputs that no kernel of the step writes, and scratch resets
    if (tid < 64) {
        rs->bias[tid] = a.bias && tid < E ? a.bias[tid] : 0.0f;
        rs->mask[tid] = 0ull;
    }
    for (int i = tid; i < 64 * kMaxB; i += kCW * 32) tb->pos[a.S + i / kMaxB][i % kMaxB] = -1;
    pdl_wait_prior_grid();  // K1's partials and operands
    if (ev && tid == 0) ev[1] = global_timer_ns();
    // the partials of (token, expert) pairs tid and tid + 256, loads issued at once
    float4 p[2][2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int i = tid + kCW * 32 * h;
        if (i < B * 64) {
            p[h][0] = __ldcg(reinterpret_cast<const float4*>(a.logits + 8 * (size_t)i));
            p[h][1] = __ldcg(reinterpret_cast<const float4*>(a.logits + 8 * (size_t)i + 4));
        }
    }
    // an unread failure of an earlier call leaves the counters unknown: this call only writes NaN
    // until the host reads the status (which resets the control block)
    if (tid == 0) *stale = __ldcg(&a.ctl->status) != 0u;
    named_bar_sync(kBarConsumers, kCW * 32);
    if (*stale) return false;
    if (warp == 0) {
        const uint32_t img = (uint32_t)H * 32;
        const uint32_t dbytes = a.int8 ? (uint32_t)((H / 128) * kDigitAtomBytes + kDigitPadBytes) : 0u;
        if (lane == 0) mbar_arrive_expect_tx(imb, dbytes + img);
        __syncwarp();
        if (lane == 1) bulk_g2s(xb, a.xb, img, imb);
        if (lane == 2 && dbytes) bulk_g2s(xd, a.xd, dbytes, imb);
    }
    if (a.int8 && tid < kMaxB * (H / 128)) xsig[tid] = __ldcg(a.xsig + tid);
    if (rv && tid == 0) rv[0] = global_timer_ns();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int i = tid + kCW * 32 * h;
        if (i < B * 64) {
            float total = __fadd_rn(__fadd_rn(__fadd_rn(p[h][0].x, p[h][0].y), p[h][0].z), p[h][0].w);
            total = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(total, p[h][1].x), p[h][1].y), p[h][1].z), p[h][1].w);
            if (a.bias) total = __fadd_rn(total, rs->bias[i & 63]);
            rs->logits[i >> 6][i & 63] = total;
        }
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    if (rv && tid == 0) rv[3] = global_timer_ns();
    // softmax + top-k: warp b serves token b; each pick sets bit (token * k + r) of its expert's mask
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
                atomicOr(&rs->mask[bi], 1ull << (b * k + rr));
                if (blockIdx.x == 0) {
                    a.ids[b * k + rr] = bi;
                    a.wts[b * k + rr] = bp;
                }
            }
        }
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    if (rv && tid == 0) rv[4] = global_timer_ns();
    // group by expert: the used experts in ascending id and their entry counts' prefix
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
    const int nu = __popcll(used);
    if (tid < 64 && c > 0) {
        const int u = __popcll(used & ((1ull << tid) - 1ull));
        const int row = a.S + u;
        const int base = a.S * B + (incl - c) + (warp == 1 ? rs->wsum[0] : 0);
        tb->expert[row] = tid;
        tb->count[row] = c;
        tb->base[row] = base;
        int n = 0;
        for (unsigned long long mm = m; mm; mm &= mm - 1ull, ++n) {
            const int q = __ffsll((long long)mm) - 1, t = q / k;
            tb->pos[row][t] = (signed char)n;
            rs->rowof[q] = base + n;
        }
    }
    if (tid == 0) {
        tb->nslot = a.S + nu;
        units->na = units->ca + routed_count(nu * (a.I / 64), units->ma, units->ra);
    }
    if (tid == 32) units->nb = units->cb + routed_count(nu * nrb, units->mb, units->rb);
    named_bar_sync(kBarConsumers, kCW * 32);
    if (rv && tid == 0) rv[5] = global_timer_ns();
    if (tid < kB) {
        // entry tid of token t: its rank among the token's entries by expert id (distinct ids)
        const int t = tid / k, id = rs->ids[tid];
        int rank = 0;
        for (int j = 0; j < k; ++j) rank += rs->ids[t * k + j] < id;
        cs->trow[t][rank] = rs->rowof[tid];
        cs->tw[t][rank] = rs->wts[tid];
    }
    named_bar_sync(kBarConsumers, kCW * 32);
    if (rv && tid == 0) rv[6] = global_timer_ns();
    return true;
}

// ======================================================================================
// K1: router logit partials and the tokens as B operands
// ======================================================================================
// One warp per CTA. CTAs [0, 8E): expert e = c / 8, segment s = c % 8; lane t < B runs the
// oracle's chain for token t over segment s (fma in ascending k from +0) and writes the
// partial sum part[t][e][s]; the experts kernel adds the 8 partials in ascending order plus the bias. The
// router segment is fetched before the dependency wait. CTAs [8E, 8E + 8 H/128): column
// t = d / (H/128), group g = d % (H/128): x[t][128g, 128g + 128) as int8 digits (+ the group's
// scale) and as two bf16 terms, in the experts kernel's operand images (zeros for t >= B). Small CTAs (no
// shared memory) so several start beside the previous layer's experts kernel on every SM.
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
        pdl_launch_dependents();  // the experts kernel launches now; it waits for this grid before it reads the partials
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
        put_terms(a.xb, kTermAtomBytes, g, t, lane, v);
        if (a.int8) {
            uint32_t w[3];
            const float sg = group_digits(v, w);
            if (lane == 0) a.xsig[t * NG + g] = sg;
            put_digits(a.xd, kDigitAtomBytes, g, t, lane, w);
        }
    }
    if (ev && lane == 0) ev[2] = global_timer_ns();
}

// ======================================================================================
// the MMA warp and the epilogue warps (experts kernel)
// ======================================================================================
// Shared state of the tensor-core pipeline of one CTA.
struct Pipe {
    uint64_t* tfull;   // [kAccSlots]: description written (1 arrival) + MMAs complete (commit)
    uint64_t* tfree;   // [kAccSlots]: the 4 epilogue warps have read the accumulator
    AccMeta* acc;      // [kAccSlots]
    uint32_t tmem;     // TMEM base (kTmemCols columns)
    volatile int* abort_flag;
    uint32_t* status;
};

// MMA warp: take the next accumulator slot (waiting until the epilogue has read it) and write
// its description; returns its index, or -1 on a timeout. publish_acc makes the description
// visible (the first of tfull's two arrivals; the MMAs' commit is the second).
UOCR_DEV int acquire_acc(Pipe& p, int grp, int slot, int rb, int gi, int flags, int lane) {
    const int j = grp % kAccSlots;
    if (grp >= kAccSlots && !mbar_wait_warp(&p.tfree[j], ((grp / kAccSlots) - 1) & 1, p.abort_flag, p.status))
        return -1;
    AccMeta& m = p.acc[j];
    if (lane == 0) {
        m.slot = slot;
        m.rb = rb;
        m.gi = gi;
        m.flags = flags;
    }
    tc_fence_after();  // the epilogue's TMEM reads precede this warp's next MMAs
    return j;
}
// int8 scales of one group into the description: 128 row scales (one float4 per lane) and,
// for down items, the 8 column scales.
UOCR_DEV void acc_scales(Pipe& p, int j, int g, const float* scl, const float* sig, int lane) {
    reinterpret_cast<float4*>(p.acc[j].scl[g])[lane] = reinterpret_cast<const float4*>(scl)[lane];
    if (sig && lane < kMaxB) p.acc[j].sig[g][lane] = sig[lane];
}
UOCR_DEV void publish_acc(Pipe& p, int j, int lane) {
    __syncwarp();
    if (lane == 0) mbar_arrive(&p.tfull[j]);  // release: the description above
}

// Epilogue warp (TMEM lane quarter q = warp % 4, row = 32 q + lane): waits for accumulator c,
// reads it and its description; returns false at the end of the work or on a timeout.
struct AccRead {
    int slot, rb, gi, flags;
    float scl[2], sig[2][kMaxB];
    uint32_t v[2][32];
};
UOCR_DEV bool read_acc(Pipe& p, int c, int q, int lane, bool want_sig, AccRead& r) {
    const int j = c % kAccSlots;
    if (!mbar_wait_warp(&p.tfull[j], (c / kAccSlots) & 1, p.abort_flag, p.status)) return false;
    const AccMeta& m = p.acc[j];
    r.slot = m.slot;
    if (r.slot < 0) return false;
    r.rb = m.rb;
    r.gi = m.gi;
    r.flags = m.flags;
    const int ng = (r.flags & 4) ? 2 : 1;
    tc_fence_after();
    const uint32_t taddr = p.tmem + ((uint32_t)(32 * q) << 16) + kAccCols * j;
    tmem_ld_32x32b_x32(taddr, r.v[0]);
    if (ng == 2) tmem_ld_32x32b_x32(taddr + 32, r.v[1]);
    if (r.flags & 1) {
        for (int g = 0; g < ng; ++g) {
            r.scl[g] = m.scl[g][32 * q + lane];
            if (want_sig) {
#pragma unroll
                for (int t = 0; t < kMaxB; ++t) r.sig[g][t] = m.sig[g][t];
            }
        }
    }
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&p.tfree[j]);
    return true;
}

// int8 group g of an accumulator -> acc[t] += undigit(planes) * (row scale * column scale)
UOCR_DEV void fold_s8(const AccRead& r, int g, const float* colsig, float (&acc)[kMaxB]) {
#pragma unroll
    for (int t = 0; t < kMaxB; ++t)
        acc[t] = __fmaf_rn(undigit((int)r.v[g][3 * t], (int)r.v[g][3 * t + 1], (int)r.v[g][3 * t + 2]),
                           __fmul_rn(r.scl[g], colsig[t]), acc[t]);
}
// bf16 accumulator (a row block's even or odd items): acc[t] += term-0 column + term-1 column
UOCR_DEV void fold_bf16(const AccRead& r, float (&acc)[kMaxB]) {
#pragma unroll
    for (int t = 0; t < kMaxB; ++t)
        acc[t] = __fadd_rn(acc[t], __fadd_rn(__uint_as_float(r.v[0][2 * t]), __uint_as_float(r.v[0][2 * t + 1])));
}

// The down operand of 128-group g of a slot (its h columns [128 g, 128 g + 128) for the slot's cnt
// entries), by one warp, into the slot's image region
// (DecodeArgs::himg): int8 digits (3 rows per entry) with their scales (gsig), or bf16 terms (2 rows
// per entry in each of the group's two 64-element atoms). Four entries' loads are issued before
// their conversions.
UOCR_DEV void write_group_image(const DecodeArgs& a, bool i8, int cnt, int base, int g, int SG, int lane) {
    unsigned char* img = a.himg + (size_t)base * a.I * 4;
    for (int e0 = 0; e0 < cnt; e0 += 4) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = e0 + u;
            if (e < cnt) v[u] = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)(base + e) * a.I + 128 * g + 4 * lane));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = e0 + u;
            if (e < cnt) {
                if (i8) {
                    uint32_t w[3];
                    const float sg = group_digits(v[u], w);
                    if (lane == 0) a.gsig[(size_t)(base + e) * SG + g] = sg;
                    put_digits(img, (size_t)cnt * 384, g, e, lane, w);
                } else {
                    put_terms(img, (size_t)cnt * 256, g, e, lane, v[u]);
                }
            }
        }
    }
}

// ======================================================================================
// the experts kernel: route, gate/up (phase A), down (phase B), combine
// ======================================================================================
// out[t][128 rb + c] for the B tokens and the block's 128 columns by the 128 epilogue threads
// (thread i: token i / 16, the 8 columns from 8 (i % 16)): the token's shared rows in order, then
// its routed rows in ascending expert id (w * y), rows loaded 8 at a time; NaN when the call failed.
UOCR_DEV void combine_block(const DecodeArgs& a, const CombineSmem* cs, int rb, bool failed, int i) {
    const int t = i >> 4, c = kRowBlock * rb + 8 * (i & 15);
    if (t >= a.B) return;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = failed ? __uint_as_float(0x7FC00000u) : 0.0f;
    const int nrows = a.S + a.topk;  // row r < S: shared row r; else routed row r - S
    for (int r0 = 0; r0 < nrows && !failed; r0 += 8) {
        float4 v[8][2];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int r = r0 + u;
            if (r < nrows) {
                const int row = r < a.S ? r * a.B + t : cs->trow[t][r - a.S];
                const float* src = a.y + (size_t)row * a.H + c;
                v[u][0] = __ldcg(reinterpret_cast<const float4*>(src));
                v[u][1] = __ldcg(reinterpret_cast<const float4*>(src + 4));
            }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int r = r0 + u;
            if (r < nrows) {
                const float e[8] = {v[u][0].x, v[u][0].y, v[u][0].z, v[u][0].w,
                                    v[u][1].x, v[u][1].y, v[u][1].z, v[u][1].w};
                if (r < a.S) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], e[j]);
                } else {
                    const float w = cs->tw[t][r - a.S];
#pragma unroll
                    for (int j = 0; j < 8; ++j) acc[j] = __fmaf_rn(w, e[j], acc[j]);
                }
            }
        }
    }
    float* o = a.out + (size_t)t * a.H + c;
    *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
    *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
}
// The same block written NaN by one warp alone (a failure path: no loads).
UOCR_DEV void nan_block(const DecodeArgs& a, int rb, int lane) {
    const float nan = __uint_as_float(0x7FC00000u);
    for (int t = 0; t < a.B; ++t)
        *reinterpret_cast<float4*>(a.out + (size_t)t * a.H + kRowBlock * rb + 4 * lane) = make_float4(nan, nan, nan, nan);
}
// `n` more shares of combined column blocks (4 shares a block: one per epilogue warp), counted by
// lane 0 of the calling warp (every lane calls); the share that completes the call has the warp
// reset the call's words for the next call.
// No fence before the count: the call's reads of the words the last count resets (call_fail by
// acquire loads, the slot counters long before) are ordered before it, and the output stores
// need no order with it (the kernel's completion publishes them).
// Only the words of the call's nslot slots are reset: the slot counters the call used (hdone, or
// imgdone and the I/128 group counters per slot).
UOCR_DEV void count_combined(const DecodeArgs& a, uint32_t n, int lane, int nslot, bool img_call) {
    int last = 0;
    if (lane == 0) last = atomicAdd(&a.ctl->cdone, n) + n == 4u * (uint32_t)(a.H / kRowBlock);
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    const int NG3 = a.I / 128;
    if (img_call) {
        for (int i = lane; i < nslot; i += 32) a.ctl->imgdone[i] = 0u;
        for (int i = lane; i < nslot * NG3; i += 32) a.ctl->gcnt[(i / NG3) * kDecodeMaxGroups + i % NG3] = 0u;
    } else {
        for (int i = lane; i < nslot; i += 32) a.ctl->hdone[i] = 0u;
    }
    __syncwarp();
    if (lane == 0) {
        a.ctl->call_fail = 0u;
        __threadfence();
        atomicExch(&a.ctl->cdone, 0u);
    }
}

// Persistent, one CTA per SM (every CTA resident: they wait on each other's units), 9 warps:
// warp 8 streams items (one bulk copy each) into a ring of fixed stages, first the gate/up units
// (phase A: shared ones while the CTA routes, then routed), then the down units (phase B); warps
// 0 and 1 issue their tcgen05 MMAs, alternate accumulator groups each (B operand: the tokens'
// images from K1 in phase A, the slot run's h image in phase B); warps 4-7 drain the
// accumulators: phase A -> h rows (SwiGLU) and a count per slot; phase B -> y rows and a count per
// output column block, whose completing arrival has its CTA combine the block. Warps 2-3 (phase B)
// turn each slot run's h rows, once every CTA's gate/up units of that slot are counted, into the
// run's operand image. Warps 0-7 route first.
__global__ void __launch_bounds__(kThreads, 1)
decode_experts_kernel(DecodeArgs a, int nst, uint32_t stage_bytes, uint32_t off_tbl, uint32_t off_route,
                      uint32_t off_meta, uint32_t off_acc, uint32_t off_cs, uint32_t off_sig, uint32_t off_hsig,
                      uint32_t off_img, uint32_t off_stages) {
    extern __shared__ __align__(1024) unsigned char smem[];
    __shared__ int abort_flag, stale, routed;
    // 128-groups whose gate/up arrivals this CTA's epilogue completed, handed to the stagers in
    // order (a slot << 8 | group | 1 << 31 word each; 0 = not yet posted), and the epilogue warps
    // done with their gate/up units
    __shared__ uint32_t jobs[kMaxJobs];
    __shared__ int njobs, a_warps_done;
    __shared__ uint32_t tmem_base, cta_fail;  // cta_fail: this CTA's failure code (published at exit)
    __shared__ Units units;
    uint32_t* fail = &cta_fail;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + nst;          // the MMAs reading the stage are complete
    uint64_t* table_ready = empty + nst;
    uint64_t* tfull = table_ready + 1;     // [kAccSlots]
    uint64_t* tfree = tfull + kAccSlots;   // [kAccSlots]
    uint64_t* mdone = tfree + kAccSlots;   // the MMA warp's drain
    uint64_t* adone = mdone + 1;           // every gate/up MMA is complete (the image region is free)
    uint64_t* hready = adone + 1;          // [2]: a run's image is staged (3 stager warps)
    uint64_t* bfree = hready + 2;          // [2]: the MMAs reading a run's image are complete
    uint64_t* ubar = bfree + 2;            // the 4 epilogue warps at a down unit's end
    uint64_t* imb = ubar + 1;              // the tokens' operand images have arrived
    SlotTable* tb = reinterpret_cast<SlotTable*>(smem + off_tbl);
    RouteSmem* rs = reinterpret_cast<RouteSmem*>(smem + off_route);
    ItemMeta* meta = reinterpret_cast<ItemMeta*>(smem + off_meta);
    AccMeta* accm = reinterpret_cast<AccMeta*>(smem + off_acc);
    CombineSmem* cs = reinterpret_cast<CombineSmem*>(smem + off_cs);
    float* xsig = reinterpret_cast<float*>(smem + off_sig);
    float* hsig = reinterpret_cast<float*>(smem + off_hsig);  // [2][8][sig stride]
    unsigned char* xb = smem + off_img;                       // phase A: bf16 terms image
    unsigned char* xd = smem + off_img + (size_t)a.H * 32;    // phase A: int8 digits image
    unsigned char* hb = smem + off_img;                       // phase B: two run images of I * 32 bytes
    unsigned char* stages = smem + off_stages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NG3 = a.I / 128, nrb = a.H / kRowBlock;
    const uint32_t img_bytes = (uint32_t)a.I * 32;
    const int SG = decode_sig_stride(a.I);  // floats per row of the digit scales
    const uint32_t hd_target = 4u * (uint32_t)(a.I / 64) + (uint32_t)a.hold_extra;  // gate/up arrivals per slot
    const uint32_t ig_target = (uint32_t)NG3 + (uint32_t)a.hold_extra;             // written 128-groups per slot
    // How this call makes the down operands (measured per batch): B = 8, and bf16 layers from B = 4,
    // build each slot's image once during the gate/up phase (image warp) and bulk-copy it; smaller
    // batches have the stagers convert each run's h rows at the phase change.
    const bool img_call = a.B >= 8 || (!a.int8 && a.B >= 4);
    unsigned long long* ev = a.trace ? trace_rec(a, 0, a.trace_items / 2 - 1) : nullptr;
    if (ev && tid == 0) ev[0] = global_timer_ns();
    if (smem_addr(smem) & 1023u) {  // the swizzled operands need 1024-byte alignment (same in every CTA)
        if (tid == 0) set_status(&a.ctl->status, kStatusMisaligned);
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 2);  // the issuing MMA warp's commit + the other MMA warp's arrival
        }
        mbar_init(table_ready, 1);
        for (int j = 0; j < kAccSlots; ++j) {
            mbar_init(&tfull[j], 2);
            mbar_init(&tfree[j], 4);
        }
        mbar_init(mdone, 2);  // both MMA warps' commits
        mbar_init(adone, 2);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&hready[b], img_call ? 1 : 2);  // warp 2 with a copied run's bytes, or both stagers
            mbar_init(&bfree[b], 2);   // both MMA warps' commits
        }
        mbar_init(ubar, 4);
        mbar_init(imb, 1);
        abort_flag = 0;
        njobs = 0;
        a_warps_done = 0;
        stale = 0;
        routed = 0;
        cta_fail = 0;
        cs->req[0] = cs->req[1] = -1;
        // the shared-expert units (known from the shape)
        const size_t a_rt = (size_t)w13_items(a.H, a.int8 != 0) * w13_item_bytes(a.int8 != 0);
        shared_split(a.S * (a.I / 64), (size_t)w13_items(a.H, false) * w13_item_bytes(false), a_rt, units.ca,
                     units.ma, units.ra);
        shared_split(a.S * nrb, w2_rb_bytes(a.I, false), w2_rb_bytes(a.I, a.int8 != 0), units.cb, units.mb, units.rb);
        units.na = units.ca;
        units.nb = 0;
        fence_mbar_init();
        pdl_launch_dependents();  // the next layer's first kernel launches early; it waits for this grid
    }
    if (warp == 0) tmem_alloc(&tmem_base, kTmemCols);
    load_shared_slots(tb, a, tid, blockDim.x);
    for (int i = tid; i < kMaxJobs; i += blockDim.x) jobs[i] = 0u;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    Pipe pipe{tfull, tfree, accm, tmem_base, &abort_flag, fail};

    if (warp == 8) {
        // ---------------- producer: one bulk copy per item into the stage ring ----------------
        int n = 0, st = 0;
        uint32_t round = 0;
        bool ok = true, waited = false;
        const uint64_t stream_policy = l2_evict_first_policy();  // weights are read once per step
        auto wait_table = [&]() {
            if (!waited) {
                ok = mbar_wait_warp(table_ready, 0, &abort_flag, fail) && routed;
                waited = true;
            }
        };
        int grp = 0;  // accumulator groups handed out
        // an int8 item is a group of its own; a bf16 unit's items form two groups (even and odd
        // items), issued by the two MMA warps in turn
        auto item_grp = [&](bool i8, int ki, int nk) {
            if (i8) return grp++;
            const int g = grp + (ki & 1);
            if (ki == nk - 1) grp += nk > 1 ? 2 : 1;
            return g;
        };
        auto issue = [&](const unsigned char* src, uint32_t bytes, int slot, int rb, int ki, int phase, int run,
                         int g) {
            if (ok && round > 0 && !mbar_wait_warp(&empty[st], (round - 1) & 1, &abort_flag, fail)) ok = false;
            if (!ok) return;
            if (lane == 0) {
                meta[st].slot = slot;
                meta[st].rb = rb;
                meta[st].ki = ki;
                meta[st].phase = phase;
                meta[st].run = run;
                meta[st].grp = g;
                mbar_arrive_expect_tx(&full[st], bytes);
                bulk_g2s_hint(stages + (size_t)st * stage_bytes, src, bytes, &full[st], stream_policy);
                unsigned long long* tr = trace_rec(a, phase, n);
                if (tr) tr[4] = global_timer_ns();
            }
            __syncwarp();
            ++n;
            if (++st == nst) {
                st = 0;
                ++round;
            }
        };
        auto issue_a = [&](int slot, int rb) {
            const bool i8 = slot >= a.S && a.int8;
            const uint32_t bytes = (uint32_t)w13_item_bytes(i8);
            const unsigned char* base =
                slot < a.S ? reinterpret_cast<const unsigned char*>(a.w13_shared) +
                                 (size_t)tb->expert[slot] * w13_expert_bytes(a.I, a.H, false)
                           : reinterpret_cast<const unsigned char*>(a.w13) +
                                 (size_t)tb->expert[slot] * w13_expert_bytes(a.I, a.H, i8);
            const int nk = w13_items(a.H, i8);
            for (int ki = 0; ki < nk && ok; ++ki)
                issue(base + ((size_t)rb * nk + ki) * bytes, bytes, slot, rb, ki, 0, -1, item_grp(i8, ki, nk));
        };
        const int ns_a = units.ca;
        for (int i = 0; i < ns_a && ok; ++i) {  // shared units: streamed while routing
            int slot, rb;
            unit_a(units, a, i, slot, rb);
            issue_a(slot, rb);
        }
        wait_table();
        int runs = 0, prev = -1;
        if (ok) {
            for (int i = ns_a; i < units.na && ok; ++i) {
                int slot, rb;
                unit_a(units, a, i, slot, rb);
                issue_a(slot, rb);
            }
            for (int i = 0; i < units.nb && ok; ++i) {
                int slot, rb;
                unit_b(units, a, i, slot, rb);
                const bool i8 = slot >= a.S && a.int8;
                const unsigned char* base =
                    slot < a.S ? reinterpret_cast<const unsigned char*>(a.w2_shared) +
                                     (size_t)tb->expert[slot] * w2_expert_bytes(a.H, a.I, false)
                               : reinterpret_cast<const unsigned char*>(a.w2) +
                                     (size_t)tb->expert[slot] * w2_expert_bytes(a.H, a.I, i8);
                base += (size_t)rb * w2_rb_bytes(a.I, i8);
                const int run = slot != prev ? runs++ : -1;
                prev = slot;
                const int nk = w2_items(a.I, i8);
                for (int ki = 0; ki < nk && ok; ++ki)
                    issue(base + w2_item_offset(i8, ki), (uint32_t)item_bytes(w2_item_atoms(a.I, i8, ki), i8), slot,
                          rb, ki, 1, ki == 0 ? run : -1, item_grp(i8, ki, nk));
            }
        }
        if (lane == 0) {
            if (!ok) {
                abort_flag = 1;
                for (int q = max(0, n - nst); q < n; ++q) mbar_wait(&full[q % nst], (q / nst) & 1, nullptr);
            } else if (round == 0 || mbar_wait(&empty[st], (round - 1) & 1, fail)) {
                meta[st].slot = -1;  // end marker, published as accumulator group `grp`
                meta[st].grp = grp;
                mbar_arrive(&full[st]);
            } else {
                abort_flag = 1;
            }
        }
        __syncwarp();
    } else {
        // ---------------- warps 0-7: route; then MMA (0), stagers (1-3), epilogue (4-7) ----------------
        const bool ok_route = cta_route(a, xd, xb, xsig, imb, rs, tb, cs, &units, &stale, tid, ev);
        if (tid == 0) {
            if (ok_route) routed = 1;
            else abort_flag = 1;
            mbar_arrive(table_ready);
        }
        named_bar_sync(kBarConsumers, kCW * 32);
        if (ev && tid == 0) ev[2] = global_timer_ns();
        if (warp <= 1) {
            // ---------------- MMA warps: warp w issues the accumulator groups g with g % 2 == w ----------------
            // Both walk every stage in order (the owner's commit and the other's arrival free it).
            const uint32_t xd_s = smem_addr(xd), xb_s = smem_addr(xb), hb_s = smem_addr(hb);
            const int nk8 = w13_items(a.H, true), nk16 = w13_items(a.H, false);
            bool ok = routed != 0, b_started = false;
            int cur = 0, b = 0;
            if (ok && !mbar_wait_warp(imb, 0, &abort_flag, fail)) ok = false;  // the tokens' operand images
            for (int n = 0; ok; ++n) {
                const int st = n % nst;
                const uint64_t t_wait = a.trace ? global_timer_ns() : 0;
                if (!mbar_wait_warp(&full[st], (n / nst) & 1, &abort_flag, fail)) {
                    ok = false;
                    break;
                }
                const int slot = meta[st].slot, grp = meta[st].grp;
                if (slot < 0) {
                    if ((grp & 1) == warp) {  // the end marker's accumulator group is this warp's
                        const int j = acquire_acc(pipe, grp, -1, 0, 0, 0, lane);
                        if (j >= 0) {
                            publish_acc(pipe, j, lane);
                            if (lane == 0) mbar_arrive(&tfull[j]);
                        } else {
                            ok = false;
                        }
                    }
                    break;
                }
                const int rb = meta[st].rb, ki = meta[st].ki, phase = meta[st].phase, run = meta[st].run;
                if (phase == 1) {
                    if (!b_started) {  // the image region may be restaged once every gate/up MMA is done
                        if (lane == 0) umma_commit(adone);
                        b_started = true;
                    }
                    if (run >= 0) {
                        // a run starts: the previous run's image is free once its MMAs complete
                        if (run > 0 && lane == 0) umma_commit(&bfree[(run - 1) & 1]);
                        b = run & 1;
                        if (!mbar_wait_warp(&hready[b], (run >> 1) & 1, &abort_flag, fail)) {
                            ok = false;
                            break;
                        }
                    }
                }
                if ((grp & 1) != warp) {  // the other MMA warp's item: done with the stage's description
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&empty[st]);
                    continue;
                }
                unsigned long long* tr = a.trace ? trace_rec(a, phase, n) : nullptr;
                if (tr && lane == 0) {
                    tr[0] = t_wait;
                    tr[1] = global_timer_ns();
                }
                const bool i8 = slot >= a.S && a.int8;
                unsigned char* item = stages + (size_t)st * stage_bytes;
                const uint32_t item_s = smem_addr(item);
                if (phase == 0) {
                    if (i8) {
                        // both groups of the item in one accumulator (columns 0-31, 32-63)
                        const float* scl = reinterpret_cast<const float*>(item + 2 * kAtomBytes);
                        const int j = acquire_acc(pipe, grp, slot, rb, 2 * ki, 1 | 4 | (ki == nk8 - 1 ? 2 : 0), lane);
                        if (j < 0) {
                            ok = false;
                            break;
                        }
                        if (tr && lane == 0) tr[5] = global_timer_ns();
                        acc_scales(pipe, j, 0, scl, nullptr, lane);
                        acc_scales(pipe, j, 1, scl + kRowBlock, nullptr, lane);
                        publish_acc(pipe, j, lane);
                        if (lane == 0) {
#pragma unroll
                            for (int g = 0; g < 2; ++g)
#pragma unroll
                                for (int s = 0; s < 4; ++s)
                                    umma_i8(pipe.tmem + kAccCols * j + 32u * g, umma_desc_sw128(item_s + g * kAtomBytes + 32 * s),
                                            umma_desc_sw128(xd_s + (2 * ki + g) * kDigitAtomBytes + 32 * s), kIdescS8, s > 0);
                            umma_commit(&tfull[j]);
                        }
                    } else {
                        if (ki < 2) {  // this warp's group of the unit: its even or odd items
                            cur = acquire_acc(pipe, grp, slot, rb, 0, (ki & 1) || nk16 == 1 ? 2 : 0, lane);
                            if (cur < 0) {
                                ok = false;
                                break;
                            }
                            publish_acc(pipe, cur, lane);
                        }
                        if (lane == 0) {
#pragma unroll
                            for (int at = 0; at < 2; ++at)
#pragma unroll
                                for (int s = 0; s < 4; ++s)
                                    umma_f16(pipe.tmem + kAccCols * cur, umma_desc_sw128(item_s + at * kAtomBytes + 32 * s),
                                             umma_desc_sw128(xb_s + (2 * ki + at) * kTermAtomBytes + 32 * s), kIdescBf16,
                                             ((ki >> 1) | at | s) != 0);
                            if (ki + 2 >= nk16) umma_commit(&tfull[cur]);
                        }
                    }
                } else {
                    const int nk = w2_items(a.I, i8);
                    const uint32_t img_s = hb_s + (uint32_t)b * img_bytes;
                    if (i8) {
                        const int at = w2_item_atoms(a.I, true, ki);
                        const int j = acquire_acc(pipe, grp, slot, rb, 2 * ki,
                                                  8 | 1 | (at == 2 ? 4 : 0) | (ki == nk - 1 ? 2 : 0), lane);
                        if (j < 0) {
                            ok = false;
                            break;
                        }
                        if (tr && lane == 0) tr[5] = global_timer_ns();
                        const float* scl = reinterpret_cast<const float*>(item + at * kAtomBytes);
                        for (int g = 0; g < at; ++g) {
                            float sig[kMaxB];
#pragma unroll
                            for (int t = 0; t < kMaxB; ++t) sig[t] = hsig[(b * kMaxB + t) * SG + 2 * ki + g];
                            acc_scales(pipe, j, g, scl + g * kRowBlock, sig, lane);
                        }
                        publish_acc(pipe, j, lane);
                        if (lane == 0) {
                            for (int g = 0; g < at; ++g)
#pragma unroll
                                for (int s = 0; s < 4; ++s)
                                    umma_i8(pipe.tmem + kAccCols * j + 32u * g, umma_desc_sw128(item_s + g * kAtomBytes + 32 * s),
                                            umma_desc_sw128(img_s + (2 * ki + g) * kDigitAtomBytes + 32 * s), kIdescS8, s > 0);
                            umma_commit(&tfull[j]);
                        }
                    } else {
                        if (ki < 2) {  // this warp's group of the unit: its even or odd items
                            cur = acquire_acc(pipe, grp, slot, rb, 0, (ki & 1) || nk == 1 ? 8 | 2 : 8, lane);
                            if (cur < 0) {
                                ok = false;
                                break;
                            }
                            publish_acc(pipe, cur, lane);
                        }
                        if (lane == 0) {
#pragma unroll
                            for (int at = 0; at < 2; ++at)
#pragma unroll
                                for (int s = 0; s < 4; ++s)
                                    umma_f16(pipe.tmem + kAccCols * cur, umma_desc_sw128(item_s + at * kAtomBytes + 32 * s),
                                             umma_desc_sw128(img_s + (2 * ki + at) * kTermAtomBytes + 32 * s), kIdescBf16,
                                             ((ki >> 1) | at | s) != 0);
                            if (ki + 2 >= nk) umma_commit(&tfull[cur]);
                        }
                    }
                }
                __syncwarp();
                if (tr && lane == 0) tr[6] = global_timer_ns();
                if (lane == 0) umma_commit(&empty[st]);  // the stage is free once these MMAs complete
                if (tr && lane == 0) {
                    tr[2] = global_timer_ns();
                    tr[3] = ((unsigned long long)slot << 32) | ((unsigned)rb << 16) | (unsigned)ki;
                }
                __syncwarp();
            }
            if (!ok && lane == 0) abort_flag = 1;
            if (lane == 0) {
                if (!b_started) umma_commit(adone);
                umma_commit(mdone);  // every MMA complete before TMEM is released
                mbar_wait(mdone, 0, fail);
            }
            __syncwarp();
            if (ev && lane == 0) ev[3] = global_timer_ns();
        } else if (warp <= 3) {
            // ---------------- stagers (warps 2-3) ----------------
            // Gate/up phase, warp 3 (the image warp): takes the 128-groups of many-entry slots this
            // CTA's epilogue completed, in the order it posted them, writes each group's image and
            // counts it, until every epilogue warp is past its gate/up units and no posted group is left.
            bool ok = routed != 0;
            if (warp == 3 && img_call) {
                int next = 0;
                uint64_t t0 = 0;
                for (uint32_t spin = 0; ok; ++spin) {
                    uint32_t job = 0;
                    if (next < kMaxJobs) job = ld_acquire_cta_u32(&jobs[next]);
                    if (job) {
                        const int slot = (int)((job >> 8) & 0xFFu), g = (int)(job & 0xFFu);
                        write_group_image(a, slot >= a.S && a.int8, tb->count[slot], tb->base[slot], g, SG, lane);
                        __syncwarp();
                        if (lane == 0) red_release_gpu_add(&a.ctl->imgdone[slot], 1u);
                        ++next;
                        continue;
                    }
                    if (ld_acquire_cta_u32(&a_warps_done) == 4u) {
                        if (next >= kMaxJobs || ld_acquire_cta_u32(&jobs[next]) == 0u) break;
                        continue;
                    }
                    if ((spin & 31) == 0) {
                        int give_up = 0;
                        if (lane == 0) {
                            const uint64_t now = global_timer_ns();
                            if (t0 == 0) t0 = now;
                            const bool aborted = *reinterpret_cast<volatile int*>(&abort_flag) != 0;
                            give_up = aborted || now - t0 > kWaitBudgetNs;
                            if (give_up && !aborted) set_status(fail, kStatusWaitTimeout);
                        }
                        if (__shfl_sync(0xffffffffu, give_up, 0)) ok = false;
                    }
                    __nanosleep(64);
                }
            }
            // Down runs in the producer's order; run r uses image r % 2. Once the image region is free:
            //   img_call:  warp 2, when every 128-group image of the slot is written, posts the bytes
            //              on hready and bulk-copies the slot's groups (int8: digits, then the
            //              scales) or atoms (bf16);
            //   otherwise: both warps, when every CTA's gate/up units of the slot are counted, turn
            //              its h rows (L2) into int8 digit rows and their scales, or bf16 terms, and
            //              arrive on hready.
            const int rank = warp - 2;
            unsigned long long* sv = a.trace ? trace_rec(a, 1, a.trace_items / 2 - 3) : nullptr;
            int r = 0, prev = -1;
            for (int i = 0; i < units.nb && ok && (!img_call || warp == 2); ++i) {
                int slot, rb;
                unit_b(units, a, i, slot, rb);
                if (slot == prev) continue;
                prev = slot;
                const int b = r & 1;
                unsigned long long* tv = sv && rank == 0 && lane == 0 && r < 2 ? sv + 4 * r : nullptr;
                // the image region: free of gate/up MMAs (runs 0, 1), or of run r - 2's MMAs
                if (r < 2) ok = mbar_wait_warp(adone, 0, &abort_flag, fail);
                else ok = mbar_wait_warp(&bfree[b], ((r - 2) >> 1) & 1, &abort_flag, fail);
                if (tv) tv[0] = global_timer_ns();
                if (!ok) break;
                const int cnt = tb->count[slot], base = tb->base[slot];
                const bool i8 = slot >= a.S && a.int8, bulk = img_call;
                unsigned char* img = hb + (size_t)b * img_bytes;
                {
                    int done = 0;
                    if (lane == 0)
                        done = wait_counter_geq(bulk ? &a.ctl->imgdone[slot] : &a.ctl->hdone[slot], bulk ? ig_target : hd_target,
                                                fail);
                    ok = __shfl_sync(0xffffffffu, done, 0) != 0;
                }
                if (!ok) break;
                if (tv) tv[1] = global_timer_ns();
                if (bulk) {
                    const int nparts = i8 ? NG3 : 2 * NG3;  // 128-groups (int8) or 64-element atoms (bf16)
                    const uint32_t part = (uint32_t)cnt * (i8 ? 384u : 256u);
                    const uint32_t sbytes = i8 ? (uint32_t)(cnt * SG * 4) : 0u;
                    const unsigned char* src = a.himg + (size_t)base * a.I * 4;
                    if (lane == 0) {
                        fence_proxy_async_global();  // the image warps' generic writes, read next by bulk copies
                        fence_proxy_async_smem();    // this region's earlier generic writes and reads
                        mbar_arrive_expect_tx(&hready[b], (uint32_t)nparts * part + sbytes);
                    }
                    __syncwarp();
                    for (int q = lane; q < nparts; q += 32)
                        bulk_g2s(img + (size_t)q * (i8 ? kDigitAtomBytes : kTermAtomBytes), src + (size_t)q * part, part,
                                 &hready[b]);
                    if (lane == 31 && sbytes)
                        bulk_g2s(hsig + b * kMaxB * SG, a.gsig + (size_t)base * SG, sbytes, &hready[b]);
                } else {
                    const int ntask = cnt * NG3;
                    for (int t0 = rank; t0 < ntask; t0 += 4 * 2) {
                        float4 v[4];  // four tasks' loads issued before any of their stores
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int task = t0 + u * 2;
                            if (task < ntask) {
                                const int e = task / NG3, g = task - e * NG3;
                                v[u] = __ldcg(reinterpret_cast<const float4*>(a.h + (size_t)(base + e) * a.I + 128 * g + 4 * lane));
                            }
                        }
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int task = t0 + u * 2;
                            if (task < ntask) {
                                const int e = task / NG3, g = task - e * NG3;
                                if (i8) {
                                    uint32_t w[3];
                                    const float sg = group_digits(v[u], w);
                                    if (lane == 0) hsig[(b * kMaxB + e) * SG + g] = sg;
                                    put_digits(img, kDigitAtomBytes, g, e, lane, w);
                                } else {
                                    put_terms(img, kTermAtomBytes, g, e, lane, v[u]);
                                }
                            }
                        }
                    }
                    fence_proxy_async_smem();  // generic writes of the image, read next by the tensor cores
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&hready[b]);
                }
                if (tv) tv[2] = global_timer_ns();
                ++r;
            }
            if (!ok && lane == 0) abort_flag = 1;
        } else {
            // ---------------- epilogue (warps 4-7) ----------------
            const int q = warp & 3, row = 32 * q + lane, ie = tid - 128;
            float acc[kMaxB];
#pragma unroll
            for (int t = 0; t < kMaxB; ++t) acc[t] = 0.0f;
            int ia = 0, ib = 0;  // units of each phase counted so far (in the partition's order)
            const uint32_t yd_target = 4u * (uint32_t)tb->nslot;
            bool ok = routed != 0, a_signalled = false;
            for (int c = 0; ok; ++c) {
                if (!a_signalled && ia == units.na) {
                    // this warp's gate/up units are done (jobs posted): the stagers may move on
                    a_signalled = true;
                    __syncwarp();
                    if (lane == 0) st_release_cta_add(&a_warps_done, 1);
                }
                AccRead r;
                if (!read_acc(pipe, c, q, lane, true, r)) break;
                if (r.flags & 1) {
                    for (int g = 0; g < ((r.flags & 4) ? 2 : 1); ++g) {
                        if (r.flags & 8) {
                            fold_s8(r, g, r.sig[g], acc);
                        } else {
                            float colsig[kMaxB];
#pragma unroll
                            for (int t = 0; t < kMaxB; ++t) colsig[t] = xsig[t * (a.H / 128) + r.gi + g];
                            fold_s8(r, g, colsig, acc);
                        }
                    }
                } else {
                    fold_bf16(r, acc);
                }
                if (!(r.flags & 2)) continue;
                const int cnt = tb->count[r.slot], base = tb->base[r.slot];
                if (!(r.flags & 8)) {
                    // gate/up unit done: SwiGLU (gate row lane % 16 < 8 with the up row 8 lanes up) -> h
                    const bool gate = (lane & 15) < 8;
                    const int pair = 64 * r.rb + 8 * (row >> 4) + (row & 7);
#pragma unroll
                    for (int t = 0; t < kMaxB; ++t) {
                        const float u = __shfl_xor_sync(0xffffffffu, acc[t], 8);
                        const int pos = tb->pos[r.slot][t];
                        if (gate && pos >= 0) a.h[(size_t)(base + pos) * a.I + pair] = silu(acc[t]) * u;
                        acc[t] = 0.0f;
                    }
                    __syncwarp();
                    if (!img_call) {
                        // counted; the down phase's stagers make this slot's operand
                        if (lane == 0) red_release_gpu_add(&a.ctl->hdone[r.slot], 1u);
                    } else if (lane == 0) {
                        // the arrival that completes the slot's 128-group hands the group to the image warp
                        const int g = r.rb >> 1;
                        if (atom_acq_rel_gpu_add(&a.ctl->gcnt[r.slot * kDecodeMaxGroups + g], 1u) + 1u == 8u) {
                            const int j = atomicAdd(&njobs, 1);
                            if (j < kMaxJobs) st_release_cta_u32(&jobs[j], (1u << 31) | ((uint32_t)r.slot << 8) | (uint32_t)g);
                            else set_status(fail, kStatusBadCount);
                        }
                    }
                    ++ia;
                } else {
                    // down unit done: y rows; the arrival that completes the column block has this
                    // CTA's 4 epilogue warps combine it
#pragma unroll
                    for (int t = 0; t < kMaxB; ++t) {
                        if (t < cnt) a.y[(size_t)(base + t) * a.H + kRowBlock * r.rb + row] = acc[t];
                        acc[t] = 0.0f;
                    }
                    __syncwarp();
                    int setter = 0;  // this warp's arrival completed the column block
                    if (lane == 0) {
                        if (atom_acq_rel_gpu_add(&a.ctl->ydone[r.rb], 1u) + 1u == yd_target) {
                            atomicExch(&a.ctl->ydone[r.rb], 0u);
                            cs->req[ib & 1] = (ib << 8) | (r.rb + 1);
                            setter = 1;
                        }
                        mbar_arrive(ubar);
                    }
                    setter = __shfl_sync(0xffffffffu, setter, 0);
                    ++ib;
                    __syncwarp();
                    const bool met = mbar_wait_warp(ubar, (ib - 1) & 1, &abort_flag, fail);
                    if (!met) {
                        // a warp of this CTA is gone: a block this warp completed is written NaN by it alone
                        if (setter) {
                            if (lane == 0) atomicOr(&a.ctl->call_fail, 1u);
                            __syncwarp();
                            nan_block(a, r.rb, lane);
                            __syncwarp();
                            count_combined(a, 4u, lane, tb->nslot, img_call);
                        }
                        ok = false;
                        break;
                    }
                    const int req = *reinterpret_cast<volatile int*>(&cs->req[(ib - 1) & 1]);
                    const bool mine = req >= 0 && (req >> 8) == ib - 1;
                    if (mine) {
                        const bool failed = ld_acquire_gpu(&a.ctl->call_fail) != 0u;
                        combine_block(a, cs, (req & 255) - 1, failed, ie);
                        __syncwarp();
                        count_combined(a, 1u, lane, tb->nslot, img_call);
                    }
                }
            }
            if (routed) {
                // wind-down after a failure: count this warp's remaining units (the call fails, so
                // every block is written NaN), so that no CTA waits for them
                if (ia < units.na || ib < units.nb) {
                    if (lane == 0) atomicOr(&a.ctl->call_fail, 1u);
                    abort_flag = 1;
                }
                for (; ia < units.na; ++ia) {
                    int slot, rb;
                    unit_a(units, a, ia, slot, rb);
                    if (lane == 0) {
                        __threadfence();
                        // a group this completes is counted written (the call fails: its image is not used)
                        if (!img_call) atomicAdd(&a.ctl->hdone[slot], 1u);
                        else if (atomicAdd(&a.ctl->gcnt[slot * kDecodeMaxGroups + (rb >> 1)], 1u) + 1u == 8u)
                            atomicAdd(&a.ctl->imgdone[slot], 1u);
                    }
                __syncwarp();
                if (!a_signalled && lane == 0) st_release_cta_add(&a_warps_done, 1);
                }
                for (; ib < units.nb; ++ib) {
                    int slot, rb;
                    unit_b(units, a, ib, slot, rb);
                    int last = 0;
                    if (lane == 0) {
                        __threadfence();
                        last = atomicAdd(&a.ctl->ydone[rb], 1u) + 1u == yd_target;
                        if (last) atomicExch(&a.ctl->ydone[rb], 0u);
                    }
                    if (__shfl_sync(0xffffffffu, last, 0)) {
                        nan_block(a, rb, lane);
                        __syncwarp();
                        count_combined(a, 4u, lane, tb->nslot, img_call);
                    }
                }
            }
            if (ev && tid == 128) ev[4] = global_timer_ns();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
    if (tid == 0 && cta_fail) set_status(&a.ctl->status, cta_fail);
    if (stale) {
        // an earlier call's failure is unread: NaN over this CTA's share of the output
        const int total = a.B * a.H;
        const int lo = (int)((long long)total * blockIdx.x / gridDim.x);
        const int hi = (int)((long long)total * (blockIdx.x + 1) / gridDim.x);
        for (int o = lo + tid; o < hi; o += blockDim.x) a.out[o] = __uint_as_float(0x7FC00000u);
    }
}

// ======================================================================================
// host side
// ======================================================================================
static size_t up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Launch with programmatic dependent launch allowed (the grid may start before the previous
// kernel of the stream has finished; it waits for it with griddepcontrol.wait).
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
    // The experts kernel leaves room on its SM for its own static shared memory (< 1 KB) and its
    // reservation, and for the next layer's K1 CTAs (no shared memory, 1 KB reservation each), so
    // those start beside it. The dynamic region is 1024-byte aligned (the swizzled operands).
    const int k1_ctas = a.E * 8 + kMaxB * (a.H / 128);
    const int k1_per_sm = (k1_ctas + sms - 1) / sms;
    max_smem = std::min(max_smem - 1024, sm_smem - 1024 - 1024 - 1024 * k1_per_sm);
    max_smem &= ~1023;
    if (g_decode_trace) {
        a.trace = g_decode_trace;
        a.trace_items = (int)(g_decode_trace_bytes / (sizeof(unsigned long long) * 8 * (size_t)sms)) & ~1;
    }
    a.hold_extra = g_decode_wait_extra;

    // ---- K1: logit partials (one CTA per expert and segment) and the B operand images
    {
        void* args[] = {&a};
        err = launch_pdl(reinterpret_cast<const void*>(decode_logits_kernel), dim3(k1_ctas), dim3(32), 0, st, args);
        if (err != cudaSuccess) return err;
    }
    // ---- the experts kernel: a stage holds one item of either phase; the image region holds
    // K1's operand images, then two run images
    const uint32_t stage_bytes =
        (uint32_t)up(std::max(w13_item_bytes(false), a.int8 ? w13_item_bytes(true) : size_t(0)), 1024);
    const size_t off_tbl = 512;  // the mbarriers before it
    const size_t off_route = off_tbl + up(sizeof(SlotTable), 128);
    const size_t off_meta = off_route + up(sizeof(RouteSmem), 128);
    const size_t off_acc = off_meta + up(sizeof(ItemMeta) * 8, 128);
    const size_t off_cs = off_acc + up(sizeof(AccMeta) * kAccSlots, 128);
    const size_t off_sig = off_cs + up(sizeof(CombineSmem), 128);
    const size_t off_hsig = off_sig + up(sizeof(float) * kMaxB * (a.H / 128), 128);
    const size_t off_img = up(off_hsig + sizeof(float) * 2 * kMaxB * decode_sig_stride(a.I), 1024);
    // phase A: the bf16 terms image, then the int8 digits image; phase B: two run images (bf16 runs
    // need I * 32 bytes, int8 runs I * 24 + 1 KB)
    const size_t img = std::max((size_t)a.H * 32 + (a.int8 ? (size_t)(a.H / 128) * kDigitAtomBytes + kDigitPadBytes : 0),
                                (size_t)2 * a.I * 32);
    const size_t off_stages = up(off_img + img, 1024);
    if ((size_t)max_smem < off_stages + 2 * (size_t)stage_bytes) return cudaErrorInvalidConfiguration;
    int nst = (int)std::min<size_t>(8, ((size_t)max_smem - off_stages) / stage_bytes);
    const size_t smem = off_stages + (size_t)nst * stage_bytes;
    const void* k = reinterpret_cast<const void*>(decode_experts_kernel);
    err = ensure_smem_optin(k, smem);
    if (err != cudaSuccess) return err;
    // the CTAs wait on each other's units, so all of them must be resident at once: one per SM
    // must fit (refused otherwise). The launch is not cooperative: a cooperative grid waits for
    // the router kernel to finish before any CTA starts, where a programmatic dependent launch
    // lets every CTA start on the SM the previous layer's CTA leaves, route-independent shared
    // weights streaming while the router runs. A kernel of another stream that holds SMs can
    // keep CTAs out; the bounded waits then end the call with NaN and a status, never a hang.
    int per_sm = 0;
    err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem);
    if (err != cudaSuccess) return err;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    uint32_t o[9] = {(uint32_t)off_tbl, (uint32_t)off_route, (uint32_t)off_meta, (uint32_t)off_acc, (uint32_t)off_cs,
                     (uint32_t)off_sig, (uint32_t)off_hsig, (uint32_t)off_img, (uint32_t)off_stages};
    uint32_t sb = stage_bytes;
    void* args[] = {&a, &nst, &sb, &o[0], &o[1], &o[2], &o[3], &o[4], &o[5], &o[6], &o[7], &o[8]};
    err = launch_pdl(k, dim3(sms), dim3(kThreads), smem, st, args);
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}

}  // namespace uocr
