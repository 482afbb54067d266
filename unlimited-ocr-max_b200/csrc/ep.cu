// Expert-parallel bookkeeping on the device: the dispatch plan with the bf16 row gather, and
// the combine of the returned partial rows. The reference runs the MoE on one device; these
// serve the B200 build's expert-parallel prefill (ep.py). The row order (destination rank,
// then token) and the sum order of the combine (ascending source rank, from +0, then the
// shared-expert term) are the ones ep.py's plan_dispatch / sum_partials state, bit for bit.
//
// Dispatch, three launches:
//   count:  (chunks of kChunk tokens) per token the bit mask of ranks that own one of its
//           experts; per chunk and rank the number of tokens with that bit (warp ballots).
//   plan:   (chunks) each CTA sums the chunk counts of all chunks (rank totals, hence each
//           rank's first row) and of the chunks before it, ranks its tokens per destination with
//           ballot prefixes and writes inv, meta and the row -> token map. CTA 0 writes the
//           per-rank row counts.
//   copy:   (8 SM-widths of CTAs, a warp per row) rows x fp32 -> bf16 (round to nearest even),
//           16-byte stores.
// HBM bytes: x read once per destination (the re-reads of a token's row hit L2), rows written
// once: about T * H * 4 + rows * H * 2.
//
// The peer path (ExpertParallelMoE's forward) replaces the all-to-alls with stores into the other
// ranks' exchange buffers (mapped with CUDA IPC: plain loads and stores over NVLink, no multicast):
//   plan:   as above, but each (token, destination) row's slot metadata (local expert ids and
//           weights) goes straight to the destination's buffer, slot `rank`, at the row's position
//           among the rows for that destination; inv[p][t] is that position.
//   send:   rows x fp32 -> bf16 stored straight to the destinations; the grid's last CTA then
//           publishes, per destination, the row count and the epoch (release, system scope).
//   wait:   (before the expert products) one lane per source waits (bounded) for that source's
//           epoch, reads its row count, and records the slot's failure (no data in time, or a count
//           above the slot's capacity).
//   (the expert products and the partial rows sent back: prefill.cu, peer mode)
//   combine: every CTA first waits (bounded) for every expert rank's partial flag of this epoch,
//           then sums its tokens' partial rows in ascending rank order from +0, then + `add`; a CTA
//           whose wait failed, or that sees a failure flagged, writes NaN for its tokens.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

#include <cuda_bf16.h>

namespace uocr {

namespace {

constexpr int kChunk = 256;  // tokens per CTA (one per thread)

__global__ void __launch_bounds__(kChunk)
ep_count_kernel(const int32_t* __restrict__ ids, int T, int k, const int32_t* __restrict__ owner, int E, int world,
                uint8_t* __restrict__ mask_out, int32_t* __restrict__ counts) {
    __shared__ int wcount[kChunk / 32][kEpMaxWorld];
    const int t = blockIdx.x * kChunk + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned mask = 0;
    if (t < T) {
        for (int s = 0; s < k; ++s) {
            const int e = ids[(size_t)t * k + s];
            const int o = (e >= 0 && e < E) ? owner[e] : -1;
            if (o >= 0 && o < world) mask |= 1u << o;
        }
        mask_out[t] = (uint8_t)mask;
    }
    for (int p = 0; p < world; ++p) {
        const unsigned b = __ballot_sync(0xffffffffu, (mask >> p) & 1u);
        if (lane == 0) wcount[warp][p] = __popc(b);
    }
    __syncthreads();
    if (threadIdx.x < world) {
        int c = 0;
        for (int w = 0; w < kChunk / 32; ++w) c += wcount[w][threadIdx.x];
        counts[(size_t)blockIdx.x * world + threadIdx.x] = c;
    }
}

__global__ void __launch_bounds__(kChunk)
ep_plan_kernel(int T, const int32_t* __restrict__ ids,
                 const float* __restrict__ wts, int k, const int32_t* __restrict__ owner,
                 const int32_t* __restrict__ local, int E, int world, const uint8_t* __restrict__ masks,
                 const int32_t* __restrict__ counts, int nchunks, long long* __restrict__ send_counts,
                 int32_t* __restrict__ order, int32_t* __restrict__ meta, int32_t* __restrict__ inv) {
    __shared__ int total[kEpMaxWorld], before[kEpMaxWorld], first[kEpMaxWorld];
    __shared__ int wpre[kChunk / 32][kEpMaxWorld];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chunk = blockIdx.x;

    // warp p: rank p's total over all chunks and over the chunks before this one
    if (warp < world) {
        int tot = 0, bef = 0;
        for (int c = lane; c < nchunks; c += 32) {
            const int v = counts[(size_t)c * world + warp];
            tot += v;
            if (c < chunk) bef += v;
        }
        for (int off = 16; off >= 1; off >>= 1) {
            tot += __shfl_xor_sync(0xffffffffu, tot, off);
            bef += __shfl_xor_sync(0xffffffffu, bef, off);
        }
        if (lane == 0) {
            total[warp] = tot;
            before[warp] = bef;
        }
    }
    const int t = chunk * kChunk + threadIdx.x;
    const unsigned mask = t < T ? masks[t] : 0u;
    for (int p = 0; p < world; ++p) {
        const unsigned b = __ballot_sync(0xffffffffu, (mask >> p) & 1u);
        if (lane == 0) wpre[warp][p] = __popc(b);
    }
    __syncthreads();
    if (threadIdx.x < world) {
        int f = 0;
        for (int q = 0; q < (int)threadIdx.x; ++q) f += total[q];
        first[threadIdx.x] = f + before[threadIdx.x];
        if (chunk == 0) send_counts[threadIdx.x] = total[threadIdx.x];
    }
    __syncthreads();
    for (int p = 0; p < world; ++p) {
        const unsigned b = __ballot_sync(0xffffffffu, (mask >> p) & 1u);
        if (t < T) {
            int row = -1;
            if ((mask >> p) & 1u) {
                int pre = 0;
                for (int w = 0; w < warp; ++w) pre += wpre[w][p];
                row = first[p] + pre + __popc(b & ((1u << lane) - 1u));
                int32_t* m = meta + (size_t)row * 2 * k;
                for (int s = 0; s < k; ++s) {
                    const int e = ids[(size_t)t * k + s];
                    const bool mine = e >= 0 && e < E && owner[e] == p;
                    m[s] = mine ? local[e] : -1;
                    m[k + s] = mine ? __float_as_int(wts[(size_t)t * k + s]) : 0;
                }
                order[row] = t;
            }
            inv[(size_t)p * T + t] = row;
        }
    }
}

// rows[r] = bf16(x[order[r]]) for r < the total row count: one warp per row at a time, 8
// elements (two float4 loads, one 16-byte store) per lane step, the loads of a lane's steps
// issued together.
__global__ void __launch_bounds__(256)
ep_copy_rows_kernel(const float* __restrict__ x, int H, const long long* __restrict__ send_counts, int world,
                    const int32_t* __restrict__ order, __nv_bfloat16* __restrict__ rows) {
    long long n = 0;
    for (int p = 0; p < world; ++p) n += send_counts[p];
    const int lane = threadIdx.x & 31;
    const int per_row = H / 8;
    for (long long r = blockIdx.x * 8LL + (threadIdx.x >> 5); r < n; r += gridDim.x * 8LL) {
        const float* src = x + (size_t)order[r] * H;
        __nv_bfloat16* dst = rows + (size_t)r * H;
        for (int c0 = 0; c0 < per_row; c0 += 32 * 4) {
            float4 a[4], b[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < per_row) {
                    a[u] = *reinterpret_cast<const float4*>(src + 8 * c);
                    b[u] = *reinterpret_cast<const float4*>(src + 8 * c + 4);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < per_row) {
                    __nv_bfloat162 o[4] = {__floats2bfloat162_rn(a[u].x, a[u].y), __floats2bfloat162_rn(a[u].z, a[u].w),
                                           __floats2bfloat162_rn(b[u].x, b[u].y), __floats2bfloat162_rn(b[u].z, b[u].w)};
                    *reinterpret_cast<uint4*>(dst + 8 * c) = *reinterpret_cast<uint4*>(o);
                }
            }
        }
    }
}

// out[t] = sum over ranks p ascending of partials[inv[p][t]] (rows with inv < 0 skipped; the sum
// starts from +0), then + add[t] when given. One thread per 4 columns of a token.
__global__ void ep_combine_kernel(const float* __restrict__ part, long long nrows, const int32_t* __restrict__ inv,
                                  int T, int world, int H, const float* __restrict__ add, float* __restrict__ out) {
    const int H4 = H / 4;
    const long long n = (long long)T * H4;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / H4), c = (int)(i - (long long)t * H4);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < world; ++p) {
            const int r = inv[(size_t)p * T + t];
            if (r < 0 || r >= nrows) continue;
            const float4 v = *reinterpret_cast<const float4*>(part + (size_t)r * H + 4 * c);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (add) {
            const float4 v = *reinterpret_cast<const float4*>(add + (size_t)t * H + 4 * c);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        *reinterpret_cast<float4*>(out + (size_t)t * H + 4 * c) = acc;
    }
}

// ---- peer path ----------------------------------------------------------------------------------

// The plan of the peer path: per token and destination rank, the row's position in the destination's
// slot `rank` (inv), its slot metadata stored into the destination's buffer, and the send order.
__global__ void __launch_bounds__(kChunk)
ep_peer_plan_kernel(EpPeers P, EpPeerLayout L, int T, const int32_t* __restrict__ ids, const float* __restrict__ wts,
                    const int32_t* __restrict__ owner, const int32_t* __restrict__ local, int E,
                    const uint8_t* __restrict__ masks, const int32_t* __restrict__ counts, int nchunks,
                    long long* __restrict__ send_counts, int32_t* __restrict__ order, int32_t* __restrict__ inv) {
    __shared__ int total[kEpMaxWorld], before[kEpMaxWorld], first[kEpMaxWorld];
    __shared__ int wpre[kChunk / 32][kEpMaxWorld];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int chunk = blockIdx.x, world = P.world, k = P.k;
    if (warp < world) {
        int tot = 0, bef = 0;
        for (int c = lane; c < nchunks; c += 32) {
            const int v = counts[(size_t)c * world + warp];
            tot += v;
            if (c < chunk) bef += v;
        }
        for (int off = 16; off >= 1; off >>= 1) {
            tot += __shfl_xor_sync(0xffffffffu, tot, off);
            bef += __shfl_xor_sync(0xffffffffu, bef, off);
        }
        if (lane == 0) {
            total[warp] = tot;
            before[warp] = bef;
        }
    }
    const int t = chunk * kChunk + threadIdx.x;
    const unsigned mask = t < T ? masks[t] : 0u;
    for (int p = 0; p < world; ++p) {
        const unsigned b = __ballot_sync(0xffffffffu, (mask >> p) & 1u);
        if (lane == 0) wpre[warp][p] = __popc(b);
    }
    __syncthreads();
    if (threadIdx.x < world) {
        int f = 0;
        for (int q = 0; q < (int)threadIdx.x; ++q) f += total[q];
        first[threadIdx.x] = f;
        if (chunk == 0) send_counts[threadIdx.x] = total[threadIdx.x];
    }
    __syncthreads();
    for (int p = 0; p < world; ++p) {
        const unsigned b = __ballot_sync(0xffffffffu, (mask >> p) & 1u);
        if (t < T) {
            int pos = -1;
            if ((mask >> p) & 1u) {
                int pre = 0;
                for (int w = 0; w < warp; ++w) pre += wpre[w][p];
                pos = before[p] + pre + __popc(b & ((1u << lane) - 1u));
                const size_t slot_row = (size_t)P.rank * P.cap + pos;
                int32_t* me = reinterpret_cast<int32_t*>(P.buf[p] + L.eid) + slot_row * k;
                float* mw = reinterpret_cast<float*>(P.buf[p] + L.w) + slot_row * k;
                for (int s = 0; s < k; ++s) {
                    const int e = ids[(size_t)t * k + s];
                    const bool mine = e >= 0 && e < E && owner[e] == p;
                    me[s] = mine ? local[e] : -1;
                    mw[s] = mine ? wts[(size_t)t * k + s] : 0.0f;
                }
                order[first[p] + pos] = t;
            }
            inv[(size_t)p * T + t] = pos;
        }
    }
    __threadfence_system();  // the metadata stores reach the destinations before the send kernel's flags
}

// Rows to the destinations (warp per row, 16-byte stores), then the grid's last CTA publishes the
// per-destination count and epoch.
__global__ void __launch_bounds__(256)
ep_peer_send_kernel(EpPeers P, EpPeerLayout L, const float* __restrict__ x, const long long* __restrict__ send_counts,
                    const int32_t* __restrict__ order, unsigned int* __restrict__ done) {
    const int world = P.world, H = P.H;
    long long first[kEpMaxWorld + 1];
    first[0] = 0;
    for (int p = 0; p < world; ++p) first[p + 1] = first[p] + send_counts[p];
    const long long n = first[world];
    const int lane = threadIdx.x & 31;
    const int per_row = H / 8;
    for (long long r = blockIdx.x * 8LL + (threadIdx.x >> 5); r < n; r += gridDim.x * 8LL) {
        int p = 0;
        while (r >= first[p + 1]) ++p;
        const float* src = x + (size_t)order[r] * H;
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(P.buf[p] + L.rows) +
                             ((size_t)P.rank * P.cap + (size_t)(r - first[p])) * H;
        for (int c0 = 0; c0 < per_row; c0 += 32 * 4) {
            float4 a[4], b[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < per_row) {
                    a[u] = *reinterpret_cast<const float4*>(src + 8 * c);
                    b[u] = *reinterpret_cast<const float4*>(src + 8 * c + 4);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int c = c0 + u * 32 + lane;
                if (c < per_row) {
                    __nv_bfloat162 o[4] = {__floats2bfloat162_rn(a[u].x, a[u].y), __floats2bfloat162_rn(a[u].z, a[u].w),
                                           __floats2bfloat162_rn(b[u].x, b[u].y), __floats2bfloat162_rn(b[u].z, b[u].w)};
                    *reinterpret_cast<uint4*>(dst + 8 * c) = *reinterpret_cast<uint4*>(o);
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(done, 1u) == gridDim.x - 1) {
            *done = 0u;  // for the next call
            __threadfence_system();
            for (int p = 0; p < world; ++p) {
                EpSig* sig = reinterpret_cast<EpSig*>(P.buf[p] + L.sig) + P.rank;
                sig->disp_count = (unsigned long long)send_counts[p];
                st_release_sys_u64(&sig->disp_epoch, P.epoch);
            }
        }
    }
}

// One lane per source rank: wait (bounded) for the source's rows of this epoch; its row count and
// whether the slot failed into the header of the local scratch.
__global__ void ep_peer_wait_kernel(EpPeers P, EpPeerLayout L, int* __restrict__ slot_counts,
                                    int* __restrict__ slot_fail) {
    const int q = threadIdx.x;
    if (q >= P.world) return;
    uint32_t* status = reinterpret_cast<uint32_t*>(P.buf[P.rank] + L.status);
    const EpSig* sig = reinterpret_cast<const EpSig*>(P.buf[P.rank] + L.sig) + q;
    bool ok = ld_acquire_sys_u64(&sig->disp_epoch) >= P.epoch;
    if (!ok) {
        const uint64_t t0 = global_timer_ns();
        while (!(ok = ld_acquire_sys_u64(&sig->disp_epoch) >= P.epoch)) {
            __nanosleep(256);
            if (global_timer_ns() - t0 > kEpWaitBudgetNs) break;
        }
    }
    unsigned long long n = ok ? *reinterpret_cast<const volatile unsigned long long*>(&sig->disp_count) : 0ull;
    int fail = 0;
    if (!ok) {
        set_status(status, kStatusWaitTimeout);
        fail = 1;
    } else if (n > (unsigned long long)P.cap) {
        set_status(status, kStatusBadCount);
        fail = 1;
    }
    slot_counts[q] = fail ? 0 : (int)n;
    slot_fail[q] = fail;
}

// out[t] = (sum over expert ranks p ascending, from +0, of bf16 partial row inv[p][t] of slot p) + add[t]
// after every rank's partial flag of this epoch; NaN rows when a wait failed or a failure is flagged.
__global__ void __launch_bounds__(256)
ep_peer_combine_kernel(EpPeers P, EpPeerLayout L, const int32_t* __restrict__ inv, int T,
                       const float* __restrict__ add, float* __restrict__ out) {
    __shared__ int bad;
    const int world = P.world, H = P.H, H8 = H / 8;
    if (threadIdx.x == 0) {
        uint32_t* status = reinterpret_cast<uint32_t*>(P.buf[P.rank] + L.status);
        int b = 0;
        for (int p = 0; p < world; ++p) {
            const EpSig* sig = reinterpret_cast<const EpSig*>(P.buf[P.rank] + L.sig) + p;
            unsigned long long f = ld_acquire_sys_u64(&sig->part_flag);
            if ((f >> 1) < P.epoch) {
                const uint64_t t0 = global_timer_ns();
                while (((f = ld_acquire_sys_u64(&sig->part_flag)) >> 1) < P.epoch) {
                    __nanosleep(256);
                    if (global_timer_ns() - t0 > kEpWaitBudgetNs) break;
                }
            }
            if ((f >> 1) < P.epoch) {
                set_status(status, kStatusWaitTimeout);
                b = 1;
            } else if (f & 1ull) {
                b = 1;
            }
        }
        if (*reinterpret_cast<volatile uint32_t*>(status) != 0u) b = 1;
        bad = b;
    }
    __syncthreads();
    const long long n = (long long)T * H8;
    const long long i0 = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    for (long long i = i0; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / H8), c = (int)(i - (long long)t * H8);
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (bad) {
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = __uint_as_float(0x7FC00000u);
        } else {
            for (int p = 0; p < world; ++p) {
                const int r = inv[(size_t)p * T + t];
                if (r < 0) continue;
                const uint4 v = *reinterpret_cast<const uint4*>(
                    reinterpret_cast<const uint16_t*>(P.buf[P.rank] + L.part) + ((size_t)p * P.cap + r) * H + 8 * c);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    acc[2 * j] = __fadd_rn(acc[2 * j], bf16lo(w[j]));
                    acc[2 * j + 1] = __fadd_rn(acc[2 * j + 1], bf16hi(w[j]));
                }
            }
            if (add) {
                const float4 a0 = *reinterpret_cast<const float4*>(add + (size_t)t * H + 8 * c);
                const float4 a1 = *reinterpret_cast<const float4*>(add + (size_t)t * H + 8 * c + 4);
                const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], av[j]);
            }
        }
        float* o = out + (size_t)t * H + 8 * c;
        *reinterpret_cast<float4*>(o) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4*>(o + 4) = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
}

}  // namespace

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

EpPeerLayout ep_peer_layout(int world, int cap, int H, int k) {
    EpPeerLayout d{};
    const size_t slots = (size_t)world * cap;
    size_t off = 0;
    d.status = off; off += kCtlClearBytes;  // status region (cleared whole after a failure)
    d.sig = off; off += align256(sizeof(EpSig) * kEpMaxWorld);
    d.eid = off; off += align256(slots * k * sizeof(int32_t));
    d.w = off; off += align256(slots * k * sizeof(float));
    d.rows = off; off += align256(slots * H * sizeof(uint16_t));
    d.part = off; off += align256(slots * H * sizeof(uint16_t));
    d.total = off;
    return d;
}

EpPeerScratch ep_peer_scratch(int world, int cap, int H, int I, int E, int k, bool int8, size_t prefill_bytes) {
    (void)H; (void)I; (void)E; (void)int8;
    EpPeerScratch d{};
    const size_t nchunks = ((size_t)cap + kChunk - 1) / kChunk;
    size_t off = 0;
    d.hdr = off; off += 256;
    d.masks = off; off += align256((size_t)cap);
    d.chunk_counts = off; off += align256(nchunks * world * sizeof(int32_t));
    d.order = off; off += align256((size_t)cap * world * sizeof(int32_t));
    d.send_counts = off; off += align256((size_t)world * sizeof(long long));
    d.prefill = off; off += align256(prefill_bytes);
    d.total = off;
    (void)k;
    return d;
}

cudaError_t launch_ep_peer_dispatch(const EpPeers& P, const float* x, int T, const int32_t* ids, const float* wts,
                                    const int32_t* owner, const int32_t* local, int E, int32_t* inv, char* ws,
                                    const EpPeerScratch& d, cudaStream_t st) {
    const EpPeerLayout L = ep_peer_layout(P.world, P.cap, P.H, P.k);
    const int nchunks = (T + kChunk - 1) / kChunk;
    uint8_t* masks = reinterpret_cast<uint8_t*>(ws + d.masks);
    int32_t* counts = reinterpret_cast<int32_t*>(ws + d.chunk_counts);
    int32_t* order = reinterpret_cast<int32_t*>(ws + d.order);
    long long* send_counts = reinterpret_cast<long long*>(ws + d.send_counts);
    unsigned int* done = reinterpret_cast<unsigned int*>(ws + d.hdr + kEpHdrDoneDispatch);
    if (nchunks > 0) {
        ep_count_kernel<<<nchunks, kChunk, 0, st>>>(ids, T, P.k, owner, E, P.world, masks, counts);
        ep_peer_plan_kernel<<<nchunks, kChunk, 0, st>>>(P, L, T, ids, wts, owner, local, E, masks, counts, nchunks,
                                                        send_counts, order, inv);
    } else {
        cudaError_t err = cudaMemsetAsync(send_counts, 0, sizeof(long long) * P.world, st);
        if (err != cudaSuccess) return err;
    }
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long max_rows = (long long)T * P.world;
    long long blocks = (max_rows + 7) / 8;
    if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
    if (blocks < 1) blocks = 1;
    ep_peer_send_kernel<<<(unsigned)blocks, 256, 0, st>>>(P, L, x, send_counts, order, done);
    return cudaGetLastError();
}

cudaError_t launch_ep_peer_wait(const EpPeers& P, char* ws, const EpPeerScratch& d, cudaStream_t st) {
    const EpPeerLayout L = ep_peer_layout(P.world, P.cap, P.H, P.k);
    ep_peer_wait_kernel<<<1, 32, 0, st>>>(P, L, reinterpret_cast<int*>(ws + d.hdr + kEpHdrSlotCounts),
                                          reinterpret_cast<int*>(ws + d.hdr + kEpHdrSlotFail));
    return cudaGetLastError();
}

cudaError_t launch_ep_peer_combine(const EpPeers& P, const int32_t* inv, int T, const float* add, float* out,
                                   cudaStream_t st) {
    const EpPeerLayout L = ep_peer_layout(P.world, P.cap, P.H, P.k);
    const long long n = (long long)T * (P.H / 8);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long blocks = (n + 255) / 256;
    if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
    if (blocks < 1) blocks = 1;
    ep_peer_combine_kernel<<<(unsigned)blocks, 256, 0, st>>>(P, L, inv, T, add, out);
    return cudaGetLastError();
}

size_t ep_dispatch_workspace_bytes(int T, int world) {
    const size_t nchunks = ((size_t)T + kChunk - 1) / kChunk;
    return align256((size_t)T) + align256(nchunks * world * sizeof(int32_t)) + (size_t)T * world * sizeof(int32_t);
}

cudaError_t launch_ep_dispatch(const float* x, int T, int H, const int32_t* ids, const float* wts, int k,
                               const int32_t* owner, const int32_t* local, int E, int world, long long* send_counts,
                               uint16_t* rows, int32_t* meta, int32_t* inv, void* ws, cudaStream_t st) {
    const int nchunks = (T + kChunk - 1) / kChunk;
    uint8_t* masks = reinterpret_cast<uint8_t*>(ws);
    int32_t* counts = reinterpret_cast<int32_t*>(masks + align256((size_t)T));
    int32_t* order = reinterpret_cast<int32_t*>(reinterpret_cast<char*>(counts) +
                                                align256((size_t)nchunks * world * sizeof(int32_t)));
    ep_count_kernel<<<nchunks, kChunk, 0, st>>>(ids, T, k, owner, E, world, masks, counts);
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    ep_plan_kernel<<<nchunks, kChunk, 0, st>>>(T, ids, wts, k, owner, local, E, world, masks, counts, nchunks,
                                               send_counts, order, meta, inv);
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long max_rows = (long long)T * world;
    long long blocks = (max_rows + 7) / 8;
    if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
    ep_copy_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(x, H, send_counts, world, order,
                                                          reinterpret_cast<__nv_bfloat16*>(rows));
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const float* part, long long nrows, const int32_t* inv, int T, int world, int H,
                              const float* add, float* out, cudaStream_t st) {
    const long long n = (long long)T * (H / 4);
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long blocks = (n + 255) / 256;
    if (blocks > (long long)sms * 8) blocks = (long long)sms * 8;
    ep_combine_kernel<<<(unsigned)blocks, 256, 0, st>>>(part, nrows, inv, T, world, H, add, out);
    return cudaGetLastError();
}

}  // namespace uocr
