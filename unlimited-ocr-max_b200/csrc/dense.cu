// Dense bf16 projections of the decode step (attention q/k/v/o, the dense FFN of layer 0, lm_head):
// out[m, n] = sum_k W[n, k] x[m, k] for M <= 8 rows, W streamed once from HBM through the tensor
// cores. Replaces dense_bf16_qmv (kernels/dense_bf16.mojo:119-158; decoder.py:166-184, 236-238)
// for callers that pack the weight once at load.
//
// Packed weight: W padded with zero rows to a multiple of 128 (row blocks, the MMA's M) and zero
// columns to a multiple of 128 (items), then [row block][item][2 atoms][128 rows x 128 B]: each
// atom one 64-element K range of 128 rows in the 128-byte-swizzle K-major layout, so an item
// (32 KB) copied verbatim into shared memory is the MMA's A operand (the down-projection layout
// of the expert stacks).
//
// The x operand: per K range of 64 elements one 16-row image (2 KB), rows 2t and 2t + 1 holding
// bf16(x[t]) and bf16(x[t] - bf16(x[t])) (zero rows for t >= M); x is represented to ~2^-17 of
// its magnitude and every product is exact in the tensor core's fp32 accumulation, so
// out = acc[2t] + acc[2t + 1] differs from the fp32 dot product by the accumulation order only.
//
// Work split over the SMs: the items of a row block form KC chunks of at most
// kDenseMaxChunkItems items; CTA i works on chunk i % KC of row blocks i / KC, i / KC + G', ...
// (G' = CTAs per chunk), so every CTA builds one x image (its chunk) at the start. KC = 1 when the
// row blocks alone fill the GPU (lm_head: 1010 row blocks); narrow weights split K into at most
// kDenseMaxSplit chunks (q/k/v/o: 10 row blocks x 5 chunks of two items) and the CTA that
// completes a row block's last chunk sums the chunks' fp32 partials in chunk order
// (deterministic), every chunk's loads in flight at once.
//
// Per CTA (256 threads): warp 0 streams items (one 32 KB bulk copy each, L2 evict-first) into a
// kDenseStages ring from the kernel's first microsecond -- launched with programmatic dependent
// launch, the weights of a projection stream while the previous kernel of the stream finishes --
// while warps 2-7 wait for the previous grid (griddepcontrol.wait) and build the x image; warp 1
// issues tcgen05.mma kind::f16 (M 128, N 16, K 16; 8 per item) into one of two 16-column TMEM
// accumulators per row block; warps 4-7 read the accumulator back
// (tcgen05.ld, one TMEM lane per weight row) and write out (or the partials). Every wait is
// bounded; a timeout records kStatusWaitTimeout in the workspace's status word.
//
// Bound: HBM. Algorithmic bytes per call: N x K x 2 (the weight) + M x (K + N) x 4.
#include "common.cuh"
#include "kernels.h"
#include "layout.h"
#include "sm100.cuh"

namespace uocr {
namespace {

constexpr int kDenseStages = 5;
constexpr int kDenseItemBytes = 2 * kAtomBytes;    // 32 KB: 128 rows x 128 K
constexpr int kTermAtomRows = 16;                  // 8 tokens x 2 terms
constexpr int kTermAtom = kTermAtomRows * 128;     // 2 KB: one 64-element K range of the x image
constexpr int kDenseImgItemBytes = 2 * kTermAtom;  // x image of one item's K range
constexpr int kDenseThreads = 256;
constexpr uint32_t kIdesc = umma_idesc_bf16(128, 16);
constexpr size_t kDenseSmemBytes = 1024 + (size_t)kDenseStages * kDenseItemBytes +
                                   (size_t)kDenseMaxChunkItems * kDenseImgItemBytes + 256;

struct DenseArgs {
    const unsigned char* w;  // packed weight
    const float* x;          // [M, K]
    float* out;              // [M, N]
    float* partial;          // [NB][KC][128 rows][8 rows of x] (KC > 1)
    uint32_t* ctl;           // status word at [0], per-row-block counters at [kDenseCtlCounters + rb]
    int M, N, Npad, K, NB, IPR, KC, IPC, Gp;
    int xvec;  // x 16-byte aligned: float4 loads
};

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return uint32_t(f32_to_bf16_rne(lo)) | (uint32_t(f32_to_bf16_rne(hi)) << 16);
}

__global__ void __launch_bounds__(kDenseThreads, 1) dense_stream_kernel(DenseArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    unsigned char* ring = smem;
    unsigned char* img = ring + kDenseStages * kDenseItemBytes;
    uint64_t* full = reinterpret_cast<uint64_t*>(img + kDenseMaxChunkItems * kDenseImgItemBytes);
    uint64_t* empty = full + kDenseStages;
    uint64_t* tfull = empty + kDenseStages;
    uint64_t* tempty = tfull + 2;
    uint64_t* mdone = tempty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
    int* flags = reinterpret_cast<int*>(tmem_slot + 1);  // [0] last-chunk decision, [1] failure
    uint32_t* status = a.ctl;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = blockIdx.x % a.KC;
    const int j0 = blockIdx.x / a.KC;
    const int it0 = chunk * a.IPC;
    const int nit = min(a.IPR, it0 + a.IPC) - it0;
    const int nrb = j0 < a.NB ? (a.NB - 1 - j0) / a.Gp + 1 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kDenseStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], 4);
        }
        mbar_init(mdone, 1);
        flags[0] = flags[1] = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, 32);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // the next kernel of the stream may start its CTAs (and stream its weights) on the SMs this
    // grid leaves free; it reads nothing of ours before its own griddepcontrol.wait
    pdl_launch_dependents();

    if (warp >= 2) {
        // x image of this CTA's chunk, by warps 2-7 while warp 0 already streams the weights: rows
        // 2t / 2t + 1 = bf16(x) / bf16(x - bf16(x)), zero for t >= M and k >= K. x is the previous
        // kernel's output: wait for that grid first (programmatic dependent launch).
        pdl_wait_prior_grid();
        const int quads = nit * 32;  // 4-element groups per token
        const int tid = threadIdx.x - 64, nthr = kDenseThreads - 64;
        for (int base = tid; base < 8 * quads; base += 4 * nthr) {
            float v[4][4];
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int idx = base + b * nthr;
                const int tt = idx / quads, k = it0 * 128 + 4 * (idx % quads);
#pragma unroll
                for (int e = 0; e < 4; ++e) v[b][e] = 0.f;
                if (idx < 8 * quads && tt < a.M) {
                    const float* src = a.x + (size_t)tt * a.K + k;
                    if (a.xvec && k + 3 < a.K) {
                        const float4 f = __ldg(reinterpret_cast<const float4*>(src));
                        v[b][0] = f.x, v[b][1] = f.y, v[b][2] = f.z, v[b][3] = f.w;
                    } else {
#pragma unroll
                        for (int e = 0; e < 4; ++e)
                            if (k + e < a.K) v[b][e] = __ldg(src + e);
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int idx = base + b * nthr;
                if (idx >= 8 * quads) break;
                const int tt = idx / quads, kl = 4 * (idx % quads);
                float lo[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) lo[e] = v[b][e] - bf16f(f32_to_bf16_rne(v[b][e]));
                unsigned char* atom = img + (kl >> 6) * kTermAtom;
                const int cb = (kl & 63) * 2;
                *reinterpret_cast<uint2*>(atom + atom_offset(2 * tt, cb)) =
                    make_uint2(pack_bf16x2(v[b][0], v[b][1]), pack_bf16x2(v[b][2], v[b][3]));
                *reinterpret_cast<uint2*>(atom + atom_offset(2 * tt + 1, cb)) =
                    make_uint2(pack_bf16x2(lo[0], lo[1]), pack_bf16x2(lo[2], lo[3]));
            }
        }
        fence_proxy_async_smem();
    }
    // the image is complete before the MMA warp issues (warps 1-7)
    if (warp >= 1) named_bar_sync(2, kDenseThreads - 32);

    if (warp == 0) {
        // ---- producer: the chunk's items of each row block, one bulk copy each
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int k = 0;
            bool ok = true;
            for (int u = 0; u < nrb && ok; ++u) {
                const unsigned char* src = a.w + ((size_t)(j0 + u * a.Gp) * a.IPR + it0) * kDenseItemBytes;
                for (int i = 0; i < nit; ++i) {
                    const int s = k % kDenseStages;
                    if (!mbar_wait(&empty[s], ((k / kDenseStages) & 1) ^ 1, status)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[s], kDenseItemBytes);
                    bulk_g2s_hint(ring + s * kDenseItemBytes, src + (size_t)i * kDenseItemBytes, kDenseItemBytes,
                                  &full[s], pol);
                    ++k;
                }
            }
            // every copy issued has landed before the CTA may leave (bounded)
            for (int s = 0; s < kDenseStages && s < k; ++s) {
                const int last = s + ((k - 1 - s) / kDenseStages) * kDenseStages;
                mbar_wait(&full[s], (last / kDenseStages) & 1, status);
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        tc_fence_after();
        if (lane == 0) {
            int k = 0;
            bool ok = true;
            for (int u = 0; u < nrb && ok; ++u) {
                const int b = u & 1;
                if (!mbar_wait(&tempty[b], ((u >> 1) & 1) ^ 1, status)) break;
                tc_fence_after();
                const uint32_t acc = tmem + 16u * (uint32_t)b;
                for (int i = 0; i < nit; ++i, ++k) {
                    const int s = k % kDenseStages;
                    if (!mbar_wait(&full[s], (k / kDenseStages) & 1, status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = smem_addr(ring + s * kDenseItemBytes);
                    const uint32_t xs = smem_addr(img + i * kDenseImgItemBytes);
#pragma unroll
                    for (int at = 0; at < 2; ++at)
#pragma unroll
                        for (int s4 = 0; s4 < 4; ++s4)
                            umma_f16(acc, umma_desc_sw128(st + at * kAtomBytes + 32 * s4),
                                     umma_desc_sw128(xs + at * kTermAtom + 32 * s4), kIdesc, (i | at | s4) != 0);
                    umma_commit(&empty[s]);
                }
                if (ok) umma_commit(&tfull[b]);
            }
            // every MMA issued has completed before the accumulators are freed (bounded)
            umma_commit(mdone);
            mbar_wait(mdone, 0, status);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---- epilogue: accumulator -> out (or the chunk's partials)
        const int q = warp & 3;
        const int r = 32 * q + lane;
        const bool split = a.KC > 1;
        for (int u = 0; u < nrb; ++u) {
            const int b = u & 1;
            const int rb = j0 + u * a.Gp;
            const bool got = mbar_wait_warp(&tfull[b], (u >> 1) & 1, nullptr, status);
            float y[8];
            if (got) {
                tc_fence_after();
                uint32_t v[16];
                tmem_ld_32x32b_x16(tmem + ((uint32_t)(32 * q) << 16) + 16u * (uint32_t)b, v);
                tmem_wait_ld();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[b]);
#pragma unroll
                for (int t = 0; t < 8; ++t) y[t] = __uint_as_float(v[2 * t]) + __uint_as_float(v[2 * t + 1]);
            }
            const int n = rb * 128 + r;
            if (!split) {
                if (!got) break;
                if (n < a.N)
                    for (int t = 0; t < a.M; ++t) a.out[(size_t)t * a.N + n] = y[t];
                continue;
            }
            // split K: publish this chunk's partial (the row's 8 values, 32 contiguous bytes); the
            // CTA whose arrival completes the row block sums the chunks' partials. Ordering: the
            // CTA barrier, then one acquire-release counter add by one thread (publishes the
            // CTA's stores, and makes the other chunks' visible to the last one)
            float4* mine = reinterpret_cast<float4*>(a.partial + (((size_t)rb * a.KC + chunk) * 128 + r) * 8);
            if (got) {
                mine[0] = make_float4(y[0], y[1], y[2], y[3]);
                mine[1] = make_float4(y[4], y[5], y[6], y[7]);
            } else if (lane == 0) {
                atomicOr(&flags[1], 1);
            }
            named_bar_sync(1, 128);
            const bool failed = *reinterpret_cast<volatile int*>(&flags[1]) != 0;
            if (threadIdx.x == 128 && !failed) {
                const uint32_t old = atom_acq_rel_gpu_add(&a.ctl[kDenseCtlCounters + rb], 1u);
                flags[0] = old == (uint32_t)(a.KC - 1);
            }
            named_bar_sync(1, 128);
            if (failed) break;
            if (*reinterpret_cast<volatile int*>(&flags[0])) {
                if (n < a.N) {
                    // sum over the chunks in ascending order, kDenseMaxSplit chunks' loads in flight
                    const float4* row = reinterpret_cast<const float4*>(a.partial + ((size_t)rb * a.KC * 128 + r) * 8);
                    float s[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) s[e] = 0.f;
                    for (int c0 = 0; c0 < a.KC; c0 += kDenseMaxSplit) {
                        float4 pv[kDenseMaxSplit][2];
#pragma unroll
                        for (int cc = 0; cc < kDenseMaxSplit; ++cc) {
                            if (c0 + cc < a.KC) {
                                pv[cc][0] = __ldcg(row + (size_t)(c0 + cc) * 256);
                                pv[cc][1] = __ldcg(row + (size_t)(c0 + cc) * 256 + 1);
                            }
                        }
#pragma unroll
                        for (int cc = 0; cc < kDenseMaxSplit; ++cc) {
                            if (c0 + cc < a.KC) {
                                s[0] += pv[cc][0].x, s[1] += pv[cc][0].y, s[2] += pv[cc][0].z, s[3] += pv[cc][0].w;
                                s[4] += pv[cc][1].x, s[5] += pv[cc][1].y, s[6] += pv[cc][1].z, s[7] += pv[cc][1].w;
                            }
                        }
                    }
                    for (int tt = 0; tt < a.M; ++tt) a.out[(size_t)tt * a.N + n] = s[tt];
                }
                if (threadIdx.x == 128) a.ctl[kDenseCtlCounters + rb] = 0;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, 32);
    }
}

__global__ void dense_pack_kernel(const uint16_t* __restrict__ w, bool kblocked, int N, int K, int IPR,
                                  long long chunks, unsigned char* __restrict__ out) {
    for (long long p = blockIdx.x * (long long)blockDim.x + threadIdx.x; p < chunks;
         p += (long long)gridDim.x * blockDim.x) {
        const long long item = p >> 11;  // 2048 16-byte chunks per 32 KB item
        const int rem = static_cast<int>(p & 2047);
        const int at = rem >> 10, r = (rem >> 3) & 127, pc = rem & 7;
        const int cj = pc ^ (r & 7);  // logical 16-byte chunk held at physical chunk pc
        const int rb = static_cast<int>(item / IPR), it = static_cast<int>(item % IPR);
        const int n = rb * 128 + r, k = it * 128 + at * 64 + cj * 8;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (n < N && k < K) {
            const uint16_t* src = kblocked ? w + ((size_t)(k >> 4) * N + n) * 16 + (k & 15) : w + (size_t)n * K + k;
            v = *reinterpret_cast<const uint4*>(src);
        }
        *reinterpret_cast<uint4*>(out + p * 16) = v;
    }
}

}  // namespace

DensePlan dense_plan(long long N, long long K, int sms) {
    DensePlan p{};
    p.NB = static_cast<int>((N + 127) / 128);
    p.IPR = static_cast<int>((K + 127) / 128);
    const int kc_min = (p.IPR + kDenseMaxChunkItems - 1) / kDenseMaxChunkItems;
    int kc = p.NB >= sms ? kc_min
                         : std::max(kc_min, std::min(std::min(p.IPR, kDenseMaxSplit), std::max(1, sms / p.NB)));
    p.IPC = (p.IPR + kc - 1) / kc;
    p.KC = (p.IPR + p.IPC - 1) / p.IPC;
    p.Gp = std::max(1, std::min(p.NB, sms / p.KC));
    p.grid = p.KC * p.Gp;
    return p;
}

cudaError_t launch_dense_pack(const uint16_t* w, bool kblocked, int N, int K, unsigned char* out, cudaStream_t st) {
    const DensePlan p = dense_plan(N, K, 1);
    const long long chunks = (long long)p.NB * p.IPR * 2048;
    const int grid = static_cast<int>(std::min<long long>((chunks + 255) / 256, 148 * 16));
    dense_pack_kernel<<<grid, 256, 0, st>>>(w, kblocked, N, K, p.IPR, chunks, out);
    return cudaGetLastError();
}

cudaError_t launch_dense_stream(const unsigned char* w, int N, int K, const float* x, int M, float* out,
                                uint32_t* ctl, float* partial, const DensePlan& p, cudaStream_t st) {
    cudaError_t err = ensure_smem_optin(reinterpret_cast<const void*>(dense_stream_kernel), kDenseSmemBytes);
    if (err != cudaSuccess) return err;
    DenseArgs a{w, x, out, partial, ctl, M, N, p.NB * 128, K, p.NB, p.IPR, p.KC, p.IPC, p.Gp,
                (reinterpret_cast<uintptr_t>(x) & 15) == 0};
    // programmatic dependent launch: the grid may start while the previous kernel of the stream
    // finishes; everything it reads or writes that a previous kernel may touch (x, out, the
    // workspace) comes after its griddepcontrol.wait
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kDenseThreads);
    cfg.dynamicSmemBytes = kDenseSmemBytes;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    void* args[] = {&a};
    return cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(dense_stream_kernel), args);
}

}  // namespace uocr
