// The MoE gate (MoEGate.__call__, unlimited_ocr_max/decoder.py:509-514) with the routing
// semantics of model_config.py:52-63,135-150: fp32 logits, optional per-expert bias (a
// benchmark input), softmax over all experts, greedy top-k, no renormalisation.
//
// Bit-exact with oracle/moe_oracle.c (oracle_route_fp32):
//   logit[t,j] = seg_0 + seg_1 + ... + seg_7 (ascending), seg_s = fma chain over
//                k in [s*H/8, (s+1)*H/8) ascending, from +0;
//   softmax: m = max_j logit; e_j = uocr_exp(logit_j - m); sum by the warp butterfly
//            (s_l = e_l + e_{l+32}, then xor 16, 8, 4, 2, 1); p_j = e_j / sum (IEEE div);
//   top-k:   k rounds of argmax by (p desc, index asc).
//
// One CTA serves kTT = 16 tokens with 256 threads (8 tokens and 128 threads for a large H). Thread (eg, s, tg) owns router rows
// j = eg + 16e (e = 0..3) over segment s and fma-chains them against the 8 tokens of token
// group tg: per 8 K elements it loads 4 x 16 B of router rows (L2) and 16 float4 of token rows
// from shared memory (each address shared by the 16 lanes of a half-warp, a broadcast) for 256
// FMAs. Lanes 0-15 = eg, lane bit 4 = low bit of s, warp = (tg, s >> 1). Two CTAs per SM.
// The FMA floor is T * 64 * H FMAs over 148 SMs x 128 FMA/clock.
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace uocr {

// Softmax over the token's logits (lane l holds experts l and l + 32, v0 / v1 = they exist) and
// greedy top-k by (probability desc, index asc); lane 0 writes ids / weights.
__device__ __forceinline__ void softmax_topk_warp(float l0, float l1, bool v0, bool v1, int topk, int lane,
                                                  int32_t* __restrict__ ids_row, float* __restrict__ wts_row) {
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
    // Each round: the largest probability, then the lowest expert index holding it. The
    // probabilities are >= +0, so their bit patterns order as signed integers; the taken (-2)
    // and absent (-1) entries are negative and never win while a valid one is left.
    for (int r = 0; r < topk; ++r) {
        const int b0 = __float_as_int(p0), b1 = __float_as_int(p1);
        const int m = __reduce_max_sync(0xffffffffu, b0 > b1 ? b0 : b1);
        const int cand = b0 == m ? lane : (b1 == m ? lane + 32 : 64);
        const int bi = __reduce_min_sync(0xffffffffu, cand);
        if (bi == lane) p0 = -2.0f;
        if (bi == lane + 32) p1 = -2.0f;
        if (lane == 0) {
            ids_row[r] = bi;
            wts_row[r] = __int_as_float(m);
        }
    }
}

// kTG token groups of 8 (2; 1 when the hidden size leaves too little shared memory)
template <int kTG>
__global__ void __launch_bounds__(128 * kTG, 2)
route_kernel(const float* __restrict__ x, int T, int H, const uint16_t* __restrict__ wg, int E,
             const float* __restrict__ bias, int topk, int32_t* __restrict__ ids_out, float* __restrict__ wts_out) {
    constexpr int kTT = 8 * kTG;
    constexpr int kRouteThreads = 128 * kTG;
    extern __shared__ float smem[];
    const int L = H / 8;     // segment length (multiple of 8)
    const int LP = L + 4;    // padded segment stride in floats
    float* xs = smem;                         // [kTT][8][LP]; reused as segs [kTT][64][8]
    float* segs = smem;
    const int region = kTT * 8 * LP > kTT * 64 * 8 ? kTT * 8 * LP : kTT * 64 * 8;
    float* logits = smem + region;            // [kTT][64]

    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * kTT;

    // stage the token rows (zeros past T): 16-byte cp.async copies, all in flight at once
    const int H4 = H / 4, L4 = L / 4;
    for (int i = tid; i < kTT * H4; i += kRouteThreads) {
        const int t = i / H4, k4 = i - t * H4;
        const int s = k4 / L4, kk4 = k4 - s * L4;
        const bool live = t0 + t < T;
        const float* src = live ? x + (size_t)(t0 + t) * H + 4 * k4 : x;
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(xs + (t * 8 + s) * LP + 4 * kk4);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(live ? 16 : 0)
                     : "memory");
    }
    asm volatile("cp.async.wait_all;\n" ::: "memory");
    __syncthreads();

    const int lane = tid & 31, warp = tid >> 5;
    const int eg = lane & 15;
    const int s = ((warp & 3) << 1) | (lane >> 4);
    const int tg = warp >> 2;
    float acc[4][8];
#pragma unroll
    for (int e = 0; e < 4; ++e)
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[e][t] = 0.0f;
    const float* xseg = xs + (tg * 8 * 8 + s) * LP;  // token tg*8 + t at xseg + t * 8 * LP
    for (int kk = 0; kk < L; kk += 8) {
        float wf[4][8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int j = eg + 16 * e;
            if (j < E) {
                unpack_bf16x8(*reinterpret_cast<const uint4*>(wg + (size_t)j * H + s * L + kk), wf[e]);
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) wf[e][q] = 0.0f;
            }
        }
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            const float4 xa = *reinterpret_cast<const float4*>(xseg + t * 8 * LP + kk);
            const float4 xb = *reinterpret_cast<const float4*>(xseg + t * 8 * LP + kk + 4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                float a = acc[e][t];
                a = __fmaf_rn(wf[e][0], xa.x, a);
                a = __fmaf_rn(wf[e][1], xa.y, a);
                a = __fmaf_rn(wf[e][2], xa.z, a);
                a = __fmaf_rn(wf[e][3], xa.w, a);
                a = __fmaf_rn(wf[e][4], xb.x, a);
                a = __fmaf_rn(wf[e][5], xb.y, a);
                a = __fmaf_rn(wf[e][6], xb.z, a);
                a = __fmaf_rn(wf[e][7], xb.w, a);
                acc[e][t] = a;
            }
        }
    }
    __syncthreads();  // token rows consumed: the region becomes segs
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int j = eg + 16 * e;
#pragma unroll
        for (int t = 0; t < 8; ++t) segs[((tg * 8 + t) * 64 + j) * 8 + s] = acc[e][t];
    }
    __syncthreads();
    for (int i = tid; i < kTT * 64; i += kRouteThreads) {
        const int t = i >> 6, j = i & 63;
        if (j < E) {
            const float* sg = segs + (t * 64 + j) * 8;
            float total = sg[0];
#pragma unroll
            for (int q = 1; q < 8; ++q) total = __fadd_rn(total, sg[q]);
            if (bias) total = __fadd_rn(total, bias[j]);
            logits[t * 64 + j] = total;
        }
    }
    __syncthreads();

    // softmax + top-k: warp w serves tokens w and w + 8 of the tile
    for (int t = warp; t < kTT && t0 + t < T; t += kRouteThreads / 32) {
        const bool v0 = lane < E, v1 = lane + 32 < E;
        const float l0 = v0 ? logits[t * 64 + lane] : -INFINITY;
        const float l1 = v1 ? logits[t * 64 + lane + 32] : -INFINITY;
        softmax_topk_warp(l0, l1, v0, v1, topk, lane, ids_out + (size_t)(t0 + t) * topk, wts_out + (size_t)(t0 + t) * topk);
    }
}

// Persistent variant for hidden sizes whose router fits in shared memory (H <= 1280 among multiples of 64): the CTA
// stages the whole router once, rows padded by 16 bytes (a warp's 32 rows at one K offset fall in
// distinct banks), then walks tiles of kRT tokens. Eight FMA warps: warp w owns segment s = w,
// lane l experts l and l + 32, for the tile's kRT tokens (8 chains); token rows arrive by
// cp.async one tile ahead (issued after the FMA warps' barrier that retires the buffer's previous
// tile). kRT finishing warps take each tile's segment partials from one of two buffers (handed
// over by mbarriers) and finish one token each (sum of the 8 partials, bias, softmax, top-k), so
// the FMA warps never wait for a softmax. Every mbarrier wait is bounded.
constexpr int kRT = 4;
constexpr int kRouteFmaThreads = 256;
constexpr int kRouteSmemThreads = kRouteFmaThreads + 32 * kRT;
constexpr uint32_t kRouteWaitPolls = 1u << 24;  // far beyond any legitimate wait; never hangs

UOCR_DEV void route_stage_tokens(const float* __restrict__ x, int T, int H, int t0, float* dst, int tid) {
    const int H4 = H / 4;
    for (int i = tid; i < kRT * H4; i += kRouteFmaThreads) {
        const int t = i / H4;
        const bool live = t0 + t < T;
        const float* src = live ? x + (size_t)(t0 + t) * H + 4 * (i - t * H4) : x;
        const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst + 4 * i);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(live ? 16 : 0) : "memory");
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
}

UOCR_DEV void route_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kRouteWaitPolls && !mbar_try_wait(bar, parity); ++i) {
    }
}

// Softmax + greedy top-k of one token from its [64][8] segment partials (the finishing warps).
UOCR_DEV void route_finish_token(const float* sg, int E, const float* __restrict__ bias, int topk, int lane,
                                 int32_t* __restrict__ ids_row, float* __restrict__ wts_row) {
    const bool v0 = lane < E, v1 = lane + 32 < E;
    float l0 = sg[lane * 8], l1 = sg[(lane + 32) * 8];
#pragma unroll
    for (int q = 1; q < 8; ++q) {
        l0 = __fadd_rn(l0, sg[lane * 8 + q]);
        l1 = __fadd_rn(l1, sg[(lane + 32) * 8 + q]);
    }
    if (bias) {
        if (v0) l0 = __fadd_rn(l0, bias[lane]);
        if (v1) l1 = __fadd_rn(l1, bias[lane + 32]);
    }
    softmax_topk_warp(v0 ? l0 : -INFINITY, v1 ? l1 : -INFINITY, v0, v1, topk, lane, ids_row, wts_row);
}

__global__ void __launch_bounds__(kRouteSmemThreads, 1)
route_smem_kernel(const float* __restrict__ x, int T, int H, const uint16_t* __restrict__ wg, int E,
                  const float* __restrict__ bias, int topk, int32_t* __restrict__ ids_out, float* __restrict__ wts_out) {
    extern __shared__ __align__(16) unsigned char rsm[];
    __shared__ uint64_t segs_full[2], segs_free[2];
    const int RS = H + 8;  // router row stride in bf16 elements
    uint16_t* wr = reinterpret_cast<uint16_t*>(rsm);                            // [64][RS]
    float* xs = reinterpret_cast<float*>(rsm + (size_t)64 * RS * 2);            // [2][kRT][H]
    float* segs = xs + 2 * kRT * H;                                             // [2][kRT][64][8]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int L = H / 8;
    const int ntiles = (T + kRT - 1) / kRT;

    if (tid == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&segs_full[i], kRouteFmaThreads);
            mbar_init(&segs_free[i], 32 * kRT);
        }
        fence_mbar_init();
    }
    if (tid < kRouteFmaThreads) {
        // router rows (zeros for j >= E), 16-byte copies, and the first tile's token rows
        const int H8 = H / 8;
        for (int i = tid; i < 64 * H8; i += kRouteFmaThreads) {
            const int j = i / H8, c = i - j * H8;
            const bool live = j < E;
            const uint16_t* src = live ? wg + (size_t)j * H + 8 * c : wg;
            const uint32_t d = (uint32_t)__cvta_generic_to_shared(wr + (size_t)j * RS + 8 * c);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(live ? 16 : 0)
                         : "memory");
        }
        asm volatile("cp.async.commit_group;\n" ::: "memory");
        if ((int)blockIdx.x < ntiles) route_stage_tokens(x, T, H, blockIdx.x * kRT, xs, tid);
    }
    __syncthreads();  // barrier initialisation visible to all warps

    if (tid < kRouteFmaThreads) {
        const int s = warp;
        const uint16_t* w0 = wr + (size_t)lane * RS + s * L;
        const uint16_t* w1 = wr + (size_t)(lane + 32) * RS + s * L;
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
            const int buf = it & 1;
            asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            // this tile's token rows (and, first time, the router) are in place; every FMA warp is
            // done with the other token buffer
            named_bar_sync(1, kRouteFmaThreads);
            const int next = tile + gridDim.x;
            if (next < ntiles) route_stage_tokens(x, T, H, next * kRT, xs + (buf ^ 1) * kRT * H, tid);
            const float* xt = xs + buf * kRT * H + s * L;
            float acc0[kRT], acc1[kRT];
#pragma unroll
            for (int t = 0; t < kRT; ++t) acc0[t] = acc1[t] = 0.0f;
#pragma unroll 4
            for (int kk = 0; kk < L; kk += 8) {
                float a[8], b[8];
                unpack_bf16x8(*reinterpret_cast<const uint4*>(w0 + kk), a);
                unpack_bf16x8(*reinterpret_cast<const uint4*>(w1 + kk), b);
#pragma unroll
                for (int t = 0; t < kRT; ++t) {
                    const float4 xa = *reinterpret_cast<const float4*>(xt + t * H + kk);
                    const float4 xb = *reinterpret_cast<const float4*>(xt + t * H + kk + 4);
                    const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                    float u = acc0[t], v = acc1[t];
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        u = __fmaf_rn(a[q], xv[q], u);
                        v = __fmaf_rn(b[q], xv[q], v);
                    }
                    acc0[t] = u;
                    acc1[t] = v;
                }
            }
            // the finishing warps are done with this buffer's previous tile (two tiles ago)
            if (it >= 2) route_wait(&segs_free[buf], ((it >> 1) - 1) & 1);
            float* so = segs + buf * kRT * 64 * 8;
#pragma unroll
            for (int t = 0; t < kRT; ++t) {
                so[(t * 64 + lane) * 8 + s] = acc0[t];
                so[(t * 64 + lane + 32) * 8 + s] = acc1[t];
            }
            mbar_arrive(&segs_full[buf]);
        }
        asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    } else {
        const int fw = warp - kRouteFmaThreads / 32;  // token fw of each tile
        int it = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
            const int buf = it & 1;
            route_wait(&segs_full[buf], (it >> 1) & 1);
            const float* sb = segs + buf * kRT * 64 * 8;
            {
                const int t = fw, tok = tile * kRT + t;
                if (tok < T)
                    route_finish_token(sb + t * 64 * 8, E, bias, topk, lane, ids_out + (size_t)tok * topk,
                                       wts_out + (size_t)tok * topk);
            }
            mbar_arrive(&segs_free[buf]);
        }
    }
}

size_t route_persistent_smem_bytes(int H) {
    return (size_t)64 * (H + 8) * 2 + (size_t)2 * kRT * H * 4 + (size_t)2 * kRT * 64 * 8 * 4;
}

size_t route_smem_bytes(int tt, int H) {
    const int LP = H / 8 + 4;
    size_t region = (size_t)tt * 8 * LP;                    // token rows
    if (region < (size_t)tt * 64 * 8) region = (size_t)tt * 64 * 8;  // or the segment partials
    return sizeof(float) * (region + (size_t)tt * 64);
}

cudaError_t launch_route(const float* x, int T, int H, const uint16_t* wg, int E, const float* bias, int topk,
                         int32_t* ids, float* wts, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    int dev = 0, optin = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (err != cudaSuccess) return err;
    const size_t psmem = route_persistent_smem_bytes(H);
    if (psmem + 64 <= (size_t)optin) {  // + the kernel's static mbarriers
        int sms = 148;
        err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (err != cudaSuccess) return err;
        err = ensure_smem_optin(reinterpret_cast<const void*>(route_smem_kernel), psmem);
        if (err != cudaSuccess) return err;
        const int ntiles = (T + kRT - 1) / kRT;
        route_smem_kernel<<<ntiles < sms ? ntiles : sms, kRouteSmemThreads, psmem, st>>>(x, T, H, wg, E, bias, topk,
                                                                                          ids, wts);
    } else if (route_smem_bytes(16, H) <= (size_t)optin / 2) {
        const size_t smem = route_smem_bytes(16, H);
        err = ensure_smem_optin(reinterpret_cast<const void*>(route_kernel<2>), smem);
        if (err != cudaSuccess) return err;
        route_kernel<2><<<(T + 15) / 16, 256, smem, st>>>(x, T, H, wg, E, bias, topk, ids, wts);
    } else {
        const size_t smem = route_smem_bytes(8, H);
        err = ensure_smem_optin(reinterpret_cast<const void*>(route_kernel<1>), smem);
        if (err != cudaSuccess) return err;
        route_kernel<1><<<(T + 7) / 8, 128, smem, st>>>(x, T, H, wg, E, bias, topk, ids, wts);
    }
    return cudaGetLastError();
}

}  // namespace uocr
