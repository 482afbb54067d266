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
// One CTA serves kTT tokens with 512 threads = 64 experts x 8 segments: thread (j, s)
// streams router row j's segment s once and fma-chains it against all kTT tokens, whose
// rows sit in shared memory padded so the 8 segments' reads fall in distinct banks.
#include "common.cuh"
#include "kernels.h"

namespace uocr {

constexpr int kRouteThreads = 512;

template <int kTT>
__global__ void __launch_bounds__(kRouteThreads)
route_kernel(const float* __restrict__ x, int T, int H, const uint16_t* __restrict__ wg, int E,
             const float* __restrict__ bias, int topk, int32_t* __restrict__ ids_out, float* __restrict__ wts_out) {
    extern __shared__ float smem[];
    const int L = H / 8;     // segment length (multiple of 8)
    const int LP = L + 4;    // padded segment stride in floats
    float* xs = smem;                         // [kTT][8][LP]
    float* segs = xs + kTT * 8 * LP;          // [kTT][64][8]
    float* logits = segs + kTT * 64 * 8;      // [kTT][64]

    const int tid = threadIdx.x;
    const int t0 = blockIdx.x * kTT;

    // stage the token rows (zeros past T)
    for (int i = tid; i < kTT * H; i += kRouteThreads) {
        const int t = i / H, k = i - t * H;
        const int s = k / L, kk = k - s * L;
        xs[(t * 8 + s) * LP + kk] = (t0 + t < T) ? x[(size_t)(t0 + t) * H + k] : 0.0f;
    }
    __syncthreads();

    const int j = tid >> 3;
    const int s = tid & 7;
    if (j < E) {
        float acc[kTT];
#pragma unroll
        for (int t = 0; t < kTT; ++t) acc[t] = 0.0f;
        const uint16_t* wrow = wg + (size_t)j * H + s * L;
        const float* xseg = xs + s * LP;
        for (int kk = 0; kk < L; kk += 8) {
            float wf[8];
            unpack_bf16x8(*reinterpret_cast<const uint4*>(wrow + kk), wf);
#pragma unroll
            for (int t = 0; t < kTT; ++t) {
                const float4 xa = *reinterpret_cast<const float4*>(xseg + t * 8 * LP + kk);
                const float4 xb = *reinterpret_cast<const float4*>(xseg + t * 8 * LP + kk + 4);
                float a = acc[t];
                a = __fmaf_rn(wf[0], xa.x, a);
                a = __fmaf_rn(wf[1], xa.y, a);
                a = __fmaf_rn(wf[2], xa.z, a);
                a = __fmaf_rn(wf[3], xa.w, a);
                a = __fmaf_rn(wf[4], xb.x, a);
                a = __fmaf_rn(wf[5], xb.y, a);
                a = __fmaf_rn(wf[6], xb.z, a);
                a = __fmaf_rn(wf[7], xb.w, a);
                acc[t] = a;
            }
        }
#pragma unroll
        for (int t = 0; t < kTT; ++t) segs[(t * 64 + j) * 8 + s] = acc[t];
    }
    __syncthreads();
    if (s == 0 && j < E) {
        for (int t = 0; t < kTT; ++t) {
            const float* sg = segs + (t * 64 + j) * 8;
            float total = sg[0];
#pragma unroll
            for (int q = 1; q < 8; ++q) total = __fadd_rn(total, sg[q]);
            if (bias) total = __fadd_rn(total, bias[j]);
            logits[t * 64 + j] = total;
        }
    }
    __syncthreads();

    // softmax + top-k: warp w serves token w of the tile
    const int warp = tid >> 5, lane = tid & 31;
    if (warp < kTT && t0 + warp < T) {
        const int t = warp;
        const bool v0 = lane < E, v1 = lane + 32 < E;
        const float l0 = v0 ? logits[t * 64 + lane] : -INFINITY;
        const float l1 = v1 ? logits[t * 64 + lane + 32] : -INFINITY;
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
        const size_t row = (size_t)(t0 + t) * topk;
        for (int r = 0; r < topk; ++r) {
            // lane-local best: lower index (lane) wins a tie with lane + 32
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
                ids_out[row + r] = bi;
                wts_out[row + r] = bp;
            }
        }
    }
}

size_t route_smem_bytes(int tt, int H) {
    const int LP = H / 8 + 4;
    return sizeof(float) * ((size_t)tt * 8 * LP + (size_t)tt * 64 * 8 + (size_t)tt * 64);
}

cudaError_t launch_route(const float* x, int T, int H, const uint16_t* wg, int E, const float* bias, int topk,
                         int32_t* ids, float* wts, cudaStream_t st) {
    if (T <= 0) return cudaSuccess;
    constexpr int TT = 8;
    const size_t smem = route_smem_bytes(TT, H);
    cudaError_t err = ensure_smem_optin(reinterpret_cast<const void*>(route_kernel<TT>), smem);
    if (err != cudaSuccess) return err;
    route_kernel<TT><<<(T + TT - 1) / TT, kRouteThreads, smem, st>>>(x, T, H, wg, E, bias, topk, ids, wts);
    return cudaGetLastError();
}

}  // namespace uocr
