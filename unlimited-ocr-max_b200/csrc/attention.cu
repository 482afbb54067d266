// Paged decode attention (paged_decode_attention, decoder.py:425-437: store_k/v_cache_ragged,
// then flash_attention_ragged with the causal mask, over the page pool of kv_cache.py:1-40).
//
// Pool: kv[pages][2 (k, v)][layers][128 rows][heads][128] fp32; request b's logical row r is
// row r % 128 of page lut[b][r / 128]. One decode step for B requests: store k_new[b] / v_new[b]
// at row write_index[b] of layer `layer`, and attend q[b] (post-RoPE, [heads][128]) over rows
// [0, attend_len[b]) with scores q.k * scale and a softmax in fp32.
//
// Flash-decoding over the rows: S CTAs per request (S = min(sub-chunks, 148 / B)); CTA (s, b) walks
// the 4-row sub-chunks s, s + S, ... of request b, warp h head h (lane l dims 4l..4l+3). A
// sub-chunk's rows of every head are contiguous in one page, so two bulk copies (k and v, heads x
// 2 KB each) bring it into one of four shared-memory stages on that stage's mbarrier, the next
// three sub-chunks' copies in flight while the current one is computed; the warp keeps an online softmax
// (max m, sum l = sum exp(s - m), acc = sum exp(s - m) v) in registers across its sub-chunks and
// writes it to the workspace at the end. The row at write_index is taken from k_new / v_new once
// its sub-chunk has landed and stored into the pool by the CTA that owns it (no CTA reads the pool
// row being replaced). The CTA whose arrival completes request b (an acquire-release counter)
// combines the S partials in ascending order with a running max (deterministic), eight at a time:
// out = sum_s e^(m_s - M) acc_s / sum_s e^(m_s - M) l_s. Bound: HBM (every attended k and v row
// read once).
#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace uocr {
namespace {

constexpr int kAttnSub = 4;       // rows per sub-chunk (one pair of bulk copies)
constexpr int kAttnStages = 4;    // shared-memory stages (copies in flight while one is computed)
constexpr int kAttnDim = 128;     // head dim (lane x 4)
constexpr int kAttnPage = 128;    // rows per page
constexpr int kAttnCombine = 8;   // partials the combining CTA loads at once

struct AttnArgs {
    const float* q;        // [B][heads][128]
    const float* k_new;    // [B][heads][128]
    const float* v_new;
    float* kv;             // the pool
    const uint32_t* lut;   // [B][lut_cols]
    const uint32_t* write_index;  // [B]
    const uint32_t* attend_len;   // [B]
    float* out;            // [B][heads][128]
    float* partial;        // [B][S][heads][130]: m, l, acc[128]
    uint32_t* ctl;         // status word at [0], per-request counters at [kAttnCtlCounters + b]
    int heads, pages, layers, layer, lut_cols, S;
    float scale;
};

__device__ __forceinline__ size_t pool_index(const AttnArgs& a, uint32_t page, int kv, int slot, int h) {
    page = min(page, (uint32_t)(a.pages - 1));
    return ((((size_t)page * 2 + kv) * a.layers + a.layer) * kAttnPage + slot) * (size_t)a.heads * kAttnDim +
           (size_t)h * kAttnDim;
}

__global__ void paged_decode_attention_kernel(AttnArgs a) {
    extern __shared__ float4 attn_smem[];  // kAttnStages x (k [4][heads][32 float4], v the same)
    __shared__ uint64_t full[kAttnStages];
    __shared__ int last;
    const int s = blockIdx.x, b = blockIdx.y;
    const int h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // rows beyond the lookup table's reach, and page ids beyond the pool, are clamped (an entry
    // past the pool reads the pool's last page, the null page of the reference's layout)
    const int n_rows = (int)min(a.attend_len[b], (uint32_t)(a.lut_cols * kAttnPage));
    const int n_sub = (n_rows + kAttnSub - 1) / kAttnSub;
    const int n_cta = min(a.S, n_sub);  // CTAs of request b with work
    if (s >= n_cta) return;             // takes no part in request b's count
    const int my_subs = (n_sub - 1 - s) / a.S + 1;
    const int wi = (int)a.write_index[b];
    const size_t qo = ((size_t)b * a.heads + h) * kAttnDim + 4 * lane;
    const float4 q = *reinterpret_cast<const float4*>(a.q + qo);
    const uint32_t* lut = a.lut + (size_t)b * a.lut_cols;
    const size_t stage_f4 = (size_t)2 * kAttnSub * a.heads * 32;  // float4s per stage (k then v)

    auto issue = [&](int it) {  // thread 0: the copies of this CTA's it-th sub-chunk into its stage
        const int r0 = (s + it * a.S) * kAttnSub, nr = min(n_rows, r0 + kAttnSub) - r0;
        const uint32_t page = lut[r0 / kAttnPage];
        const uint32_t bytes = (uint32_t)nr * a.heads * kAttnDim * 4;
        float4* sk = attn_smem + (it % kAttnStages) * stage_f4;
        float4* sv = sk + (size_t)kAttnSub * a.heads * 32;
        mbar_arrive_expect_tx(&full[it % kAttnStages], 2 * bytes);
        bulk_g2s(sk, a.kv + pool_index(a, page, 0, r0 % kAttnPage, 0), bytes, &full[it % kAttnStages]);
        bulk_g2s(sv, a.kv + pool_index(a, page, 1, r0 % kAttnPage, 0), bytes, &full[it % kAttnStages]);
    };
    if (threadIdx.x == 0) {
        for (int st = 0; st < kAttnStages; ++st) mbar_init(&full[st], 1);
        fence_mbar_init();
        for (int it = 0; it < kAttnStages && it < my_subs; ++it) issue(it);
    }
    __syncthreads();

    float m = -INFINITY, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    bool landed = true;
    for (int it = 0; it < my_subs; ++it) {
        const int r0 = (s + it * a.S) * kAttnSub, nr = min(n_rows, r0 + kAttnSub) - r0;
        float4* sk = attn_smem + (it % kAttnStages) * stage_f4;
        float4* sv = sk + (size_t)kAttnSub * a.heads * 32;
        // a wait that gave up (status recorded) leaves the rest of this warp's rows out, but the
        // warp still takes part in the CTA's barriers below
        if (landed) landed = mbar_wait_warp(&full[it % kAttnStages], (it / kAttnStages) & 1, nullptr, a.ctl);
        const int rows = landed ? nr : 0;
        if (landed && wi >= r0 && wi < r0 + nr) {
            // the new row: into this warp's shared rows (head h), and into the pool
            const float4 kn = *reinterpret_cast<const float4*>(a.k_new + qo);
            const float4 vn = *reinterpret_cast<const float4*>(a.v_new + qo);
            sk[((size_t)(wi - r0) * a.heads + h) * 32 + lane] = kn;
            sv[((size_t)(wi - r0) * a.heads + h) * 32 + lane] = vn;
            const uint32_t page = lut[wi / kAttnPage];
            *reinterpret_cast<float4*>(a.kv + pool_index(a, page, 0, wi % kAttnPage, h) + 4 * lane) = kn;
            *reinterpret_cast<float4*>(a.kv + pool_index(a, page, 1, wi % kAttnPage, h) + 4 * lane) = vn;
        }
        __syncwarp();
        float sc[kAttnSub];
        float mn = m;
#pragma unroll
        for (int i = 0; i < kAttnSub; ++i) {
            sc[i] = -INFINITY;
            if (i < rows) {
                const float4 k = sk[((size_t)i * a.heads + h) * 32 + lane];
                float d = q.x * k.x + q.y * k.y + q.z * k.z + q.w * k.w;
#pragma unroll
                for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
                sc[i] = d * a.scale;
                mn = fmaxf(mn, sc[i]);
            }
        }
        if (rows > 0) {
            const float keep = expf(m - mn);  // 0 on the first sub-chunk (m = -inf)
            l *= keep;
            acc.x *= keep, acc.y *= keep, acc.z *= keep, acc.w *= keep;
#pragma unroll
            for (int i = 0; i < kAttnSub; ++i) {
                if (i < rows) {
                    const float4 v = sv[((size_t)i * a.heads + h) * 32 + lane];
                    const float p = expf(sc[i] - mn);
                    l += p;
                    acc.x += p * v.x, acc.y += p * v.y, acc.z += p * v.z, acc.w += p * v.w;
                }
            }
            m = mn;
        }
        __syncthreads();  // every warp is done with this stage
        if (threadIdx.x == 0 && it + kAttnStages < my_subs) issue(it + kAttnStages);
    }

    float* part = a.partial + (((size_t)b * a.S + s) * a.heads + h) * (kAttnDim + 2);
    if (lane == 0) {
        part[0] = m;
        part[1] = l;
    }
    *reinterpret_cast<float2*>(part + 2 + 4 * lane) = make_float2(acc.x, acc.y);
    *reinterpret_cast<float2*>(part + 4 + 4 * lane) = make_float2(acc.z, acc.w);

    // the last CTA of request b to arrive combines
    __syncthreads();
    if (threadIdx.x == 0) last = atom_acq_rel_gpu_add(&a.ctl[kAttnCtlCounters + b], 1u) == (uint32_t)(n_cta - 1);
    __syncthreads();
    if (!last) return;
    const float* pb = a.partial + (size_t)b * a.S * a.heads * (kAttnDim + 2);
    float M = -INFINITY, L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c0 = 0; c0 < n_cta; c0 += kAttnCombine) {
        float mc[kAttnCombine], lc[kAttnCombine];
        float2 x0[kAttnCombine], x1[kAttnCombine];
#pragma unroll
        for (int j = 0; j < kAttnCombine; ++j) {
            if (c0 + j < n_cta) {
                const float* pc = pb + ((size_t)(c0 + j) * a.heads + h) * (kAttnDim + 2);
                mc[j] = __ldcg(pc);
                lc[j] = __ldcg(pc + 1);
                x0[j] = __ldcg(reinterpret_cast<const float2*>(pc + 2 + 4 * lane));
                x1[j] = __ldcg(reinterpret_cast<const float2*>(pc + 4 + 4 * lane));
            }
        }
#pragma unroll
        for (int j = 0; j < kAttnCombine; ++j) {
            if (c0 + j < n_cta && mc[j] > -INFINITY) {
                const float Mn = fmaxf(M, mc[j]);
                const float keep = expf(M - Mn), w = expf(mc[j] - Mn);
                L = L * keep + w * lc[j];
                o.x = o.x * keep + w * x0[j].x, o.y = o.y * keep + w * x0[j].y;
                o.z = o.z * keep + w * x1[j].x, o.w = o.w * keep + w * x1[j].y;
                M = Mn;
            }
        }
    }
    const float inv = 1.f / L;
    *reinterpret_cast<float4*>(a.out + qo) = make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    __syncthreads();
    if (threadIdx.x == 0) a.ctl[kAttnCtlCounters + b] = 0;
}

}  // namespace

int paged_attention_ctas(int B, int lut_cols, int sms) {
    return std::max(1, std::min(lut_cols * kAttnPage / kAttnSub, sms / std::max(B, 1)));
}

cudaError_t launch_paged_decode_attention(const float* q, const float* k_new, const float* v_new, float* kv,
                                          int pages, int layers, int layer, const uint32_t* lut, int lut_cols,
                                          const uint32_t* write_index, const uint32_t* attend_len, float* out, int B,
                                          int heads, float scale, uint32_t* ctl, float* partial, int S,
                                          cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    AttnArgs a{q, k_new, v_new, kv, lut, write_index, attend_len, out, partial, ctl,
               heads, pages, layers, layer, lut_cols, S, scale};
    const size_t smem = (size_t)kAttnStages * 2 * kAttnSub * heads * kAttnDim * 4;
    cudaError_t err = ensure_smem_optin(reinterpret_cast<const void*>(paged_decode_attention_kernel), smem);
    if (err != cudaSuccess) return err;
    paged_decode_attention_kernel<<<dim3(S, B), 32 * heads, smem, st>>>(a);
    return cudaGetLastError();
}

}  // namespace uocr
