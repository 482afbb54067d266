// The no-repeat-n-gram guard on the logits (ngram_block, kernels/ngram_block.mojo:1-151; its
// semantics are the reference's SlidingWindowNoRepeatNgramProcessor, per row b):
//
//   prefix = history[H - (n - 1) .. H)            (empty for n == 1)
//   for every start in [0, H - n + 1): if history[start .. start + n - 1) == prefix, the token
//   history[start + n - 1] is banned: out[b, token] = kNgramBlocked; every other logit is copied
//   bit for bit. n < 1, or H < n, bans nothing.
//
// The reference evaluates this per vocabulary entry (every logit scans the whole history). Here
// the scan runs once per CTA over the history, and the logits stream once: CTA (chunk, b) owns
// logits [chunk x kNgramChunk, +kNgramChunk) of row b. It loads the row's history into shared
// memory, marks in a shared bitmap every banned token that falls in its chunk (the candidate's
// last token is tested first, so nearly every start costs one comparison), then writes the chunk
// with the banned entries replaced. n is read from device memory, so a captured launch serves
// any n (n = 0 switches the guard off). Integer work; bound: HBM (logits read and written once),
// in practice launch latency: B = 8 rows of 129 280 logits (8.3 MB) take 4.0 us per launch in a
// CUDA graph with 2048-logit chunks (512 CTAs), 4.8 us with 8192-logit chunks (128 CTAs).
#include "common.cuh"
#include "kernels.h"

namespace uocr {
namespace {

constexpr int kNgramThreads = 256;
constexpr int kNgramChunk = 2048;                 // logits per CTA (a 256 B bitmap)
constexpr int kNgramMaxSmemHistory = 8192;        // history entries staged in shared memory
constexpr float kNgramBlocked = -3.0e38f;         // finite: argmax- and softmax-equivalent to -inf

// logits and out may be the same buffer (each element is read, then written, by one thread)
__global__ void __launch_bounds__(kNgramThreads) ngram_block_kernel(const float* logits, int V,
                                                                    const int32_t* __restrict__ history, int H,
                                                                    const int32_t* __restrict__ ngram, float* out,
                                                                    int vec) {
    __shared__ uint32_t banned[kNgramChunk / 32];
    __shared__ int32_t hist_s[kNgramMaxSmemHistory];
    const int b = blockIdx.y;
    const int v0 = blockIdx.x * kNgramChunk;
    const int v1 = min(V, v0 + kNgramChunk);
    const float* src = logits + (size_t)b * V;
    float* dst = out + (size_t)b * V;
    const int32_t* hrow = history + (size_t)b * H;
    const int n = __ldg(ngram);
    const bool active = n >= 1 && H >= n;

    for (int i = threadIdx.x; i < kNgramChunk / 32; i += kNgramThreads) banned[i] = 0u;
    if (active) {
        const bool staged = H <= kNgramMaxSmemHistory;
        if (staged)
            for (int i = threadIdx.x; i < H; i += kNgramThreads) hist_s[i] = hrow[i];
        __syncthreads();
        const int32_t* hs = staged ? hist_s : hrow;
        const int prefix_len = n - 1, starts = H - n + 1, prefix_at = H - prefix_len;
        for (int s = threadIdx.x; s < starts; s += kNgramThreads) {
            const int32_t tok = hs[s + prefix_len];
            if (tok < v0 || tok >= v1) continue;
            bool match = true;
            for (int j = 0; j < prefix_len; ++j) {
                if (hs[s + j] != hs[prefix_at + j]) {
                    match = false;
                    break;
                }
            }
            if (match) atomicOr(&banned[(tok - v0) >> 5], 1u << ((tok - v0) & 31));
        }
    }
    __syncthreads();

    if (vec) {  // 16-byte rows, chunk starts a multiple of 4
        for (int v = v0 + 4 * threadIdx.x; v + 3 < v1; v += 4 * kNgramThreads) {
            float4 x = *reinterpret_cast<const float4*>(src + v);
            const uint32_t bits = banned[(v - v0) >> 5] >> ((v - v0) & 31);
            if (bits & 1u) x.x = kNgramBlocked;
            if (bits & 2u) x.y = kNgramBlocked;
            if (bits & 4u) x.z = kNgramBlocked;
            if (bits & 8u) x.w = kNgramBlocked;
            *reinterpret_cast<float4*>(dst + v) = x;
        }
        const int tail = v0 + ((v1 - v0) & ~3);
        for (int v = tail + threadIdx.x; v < v1; v += kNgramThreads)
            dst[v] = (banned[(v - v0) >> 5] >> ((v - v0) & 31) & 1u) ? kNgramBlocked : src[v];
    } else {
        for (int v = v0 + threadIdx.x; v < v1; v += kNgramThreads)
            dst[v] = (banned[(v - v0) >> 5] >> ((v - v0) & 31) & 1u) ? kNgramBlocked : src[v];
    }
}

}  // namespace

cudaError_t launch_ngram_block(const float* logits, int B, int V, const int32_t* history, int H, const int32_t* ngram,
                               float* out, bool vec, cudaStream_t st) {
    if (B <= 0 || V <= 0) return cudaSuccess;
    const dim3 grid((V + kNgramChunk - 1) / kNgramChunk, B);
    ngram_block_kernel<<<grid, kNgramThreads, 0, st>>>(logits, V, history, H, ngram, out, vec ? 1 : 0);
    return cudaGetLastError();
}

}  // namespace uocr
