// uocr_moe_decode_noalloc: the decode-step MoE layer for callers that cannot allocate device
// memory.
//
// uocr_moe_decode needs a workspace buffer from its caller (routing ids and weights, the
// per-pair intermediate activations, the per-pair expert outputs, a status word). Some hosts
// have no way to provide one: a plugin interface that hands an operator only its input and
// output buffers, a runtime whose device memory is fully reserved up front, or code that
// must not call cudaMalloc at that point in its life (for example while another component
// owns the allocator). This entry point keeps that scratch in a fixed array inside the
// library instead, so the caller passes nothing but inputs and outputs.
//
// The array is a file-scope __device__ variable: every GPU that loads the library holds
// kNoAllocScratchBytes of it until the process exits. All calls on a device share it and it
// keeps the previous call's contents, so two calls whose work overlaps on the GPU (different
// streams without ordering between them) race on it. The control block at the start of the
// array is zero when the library is loaded (a __device__ array is zero-filled); a call's own
// counters return to a state the next call accepts, and every other scratch byte a call reads
// is written earlier in the same call. Its status word is sticky: a call whose device-side
// bounded wait gave up writes NaN over its output and records the failure there; until
// uocr_moe_decode_noalloc_status has read (and so cleared) it, later calls write NaN too.
//
// The first call on each device looks up the array's device address (cudaGetSymbolAddress,
// with that device current) and caches it; that first call should come before any stream
// capture on that device.
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/uocr_moe.h"
#include "common.cuh"
#include "kernels.h"

namespace {

// 1 MiB. The production layer (top_k 6, 2 shared experts, B = 8, inter 896, hidden 1280)
// needs 647 KiB: (6 + 2) * 8 pairs of (896 + 1280) fp32 values, the router logit partials, the
// tokens' MMA operand images, routing data and status.
constexpr size_t kNoAllocScratchBytes = size_t(1) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once per device.
cudaError_t scratch_address(void** out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (err != cudaSuccess) return err;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace

namespace uocr {
int set_error(int code, const char* msg);  // capi.cu: sets what uocr_last_error() reports
int read_clear_status(const void* workspace, cudaStream_t stream, uint32_t* code);  // capi.cu
}  // namespace uocr

extern "C" UOCR_API size_t uocr_moe_decode_noalloc_max_bytes(void) { return kNoAllocScratchBytes; }

extern "C" UOCR_API int uocr_moe_decode_noalloc(const uocr_moe_layer* L, const float* x, int64_t B,
                                                const float* bias, float* out, uocr_stream_t stream) {
    if (!L) return uocr::set_error(UOCR_EINVAL, "moe_decode_noalloc: null layer");
    if (B < 1 || B > 8) return uocr::set_error(UOCR_EINVAL, "moe_decode_noalloc: B must be 1..8");
    const size_t need = uocr_moe_decode_workspace_bytes(L, B);
    if (need == 0 || need > kNoAllocScratchBytes) {
        char buf[256];
        snprintf(buf, sizeof buf,
                 "moe_decode_noalloc: this layer at B=%lld needs %zu bytes of scratch, more than the built-in "
                 "%zu bytes; call uocr_moe_decode with a workspace instead",
                 (long long)B, need, kNoAllocScratchBytes);
        return uocr::set_error(UOCR_EINVAL, buf);
    }
    void* base = nullptr;
    const cudaError_t err = scratch_address(&base);
    if (err != cudaSuccess) {
        const std::string m = std::string("moe_decode_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(err);
        return uocr::set_error(UOCR_ECUDA, m.c_str());
    }
    // The regular entry point with the in-library array as its workspace (it validates the
    // layer and keeps the routing in the workspace).
    return uocr_moe_decode(L, x, B, bias, out, nullptr, nullptr, base, kNoAllocScratchBytes, stream);
}

extern "C" UOCR_API int uocr_moe_decode_noalloc_status(uocr_stream_t stream) {
    void* base = nullptr;
    const cudaError_t err = scratch_address(&base);
    if (err != cudaSuccess) {
        const std::string m = std::string("moe_decode_noalloc_status: cudaGetSymbolAddress: ") + cudaGetErrorString(err);
        return uocr::set_error(UOCR_ECUDA, m.c_str());
    }
    uint32_t code = 0;
    return uocr::read_clear_status(base, reinterpret_cast<cudaStream_t>(stream), &code);
}
