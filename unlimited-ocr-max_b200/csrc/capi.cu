// The C ABI of libuocr_moe.so (include/uocr_moe.h): host-side argument checks with the
// reference ops' error messages, then kernel launches on the caller's stream.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>

#include <cuda.h>
#include <cudaTypedefs.h>

#include "../../include/uocr_moe.h"
#include "common.cuh"
#include "kernels.h"
#include "layout.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int ok() {
    g_last_error.clear();
    return UOCR_OK;
}

int cuda_status(cudaError_t err, const char* what) {
    if (err != cudaSuccess) return fail(UOCR_ECUDA, "%s: %s", what, cudaGetErrorString(err));
    return ok();
}

cudaStream_t S(uocr_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

bool a16(const void* p) { return uocr::aligned16(p); }

}  // namespace

namespace uocr {

unsigned long long* g_decode_trace = nullptr;
size_t g_decode_trace_bytes = 0;
int g_decode_wait_extra = 0;

// Read a workspace's status word after `stream` finished; if it is set, clear it together with the
// control words a failed call may have left behind (decode: DecodeCtl; prefill and exchange
// workspaces: a status region of the same size). Returns the code read.
int read_clear_status(const void* workspace, cudaStream_t stream, uint32_t* code) {
    cudaError_t err = cudaStreamSynchronize(stream);
    if (err != cudaSuccess) return fail(UOCR_ECUDA, "device_status: synchronize: %s", cudaGetErrorString(err));
    *code = 0;
    err = cudaMemcpy(code, workspace, sizeof *code, cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) return fail(UOCR_ECUDA, "device_status: read: %s", cudaGetErrorString(err));
    if (*code) {
        err = cudaMemset(const_cast<void*>(workspace), 0, kCtlClearBytes);
        if (err != cudaSuccess) return fail(UOCR_ECUDA, "device_status: clear: %s", cudaGetErrorString(err));
        return fail(UOCR_EDEVICE, "device_status: a device-side check failed (code %u: %s); cleared", *code,
                    *code == 1 ? "a bounded wait gave up"
                    : *code == 2 ? "shared memory misaligned"
                    : *code == 3 ? "an exchanged row count above the slot capacity"
                                 : "unknown");
    }
    return ok();
}

int set_error(int code, const char* msg) {
    g_last_error = msg;
    return code;
}

cudaError_t ensure_smem_optin(const void* kernel, size_t bytes) {
    static std::mutex mu;
    static std::unordered_map<const void*, size_t> granted;  // per device would matter only across GPUs
    std::lock_guard<std::mutex> lock(mu);
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    const void* key = reinterpret_cast<const char*>(kernel) + dev;  // distinct per (kernel, device)
    auto it = granted.find(key);
    if (it != granted.end() && it->second >= bytes) return cudaSuccess;
    if (bytes <= 48 * 1024 && it == granted.end()) {
        granted[key] = 48 * 1024;
        if (bytes <= 48 * 1024) return cudaSuccess;
    }
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (err == cudaSuccess) granted[key] = bytes;
    return err;
}

}  // namespace uocr

extern "C" {

const char* uocr_last_error(void) { return g_last_error.c_str(); }

int uocr_abi_version(void) { return 6; }

// ---------------------------------------------------------------------------------------
// reference op shims
// ---------------------------------------------------------------------------------------

int uocr_moe_bf16_qmv(float* out, int64_t out_rows, int64_t out_cols, const float* x, int64_t x_rows, int64_t x_cols,
                      const int32_t* expert_ids, int64_t ids_len, const uint16_t* w, int64_t w_e, int64_t w_n,
                      int64_t w_k, uocr_stream_t stream) {
    // kernels/moe_bf16.mojo:276-285
    if (x_rows != out_rows) return fail(UOCR_EINVAL, "moe_bf16_qmv: x and output disagree on k");
    if (ids_len != out_rows) return fail(UOCR_EINVAL, "moe_bf16_qmv: expert_ids and output disagree on k");
    if (w_n != out_cols) return fail(UOCR_EINVAL, "moe_bf16_qmv: w and output disagree on N");
    if (w_k != x_cols) return fail(UOCR_EINVAL, "moe_bf16_qmv: w and x disagree on K");
    if (w_e < 1) return fail(UOCR_EINVAL, "moe_bf16_qmv: the expert stack is empty");
    if (out_rows == 0 || out_cols == 0) return ok();
    if (w_k > INT32_MAX || w_n > INT32_MAX || w_e > INT32_MAX)
        return fail(UOCR_EUNSUPPORTED, "moe_bf16_qmv: dims beyond int32");
    const bool vec = (w_k % 8 == 0) && a16(w) && a16(x);
    for (int64_t r0 = 0; r0 < out_rows; r0 += 65535) {
        const int rows = (int)std::min<int64_t>(65535, out_rows - r0);
        uocr::launch_bf16_qmv(out + r0 * out_cols, x + r0 * x_cols, expert_ids + r0, w, rows, (int)w_e, (int)w_n,
                              (int)w_k, vec, S(stream));
    }
    return cuda_status(cudaGetLastError(), "moe_bf16_qmv: launch");
}

int uocr_moe_int8_qmv(float* out, int64_t out_rows, int64_t out_cols, const float* x, int64_t x_rows, int64_t x_cols,
                      const int32_t* expert_ids, int64_t ids_len, const int8_t* w, int64_t w_e, int64_t w_n,
                      int64_t w_k, const float* scales, int64_t s_e, int64_t s_n, int64_t s_g,
                      uocr_stream_t stream) {
    // kernels/moe_int8.mojo:196-212
    if (x_rows != out_rows) return fail(UOCR_EINVAL, "moe_int8_qmv: x and output disagree on k");
    if (ids_len != out_rows) return fail(UOCR_EINVAL, "moe_int8_qmv: expert_ids and output disagree on k");
    if (w_n != out_cols) return fail(UOCR_EINVAL, "moe_int8_qmv: w and output disagree on N");
    if (w_k != x_cols) return fail(UOCR_EINVAL, "moe_int8_qmv: w and x disagree on K");
    if (w_e < 1) return fail(UOCR_EINVAL, "moe_int8_qmv: the expert stack is empty");
    if (s_e != w_e) return fail(UOCR_EINVAL, "moe_int8_qmv: scales and w disagree on E");
    if (s_n != w_n) return fail(UOCR_EINVAL, "moe_int8_qmv: scales and w disagree on N");
    if (s_g < 1 || w_k % s_g != 0) return fail(UOCR_EINVAL, "moe_int8_qmv: K must be a multiple of the group count");
    if (out_rows == 0 || out_cols == 0) return ok();
    if (w_k > INT32_MAX || w_n > INT32_MAX || w_e > INT32_MAX || out_rows > INT32_MAX)
        return fail(UOCR_EUNSUPPORTED, "moe_int8_qmv: dims beyond int32");
    const int64_t gsize = w_k / s_g;
    const bool vec = (gsize % 16 == 0) && (w_k % 16 == 0) && a16(w);
    uocr::launch_int8_qmv(out, x, expert_ids, w, scales, (int)out_rows, (int)w_e, (int)w_n, (int)w_k, (int)s_g, vec,
                          S(stream));
    return cuda_status(cudaGetLastError(), "moe_int8_qmv: launch");
}

int uocr_int8_dequant_expert(uint16_t* out, int64_t out_n, int64_t out_k, const int8_t* w, int64_t w_e, int64_t w_n,
                             int64_t w_k, const float* scales, int64_t s_e, int64_t s_n, int64_t s_g,
                             const int32_t* expert_idx, int64_t idx_len, uocr_stream_t stream) {
    // kernels/moe_int8.mojo:274-297
    if (w_n != out_n) return fail(UOCR_EINVAL, "int8_dequant_expert: w and output disagree on N");
    if (w_k != out_k) return fail(UOCR_EINVAL, "int8_dequant_expert: w and output disagree on K");
    if (w_e < 1) return fail(UOCR_EINVAL, "int8_dequant_expert: the expert stack is empty");
    if (s_e != w_e) return fail(UOCR_EINVAL, "int8_dequant_expert: scales and w disagree on E");
    if (s_n != w_n) return fail(UOCR_EINVAL, "int8_dequant_expert: scales and w disagree on N");
    if (idx_len != 1) return fail(UOCR_EINVAL, "int8_dequant_expert: `expert_idx` must be a single int32");
    if (s_g < 1 || w_k % s_g != 0)
        return fail(UOCR_EINVAL, "int8_dequant_expert: K must be a multiple of the group count");
    if (out_n == 0 || out_k == 0) return ok();
    if (w_k > INT32_MAX || w_n > INT32_MAX || w_e > INT32_MAX)
        return fail(UOCR_EUNSUPPORTED, "int8_dequant_expert: dims beyond int32");
    uocr::launch_int8_dequant(out, w, scales, expert_idx, (int)w_e, (int)w_n, (int)w_k, (int)s_g, S(stream));
    return cuda_status(cudaGetLastError(), "int8_dequant_expert: launch");
}

int uocr_dense_bf16_qmv(float* out, int64_t out_rows, int64_t out_cols, const float* x, int64_t x_rows,
                        int64_t x_cols, const uint16_t* w, int64_t w_kb, int64_t w_n, int64_t w_blk, int tile,
                        uocr_stream_t stream) {
    // kernels/dense_bf16.mojo:130-145, decoder.py:174-178
    if (tile < 1) return fail(UOCR_EINVAL, "dense_bf16_qmv: tile must be >= 1");
    if (out_rows != x_rows) return fail(UOCR_EINVAL, "dense_bf16_qmv: x and output disagree on M");
    if (w_n != out_cols) return fail(UOCR_EINVAL, "dense_bf16_qmv: w and output disagree on N");
    if (w_blk != 16) return fail(UOCR_EINVAL, "dense_bf16_qmv: w is not K-blocked by KBLOCK");
    if (w_kb * 16 != x_cols) return fail(UOCR_EINVAL, "dense_bf16_qmv: w and x disagree on K");
    if (out_rows == 0 || out_cols == 0) return ok();
    if (x_cols > INT32_MAX || w_n > INT32_MAX) return fail(UOCR_EUNSUPPORTED, "dense_bf16_qmv: dims beyond int32");
    const bool vec = a16(w) && a16(x);
    for (int64_t r0 = 0; r0 < out_rows; r0 += 65535) {
        const int rows = (int)std::min<int64_t>(65535, out_rows - r0);
        uocr::launch_dense_bf16_qmv(out + r0 * out_cols, x + r0 * x_cols, w, rows, (int)w_n, (int)x_cols, vec,
                                    S(stream));
    }
    return cuda_status(cudaGetLastError(), "dense_bf16_qmv: launch");
}

int uocr_quantize_int8_g128(const void* w, int w_dtype, int64_t rows, int64_t K, int8_t* q, float* scales,
                            int* nonfinite, uocr_stream_t stream) {
    // tools/quantize_int8.py:298-329 (quantize_per_group) and its refusals
    if (w_dtype != UOCR_DTYPE_F32 && w_dtype != UOCR_DTYPE_BF16)
        return fail(UOCR_EINVAL, "quantize_per_group: the weight must be fp32 or bf16 (dtype code %d)", w_dtype);
    if (rows < 0 || K < 0) return fail(UOCR_EINVAL, "quantize_per_group: negative shape [%lld, %lld]",
                                       (long long)rows, (long long)K);
    if (K % 128) return fail(UOCR_EINVAL, "K=%lld is not divisible by the group size 128", (long long)K);
    if (rows == 0 || K == 0) return ok();
    if (!w || !q || !scales || !nonfinite) return fail(UOCR_EINVAL, "quantize_per_group: null pointer");
    if (rows > INT64_MAX / K) return fail(UOCR_EUNSUPPORTED, "quantize_per_group: size overflows int64");
    const bool bf16 = w_dtype == UOCR_DTYPE_BF16;
    const bool vec = (reinterpret_cast<uintptr_t>(w) & 15) == 0 && (reinterpret_cast<uintptr_t>(q) & 7) == 0;
    const long long groups = static_cast<long long>(rows) * (K / 128);
    return cuda_status(uocr::launch_quantize_g128(w, bf16, groups, q, scales, nonfinite, vec, S(stream)),
                       "quantize_per_group: launch");
}

// ---------------------------------------------------------------------------------------
// dense projections of the decode step (tensor-core weight streaming)
// ---------------------------------------------------------------------------------------
static bool dense_dims_ok(int64_t N, int64_t K) {
    return N >= 1 && K >= 16 && K % 16 == 0 && N <= (int64_t)INT32_MAX - 128 && K <= (int64_t)INT32_MAX - 128;
}
static int current_sms() {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

size_t uocr_dense_packed_bytes(int64_t N, int64_t K) {
    if (!dense_dims_ok(N, K)) return 0;
    const uocr::DensePlan p = uocr::dense_plan(N, K, 1);
    return (size_t)p.NB * p.IPR * 2 * uocr::kAtomBytes;
}

int uocr_dense_pack(const uint16_t* w, int kblocked, int64_t N, int64_t K, void* packed, uocr_stream_t stream) {
    if (!dense_dims_ok(N, K))
        return fail(UOCR_EINVAL, "dense_pack: need N >= 1 and K a positive multiple of 16 (KBLOCK), got [%lld, %lld]",
                    (long long)N, (long long)K);
    if (!w || !packed) return fail(UOCR_EINVAL, "dense_pack: null pointer");
    if (!a16(w) || !a16(packed)) return fail(UOCR_EINVAL, "dense_pack: w and packed must be 16-byte aligned");
    return cuda_status(uocr::launch_dense_pack(w, kblocked != 0, (int)N, (int)K, static_cast<unsigned char*>(packed),
                                               S(stream)),
                       "dense_pack: launch");
}

size_t uocr_dense_stream_workspace_bytes(int64_t N, int64_t K) {
    if (!dense_dims_ok(N, K)) return 0;
    const uocr::DensePlan p = uocr::dense_plan(N, K, current_sms());
    return uocr::kCtlClearBytes + (p.KC > 1 ? (size_t)p.KC * 8 * p.NB * 128 * sizeof(float) : 0);
}

int uocr_dense_stream(const void* packed, int64_t N, int64_t K, const float* x, int64_t M, float* out,
                      void* workspace, size_t workspace_bytes, uocr_stream_t stream) {
    if (!dense_dims_ok(N, K))
        return fail(UOCR_EINVAL, "dense_stream: need N >= 1 and K a positive multiple of 16 (KBLOCK), got [%lld, %lld]",
                    (long long)N, (long long)K);
    if (M < 0) return fail(UOCR_EINVAL, "dense_stream: negative row count");
    if (M == 0) return ok();
    if (!packed || !x || !out || !workspace) return fail(UOCR_EINVAL, "dense_stream: null pointer");
    if (!a16(packed) || !a16(workspace)) return fail(UOCR_EINVAL, "dense_stream: packed and workspace must be 16-byte aligned");
    const uocr::DensePlan p = uocr::dense_plan(N, K, current_sms());
    const size_t need = uocr_dense_stream_workspace_bytes(N, K);
    if (workspace_bytes < need)
        return fail(UOCR_EINVAL, "dense_stream: workspace of %zu bytes, need %zu", workspace_bytes, need);
    if (p.KC > 1 && p.NB + uocr::kDenseCtlCounters > (int)(uocr::kCtlClearBytes / 4))
        return fail(UOCR_EUNSUPPORTED, "dense_stream: %d row blocks with split K exceed the control block", p.NB);
    auto* ctl = static_cast<uint32_t*>(workspace);
    float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + uocr::kCtlClearBytes);
    for (int64_t m0 = 0; m0 < M; m0 += 8) {
        const int rows = (int)std::min<int64_t>(8, M - m0);
        cudaError_t err = uocr::launch_dense_stream(static_cast<const unsigned char*>(packed), (int)N, (int)K,
                                                    x + m0 * K, rows, out + m0 * N, ctl, partial, p, S(stream));
        if (err != cudaSuccess) return cuda_status(err, "dense_stream: launch");
    }
    return ok();
}

size_t uocr_paged_attention_workspace_bytes(int64_t B, int64_t heads, int64_t lut_cols) {
    if (B < 1 || heads < 1 || heads > 12 || lut_cols < 1 || B > 2000 || lut_cols > (1 << 20)) return 0;
    return uocr::kCtlClearBytes + (size_t)B * lut_cols * 32 * heads * 130 * sizeof(float);
}

int uocr_paged_decode_attention(const float* q, const float* k_new, const float* v_new, int64_t B, int64_t heads,
                                int64_t head_dim, float* kv_pool, int64_t pages, int64_t layers, int64_t layer,
                                const uint32_t* lut, int64_t lut_cols, const uint32_t* write_index,
                                const uint32_t* attend_len, float scale, float* out, void* workspace,
                                size_t workspace_bytes, uocr_stream_t stream) {
    // paged_decode_attention, decoder.py:425-437 (store_k/v_cache_ragged + flash_attention_ragged)
    if (head_dim != 128) return fail(UOCR_EUNSUPPORTED, "paged_decode_attention: head_dim %lld (this build: 128)",
                                     (long long)head_dim);
    if (B < 0 || heads < 1) return fail(UOCR_EINVAL, "paged_decode_attention: bad B or heads");
    if (heads > 12) return fail(UOCR_EUNSUPPORTED, "paged_decode_attention: %lld heads (this build: <= 12)", (long long)heads);
    if (pages < 1 || layers < 1 || layer < 0 || layer >= layers || lut_cols < 1)
        return fail(UOCR_EINVAL, "paged_decode_attention: bad pool (pages %lld, layers %lld, layer %lld, lut_cols %lld)",
                    (long long)pages, (long long)layers, (long long)layer, (long long)lut_cols);
    if (B == 0) return ok();
    if (!q || !k_new || !v_new || !kv_pool || !lut || !write_index || !attend_len || !out || !workspace)
        return fail(UOCR_EINVAL, "paged_decode_attention: null pointer");
    if (!a16(q) || !a16(k_new) || !a16(v_new) || !a16(kv_pool) || !a16(out) || !a16(workspace))
        return fail(UOCR_EINVAL, "paged_decode_attention: q, k_new, v_new, the pool, out and the workspace must be "
                                 "16-byte aligned");
    const size_t need = uocr_paged_attention_workspace_bytes(B, heads, lut_cols);
    if (need == 0 || workspace_bytes < need)
        return fail(UOCR_EINVAL, "paged_decode_attention: workspace of %zu bytes, need %zu", workspace_bytes, need);
    auto* ctl = static_cast<uint32_t*>(workspace);
    float* partial = reinterpret_cast<float*>(static_cast<char*>(workspace) + uocr::kCtlClearBytes);
    return cuda_status(uocr::launch_paged_decode_attention(q, k_new, v_new, kv_pool, (int)pages, (int)layers, (int)layer,
                                                           lut, (int)lut_cols, write_index, attend_len, out, (int)B,
                                                           (int)heads, scale, ctl, partial,
                                                           uocr::paged_attention_ctas((int)B, (int)lut_cols,
                                                                                      current_sms()),
                                                           S(stream)),
                       "paged_decode_attention: launch");
}

int uocr_rope_qkv(const float* qkv, int64_t B, int64_t heads, int64_t head_dim, const float* cos, const float* sin,
                  float* q, float* k, float* v, uocr_stream_t stream) {
    // Attention._rope / Attention.decode, decoder.py:459-462, 478-493
    if (B < 0 || heads < 1 || head_dim < 2 || head_dim % 2 || (long long)B * heads * head_dim * 3 > INT32_MAX)
        return fail(UOCR_EINVAL, "rope_qkv: bad shape (B %lld, heads %lld, head_dim %lld)", (long long)B,
                    (long long)heads, (long long)head_dim);
    if (B == 0) return ok();
    if (!qkv || !cos || !sin || !q || !k || !v) return fail(UOCR_EINVAL, "rope_qkv: null pointer");
    return cuda_status(uocr::launch_rope_qkv(qkv, (int)B, (int)heads, (int)head_dim, cos, sin, q, k, v, S(stream)),
                       "rope_qkv: launch");
}

int uocr_embed_rows(const uint16_t* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t B, float* out,
                    uocr_stream_t stream) {
    // EmbeddingTable, decoder.py:241-249
    if (vocab < 1 || hidden < 1 || B < 0 || vocab > INT32_MAX || (long long)B * hidden > INT32_MAX)
        return fail(UOCR_EINVAL, "embed_rows: bad shape (vocab %lld, hidden %lld, B %lld)", (long long)vocab,
                    (long long)hidden, (long long)B);
    if (B == 0) return ok();
    if (!table || !ids || !out) return fail(UOCR_EINVAL, "embed_rows: null pointer");
    return cuda_status(uocr::launch_embed_rows(table, (int)vocab, (int)hidden, ids, (int)B, out, S(stream)),
                       "embed_rows: launch");
}

int uocr_silu_mul(const float* gate_up, int64_t B, int64_t inter, float* out, uocr_stream_t stream) {
    // GatedMlp.decode_rows, decoder.py:276-278
    if (B < 0 || inter < 1 || (long long)B * inter * 2 > INT32_MAX)
        return fail(UOCR_EINVAL, "silu_mul: bad shape (B %lld, inter %lld)", (long long)B, (long long)inter);
    if (B == 0) return ok();
    if (!gate_up || !out) return fail(UOCR_EINVAL, "silu_mul: null pointer");
    return cuda_status(uocr::launch_silu_mul(gate_up, (int)B, (int)inter, out, S(stream)), "silu_mul: launch");
}

int uocr_ngram_block(const float* logits, int64_t B, int64_t V, const int32_t* history, int64_t H,
                     const int32_t* ngram, float* out, uocr_stream_t stream) {
    // kernels/ngram_block.mojo:80-105 (its shape checks), semantics :1-33
    if (B < 0 || V < 0 || B > 65535 || V > INT32_MAX || H > INT32_MAX)
        return fail(UOCR_EINVAL, "ngram_block: bad shape (B %lld, V %lld, H %lld)", (long long)B, (long long)V,
                    (long long)H);
    if (H < 1) return fail(UOCR_EINVAL, "ngram_block: history is empty");
    if (!ngram) return fail(UOCR_EINVAL, "ngram_block: `ngram` must be a single int32");
    if (B == 0 || V == 0) return ok();
    if (!logits || !history || !out) return fail(UOCR_EINVAL, "ngram_block: null pointer");
    const bool vec = a16(logits) && a16(out) && V % 4 == 0;
    return cuda_status(uocr::launch_ngram_block(logits, (int)B, (int)V, history, (int)H, ngram, out, vec, S(stream)),
                       "ngram_block: launch");
}

int uocr_residual_rmsnorm(float* h, const float* add, const float* gamma, int64_t B, int64_t H, float eps,
                          float* y, uocr_stream_t stream) {
    // decoder.py:702-709 (the residual add) and RmsNorm, decoder.py:252-261
    if (B < 0 || H < 1 || H > INT32_MAX || B > INT32_MAX)
        return fail(UOCR_EINVAL, "residual_rmsnorm: bad shape [%lld, %lld]", (long long)B, (long long)H);
    if (!(eps >= 0.f)) return fail(UOCR_EINVAL, "residual_rmsnorm: eps must be >= 0");
    if (B == 0) return ok();
    if (!h || (y && !gamma)) return fail(UOCR_EINVAL, "residual_rmsnorm: null pointer");
    return cuda_status(uocr::launch_residual_rmsnorm(h, add, gamma, (int)B, (int)H, eps, y, S(stream)),
                       "residual_rmsnorm: launch");
}

// ---------------------------------------------------------------------------------------
// packing
// ---------------------------------------------------------------------------------------

static int check_pack(const char* who, int64_t E, int64_t G, int int8) {
    if (E < 1) return fail(UOCR_EINVAL, "%s: empty stack", who);
    if (int8 && (G != 128)) return fail(UOCR_EUNSUPPORTED, "%s: int8 group size %lld (this build packs G = 128)", who, (long long)G);
    return ok();
}
static bool a16p(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// gate|up: I a multiple of 64 (row blocks of 64 pairs); H a multiple of 256 (int8) / 128 (bf16)
static bool w13_dims_ok(int64_t I, int64_t H, int int8) {
    return I >= 64 && I % 64 == 0 && H >= 128 && H % (int8 ? 256 : 128) == 0 && I <= INT32_MAX && H <= INT32_MAX;
}
// down: H a multiple of 128 (row blocks), I a multiple of 128
static bool w2_dims_ok(int64_t H, int64_t I) {
    return H >= 128 && H % 128 == 0 && I >= 128 && I % 128 == 0 && I <= INT32_MAX && H <= INT32_MAX;
}

size_t uocr_moe_w13_bytes(int64_t E, int64_t I, int64_t H, int64_t group, int int8) {
    if (E < 1 || !w13_dims_ok(I, H, int8) || (int8 && group != 128)) return 0;
    return (size_t)E * uocr::w13_expert_bytes((int)I, (int)H, int8 != 0);
}

size_t uocr_moe_w2_bytes(int64_t E, int64_t H, int64_t I, int64_t group, int int8) {
    if (E < 1 || !w2_dims_ok(H, I) || (int8 && group != 128)) return 0;
    return (size_t)E * uocr::w2_expert_bytes((int)H, (int)I, int8 != 0);
}

int uocr_moe_pack_w13(const void* gate, const void* up, const float* gate_scales, const float* up_scales, int64_t E,
                      int64_t I, int64_t H, int64_t group, int int8, void* w13_out, uocr_stream_t stream) {
    int rc = check_pack("pack_w13", E, group, int8);
    if (rc) return rc;
    if (!w13_dims_ok(I, H, int8))
        return fail(UOCR_EINVAL, "pack_w13: I=%lld must be a multiple of 64 and H=%lld of %d", (long long)I,
                    (long long)H, int8 ? 256 : 128);
    if (!gate || !up || !w13_out || (int8 && (!gate_scales || !up_scales)))
        return fail(UOCR_EINVAL, "pack_w13: null pointer");
    if (!a16p(gate) || !a16p(up) || !a16p(w13_out) || ((reinterpret_cast<uintptr_t>(gate_scales) |
                                                        reinterpret_cast<uintptr_t>(up_scales)) & 3))
        return fail(UOCR_EINVAL, "pack_w13: weights and output must be 16-byte aligned, scales 4-byte aligned");
    return cuda_status(uocr::launch_pack_w13(gate, up, gate_scales, up_scales, (int)E, (int)I, (int)H, int8 != 0,
                                             (long)(I * H), (long)H, w13_out, S(stream)),
                       "pack_w13: launch");
}

int uocr_moe_pack_w2(const void* down, const float* down_scales, int64_t E, int64_t H, int64_t I, int64_t group,
                     int int8, void* w2_out, uocr_stream_t stream) {
    int rc = check_pack("pack_w2", E, group, int8);
    if (rc) return rc;
    if (!w2_dims_ok(H, I))
        return fail(UOCR_EINVAL, "pack_w2: H=%lld and I=%lld must be multiples of 128", (long long)H, (long long)I);
    if (!down || !w2_out || (int8 && !down_scales)) return fail(UOCR_EINVAL, "pack_w2: null pointer");
    if (!a16p(down) || !a16p(w2_out) || (reinterpret_cast<uintptr_t>(down_scales) & 3))
        return fail(UOCR_EINVAL, "pack_w2: weights and output must be 16-byte aligned, scales 4-byte aligned");
    return cuda_status(uocr::launch_pack_w2(down, down_scales, (int)E, (int)H, (int)I, int8 != 0, (long)(H * I),
                                            (long)I, w2_out, S(stream)),
                       "pack_w2: launch");
}

int uocr_moe_pack_shared(const uint16_t* gate, const uint16_t* up, const uint16_t* down, int64_t S_, int64_t I,
                         int64_t H, uint16_t* w13_out, uint16_t* w2_out, uocr_stream_t stream) {
    if (S_ < 1 || I < 1 || H < 1) return fail(UOCR_EINVAL, "pack_shared: empty");
    if (!w13_dims_ok(I, H, 0) || !w2_dims_ok(H, I))
        return fail(UOCR_EINVAL, "pack_shared: I=%lld and H=%lld must be multiples of 128", (long long)I, (long long)H);
    if (!gate || !up || !down || !w13_out || !w2_out) return fail(UOCR_EINVAL, "pack_shared: null pointer");
    if (!a16p(gate) || !a16p(up) || !a16p(down) || !a16p(w13_out) || !a16p(w2_out))
        return fail(UOCR_EINVAL, "pack_shared: pointers must be 16-byte aligned");
    return cuda_status(uocr::launch_pack_shared(gate, up, down, S_, I, H, w13_out, w2_out, S(stream)),
                       "pack_shared: launch");
}

// ---------------------------------------------------------------------------------------
// router
// ---------------------------------------------------------------------------------------

static int check_router(int64_t T, int64_t H, int64_t E, int64_t top_k, const float* x, const uint16_t* router,
                        const float* bias, const void* ids, const void* wts) {
    if (T < 0) return fail(UOCR_EINVAL, "route: negative token count");
    if (H < 64 || H % 64) return fail(UOCR_EINVAL, "route: hidden=%lld must be a positive multiple of 64", (long long)H);
    if (E < 1 || E > 64) return fail(UOCR_EUNSUPPORTED, "route: %lld experts; this build routes 1..64", (long long)E);
    if (top_k < 1 || top_k > E) return fail(UOCR_EINVAL, "route: top_k=%lld outside [1, E]", (long long)top_k);
    if (T > 0 && (!x || !router || !ids || !wts)) return fail(UOCR_EINVAL, "route: null pointer");
    if (!a16(x) || !a16(router)) return fail(UOCR_EINVAL, "route: x and router must be 16-byte aligned");
    (void)bias;
    return ok();
}

int uocr_moe_route(const float* x, int64_t T, int64_t H, const uint16_t* router, int64_t E, const float* bias,
                   int64_t top_k, int32_t* ids_out, float* wts_out, uocr_stream_t stream) {
    int rc = check_router(T, H, E, top_k, x, router, bias, ids_out, wts_out);
    if (rc) return rc;
    if (T == 0) return ok();
    if (T > INT32_MAX / 8) return fail(UOCR_EUNSUPPORTED, "route: too many tokens");
    return cuda_status(uocr::launch_route(x, (int)T, (int)H, router, (int)E, bias, (int)top_k, ids_out, wts_out,
                                          S(stream)),
                       "route: launch");
}

// ---------------------------------------------------------------------------------------
// decode step
// ---------------------------------------------------------------------------------------

namespace {

struct DecodeLayout {
    size_t ctl, logits, xd, xb, xsig, ids, wts, h, y, himg, gsig, total;
};

DecodeLayout decode_layout(const uocr_moe_layer* L, int64_t B) {
    DecodeLayout d{};
    const size_t pairs = (size_t)(L->top_k + L->n_shared) * (size_t)B;
    size_t off = 0;
    d.ctl = off; off += align256(sizeof(uocr::DecodeCtl));
    d.logits = off; off += align256(sizeof(float) * 8 * 64 * 8);
    d.xd = off; off += align256((size_t)L->hidden * 32);
    d.xb = off; off += align256((size_t)L->hidden * 32);
    d.xsig = off; off += align256(sizeof(float) * 8 * (size_t)(L->hidden / 128));
    d.ids = off; off += align256(sizeof(int32_t) * (size_t)B * L->top_k);
    d.wts = off; off += align256(sizeof(float) * (size_t)B * L->top_k);
    d.h = off; off += align256(sizeof(float) * pairs * (size_t)L->inter);
    d.y = off; off += align256(sizeof(float) * pairs * (size_t)L->hidden);
    d.himg = off; off += align256(sizeof(float) * pairs * (size_t)L->inter);
    d.gsig = off; off += align256(sizeof(float) * pairs * (size_t)uocr::decode_sig_stride(L->inter));
    d.total = off;
    return d;
}

int check_layer(const uocr_moe_layer* L, const char* who) {
    if (!L) return fail(UOCR_EINVAL, "%s: null layer", who);
    if (L->hidden < 128 || L->hidden % 128)
        return fail(UOCR_EINVAL, "%s: hidden=%d must be a positive multiple of 128", who, L->hidden);
    if (L->inter < 128 || L->inter % 128)
        return fail(UOCR_EINVAL, "%s: inter=%d must be a positive multiple of 128", who, L->inter);
    if (L->n_routed < 1 || L->n_routed > 64) return fail(UOCR_EUNSUPPORTED, "%s: n_routed=%d outside 1..64", who, L->n_routed);
    if (L->n_shared < 0) return fail(UOCR_EINVAL, "%s: n_shared < 0", who);
    if (L->top_k < 1 || L->top_k > L->n_routed) return fail(UOCR_EINVAL, "%s: top_k=%d outside [1, E]", who, L->top_k);
    if (L->int8 && L->group != 128)
        return fail(UOCR_EUNSUPPORTED, "%s: int8 experts need the checkpoint's group size 128", who);
    if (L->int8 && L->hidden % 256)
        return fail(UOCR_EUNSUPPORTED, "%s: int8 experts need hidden=%d to be a multiple of 256", who, L->hidden);
    if (L->top_k > uocr::kDecodeMaxTopk)
        return fail(UOCR_EUNSUPPORTED, "%s: top_k=%d above %d", who, L->top_k, uocr::kDecodeMaxTopk);
    if (!L->router || !L->w13 || !L->w2) return fail(UOCR_EINVAL, "%s: null weight pointer", who);
    if (L->n_shared > 0 && (!L->w13_shared || !L->w2_shared)) return fail(UOCR_EINVAL, "%s: null shared weights", who);
    if (!a16(L->router) || !a16(L->w13) || !a16(L->w2) || (L->n_shared && (!a16(L->w13_shared) || !a16(L->w2_shared))))
        return fail(UOCR_EINVAL, "%s: weights must be 16-byte aligned", who);
    return ok();
}

}  // namespace

size_t uocr_moe_decode_workspace_bytes(const uocr_moe_layer* L, int64_t B) {
    if (!L || B < 1) return 0;
    return decode_layout(L, B).total;
}

int uocr_moe_decode(const uocr_moe_layer* L, const float* x, int64_t B, const float* bias, float* out,
                    int32_t* ids_out, float* wts_out, void* workspace, size_t workspace_bytes, uocr_stream_t stream) {
    int rc = check_layer(L, "moe_decode");
    if (rc) return rc;
    if (B < 1 || B > 8) return fail(UOCR_EINVAL, "moe_decode: B=%lld outside 1..8 (use moe_prefill)", (long long)B);
    if (L->n_shared > uocr::kDecodeMaxShared) return fail(UOCR_EUNSUPPORTED, "moe_decode: more than 8 shared experts");
    if (L->hidden > 8192 || L->inter > 128 * uocr::kDecodeMaxGroups)
        return fail(UOCR_EUNSUPPORTED, "moe_decode: hidden above 8192 or inter above %d", 128 * uocr::kDecodeMaxGroups);
    if (!x || !out || !workspace) return fail(UOCR_EINVAL, "moe_decode: null pointer");
    if (!a16(x) || !a16(out)) return fail(UOCR_EINVAL, "moe_decode: x and out must be 16-byte aligned");
    if (bias && (reinterpret_cast<uintptr_t>(bias) & 3)) return fail(UOCR_EINVAL, "moe_decode: bias must be 4-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(UOCR_EINVAL, "moe_decode: workspace must be 256-byte aligned");
    const DecodeLayout d = decode_layout(L, B);
    if (workspace_bytes < d.total)
        return fail(UOCR_EINVAL, "moe_decode: workspace of %zu bytes, need %zu", workspace_bytes, d.total);
    char* ws = reinterpret_cast<char*>(workspace);
    uocr::DecodeArgs a{};
    a.B = (int)B; a.H = L->hidden; a.I = L->inter; a.E = L->n_routed; a.S = L->n_shared; a.topk = L->top_k;
    a.G = L->int8 ? L->group : 128; a.int8 = L->int8;
    a.x = x; a.router = L->router; a.bias = bias;
    a.ids = ids_out ? ids_out : reinterpret_cast<int32_t*>(ws + d.ids);
    a.wts = wts_out ? wts_out : reinterpret_cast<float*>(ws + d.wts);
    a.w13 = L->w13; a.w2 = L->w2;
    a.w13_shared = L->w13_shared; a.w2_shared = L->w2_shared;
    a.h = reinterpret_cast<float*>(ws + d.h);
    a.y = reinterpret_cast<float*>(ws + d.y);
    a.himg = reinterpret_cast<unsigned char*>(ws + d.himg);
    a.gsig = reinterpret_cast<float*>(ws + d.gsig);
    a.out = out;
    a.ctl = reinterpret_cast<uocr::DecodeCtl*>(ws + d.ctl);
    a.logits = reinterpret_cast<float*>(ws + d.logits);
    a.xd = reinterpret_cast<unsigned char*>(ws + d.xd);
    a.xb = reinterpret_cast<unsigned char*>(ws + d.xb);
    a.xsig = reinterpret_cast<float*>(ws + d.xsig);
    return cuda_status(uocr::launch_decode_layer(a, S(stream)), "moe_decode: launch");
}

size_t uocr_moe_prefill_workspace_bytes(const uocr_moe_layer* L, int64_t T) {
    if (!L || T < 1 || T > (int64_t(1) << 24)) return 0;
    return uocr::prefill_layout((int)T, L->hidden, L->inter, L->n_routed, L->n_shared, L->top_k, L->int8 != 0).total;
}

int uocr_moe_prefill(const uocr_moe_layer* L, const float* x, int64_t T, const float* bias, float* out,
                     int32_t* ids_out, float* wts_out, void* workspace, size_t workspace_bytes, uocr_stream_t stream) {
    int rc = check_layer(L, "moe_prefill");
    if (rc) return rc;
    if (T < 1 || T > (int64_t(1) << 24)) return fail(UOCR_EINVAL, "moe_prefill: T=%lld outside 1..2^24", (long long)T);
    if ((int64_t)(L->top_k + L->n_shared) * T >= (int64_t(1) << 31))
        return fail(UOCR_EUNSUPPORTED, "moe_prefill: (top_k + n_shared) * T rows exceed int32");
    if (L->n_shared > uocr::kDecodeMaxShared) return fail(UOCR_EUNSUPPORTED, "moe_prefill: more than 8 shared experts");
    if (L->hidden % 256) return fail(UOCR_EUNSUPPORTED, "moe_prefill: hidden=%d must be a multiple of 256", L->hidden);
    if (!x || !out || !workspace) return fail(UOCR_EINVAL, "moe_prefill: null pointer");
    if (!a16(x) || !a16(out)) return fail(UOCR_EINVAL, "moe_prefill: x and out must be 16-byte aligned");
    if (bias && (reinterpret_cast<uintptr_t>(bias) & 3)) return fail(UOCR_EINVAL, "moe_prefill: bias must be 4-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return fail(UOCR_EINVAL, "moe_prefill: workspace must be 256-byte aligned");
    const uocr::PrefillLayout d =
        uocr::prefill_layout((int)T, L->hidden, L->inter, L->n_routed, L->n_shared, L->top_k, L->int8 != 0);
    if (workspace_bytes < d.total)
        return fail(UOCR_EINVAL, "moe_prefill: workspace of %zu bytes, need %zu", workspace_bytes, d.total);
    char* ws = reinterpret_cast<char*>(workspace);
    uocr::PrefillArgs a{};
    a.T = (int)T; a.H = L->hidden; a.I = L->inter; a.E = L->n_routed; a.S = L->n_shared; a.topk = L->top_k;
    a.G = L->int8 ? L->group : 128; a.int8 = L->int8;
    a.route = 1; a.use_shared = 1; a.accumulate = 0;
    a.x = x; a.router = L->router; a.bias = bias;
    a.ids = ids_out ? ids_out : reinterpret_cast<int32_t*>(ws + d.ids);
    a.wts = wts_out ? wts_out : reinterpret_cast<float*>(ws + d.wts);
    a.w13 = L->w13; a.w2 = L->w2;
    a.w13_shared = L->w13_shared; a.w2_shared = L->w2_shared;
    a.out = out;
    return cuda_status(uocr::launch_prefill(a, ws, d, S(stream)), "moe_prefill: launch");
}

// expert-parallel pieces
// ---------------------------------------------------------------------------------------

size_t uocr_moe_ep_experts_workspace_bytes(const uocr_moe_layer* L, int64_t N) {
    if (!L || N < 1 || N > (int64_t(1) << 24)) return 0;
    return uocr::prefill_layout((int)N, L->hidden, L->inter, L->n_routed, 0, L->top_k, L->int8 != 0).total;
}

int uocr_moe_ep_experts(const uocr_moe_layer* L, const uint16_t* rows, int64_t N, const int32_t* expert_local,
                        const float* weight, float* out, void* workspace, size_t workspace_bytes,
                        uocr_stream_t stream) {
    int rc = check_layer(L, "moe_ep_experts");
    if (rc) return rc;
    if (N < 0 || N > (int64_t(1) << 24)) return fail(UOCR_EINVAL, "moe_ep_experts: N=%lld outside 0..2^24", (long long)N);
    if (N == 0) return ok();
    if ((int64_t)L->top_k * N >= (int64_t(1) << 31)) return fail(UOCR_EUNSUPPORTED, "moe_ep_experts: too many rows");
    if (L->hidden % 256) return fail(UOCR_EUNSUPPORTED, "moe_ep_experts: hidden=%d must be a multiple of 256", L->hidden);
    if (!rows || !expert_local || !weight || !out || !workspace) return fail(UOCR_EINVAL, "moe_ep_experts: null pointer");
    if (!a16(rows) || !a16(out)) return fail(UOCR_EINVAL, "moe_ep_experts: rows and out must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(UOCR_EINVAL, "moe_ep_experts: workspace must be 256-byte aligned");
    const uocr::PrefillLayout d =
        uocr::prefill_layout((int)N, L->hidden, L->inter, L->n_routed, 0, L->top_k, L->int8 != 0);
    if (workspace_bytes < d.total)
        return fail(UOCR_EINVAL, "moe_ep_experts: workspace of %zu bytes, need %zu", workspace_bytes, d.total);
    char* ws = reinterpret_cast<char*>(workspace);
    uocr::PrefillArgs a{};
    a.T = (int)N; a.H = L->hidden; a.I = L->inter; a.E = L->n_routed; a.S = 0; a.topk = L->top_k;
    a.G = L->int8 ? L->group : 128; a.int8 = L->int8;
    a.route = 0; a.use_shared = 0; a.accumulate = 0;
    a.x_bf16 = rows;
    a.ids = const_cast<int32_t*>(expert_local);
    a.wts = const_cast<float*>(weight);
    a.w13 = L->w13; a.w2 = L->w2;
    a.out = out;
    return cuda_status(uocr::launch_prefill(a, ws, d, S(stream)), "moe_ep_experts: launch");
}

size_t uocr_moe_ep_dispatch_workspace_bytes(int64_t T, int64_t world) {
    if (T < 1 || T > (int64_t(1) << 24) || world < 1 || world > uocr::kEpMaxWorld) return 0;
    return uocr::ep_dispatch_workspace_bytes((int)T, (int)world);
}

int uocr_moe_ep_dispatch(const float* x, int64_t T, int64_t H, const int32_t* ids, const float* wts, int64_t top_k,
                         const int32_t* owner, const int32_t* local, int64_t E, int64_t world, int64_t* send_counts,
                         uint16_t* rows, int32_t* meta, int32_t* inv, void* workspace, size_t workspace_bytes,
                         uocr_stream_t stream) {
    if (T < 0 || T > (int64_t(1) << 24)) return fail(UOCR_EINVAL, "moe_ep_dispatch: T=%lld outside 0..2^24", (long long)T);
    if (world < 1 || world > uocr::kEpMaxWorld)
        return fail(UOCR_EUNSUPPORTED, "moe_ep_dispatch: world=%lld outside 1..%d", (long long)world, uocr::kEpMaxWorld);
    if (H < 8 || H % 8) return fail(UOCR_EINVAL, "moe_ep_dispatch: hidden=%lld must be a positive multiple of 8", (long long)H);
    if (top_k < 1 || top_k > 64) return fail(UOCR_EINVAL, "moe_ep_dispatch: top_k=%lld outside 1..64", (long long)top_k);
    if (E < 1 || E > 4096) return fail(UOCR_EINVAL, "moe_ep_dispatch: E=%lld outside 1..4096", (long long)E);
    if (T * world * H >= (int64_t(1) << 40)) return fail(UOCR_EUNSUPPORTED, "moe_ep_dispatch: too many rows");
    if (!send_counts) return fail(UOCR_EINVAL, "moe_ep_dispatch: null pointer");
    if (T == 0) {
        cudaError_t err = cudaMemsetAsync(send_counts, 0, sizeof(int64_t) * world, S(stream));
        return cuda_status(err, "moe_ep_dispatch: clear counts");
    }
    if (!x || !ids || !wts || !owner || !local || !rows || !meta || !inv || !workspace)
        return fail(UOCR_EINVAL, "moe_ep_dispatch: null pointer");
    if (!a16(x) || !a16(rows)) return fail(UOCR_EINVAL, "moe_ep_dispatch: x and rows must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(UOCR_EINVAL, "moe_ep_dispatch: workspace must be 256-byte aligned");
    const size_t need = uocr::ep_dispatch_workspace_bytes((int)T, (int)world);
    if (workspace_bytes < need)
        return fail(UOCR_EINVAL, "moe_ep_dispatch: workspace of %zu bytes, need %zu", workspace_bytes, need);
    return cuda_status(uocr::launch_ep_dispatch(x, (int)T, (int)H, ids, wts, (int)top_k, owner, local, (int)E,
                                                (int)world, reinterpret_cast<long long*>(send_counts), rows, meta,
                                                inv, workspace, S(stream)),
                       "moe_ep_dispatch: launch");
}

int uocr_moe_ep_combine(const float* partials, int64_t n_rows, const int32_t* inv, int64_t T, int64_t world,
                        int64_t H, const float* add, float* out, uocr_stream_t stream) {
    if (T < 0 || T > (int64_t(1) << 24)) return fail(UOCR_EINVAL, "moe_ep_combine: T=%lld outside 0..2^24", (long long)T);
    if (world < 1 || world > uocr::kEpMaxWorld)
        return fail(UOCR_EUNSUPPORTED, "moe_ep_combine: world=%lld outside 1..%d", (long long)world, uocr::kEpMaxWorld);
    if (H < 4 || H % 4) return fail(UOCR_EINVAL, "moe_ep_combine: hidden=%lld must be a positive multiple of 4", (long long)H);
    if (n_rows < 0) return fail(UOCR_EINVAL, "moe_ep_combine: negative row count");
    if (T == 0) return ok();
    if (!inv || !out || (n_rows > 0 && !partials)) return fail(UOCR_EINVAL, "moe_ep_combine: null pointer");
    if (!a16(out) || (partials && !a16(partials)) || (add && !a16(add)))
        return fail(UOCR_EINVAL, "moe_ep_combine: partials, add and out must be 16-byte aligned");
    return cuda_status(uocr::launch_ep_combine(partials, (long long)n_rows, inv, (int)T, (int)world, (int)H, add, out,
                                               S(stream)),
                       "moe_ep_combine: launch");
}

size_t uocr_moe_shared_workspace_bytes(const uocr_moe_layer* L, int64_t T) {
    if (!L || T < 1 || T > (int64_t(1) << 24)) return 0;
    return uocr::prefill_layout((int)T, L->hidden, L->inter, L->n_routed, L->n_shared, 0, false).total;
}

int uocr_moe_shared_forward(const uocr_moe_layer* L, const float* x, int64_t T, float* out, int accumulate,
                            void* workspace, size_t workspace_bytes, uocr_stream_t stream) {
    if (!L) return fail(UOCR_EINVAL, "moe_shared_forward: null layer");
    if (T < 0 || T > (int64_t(1) << 24)) return fail(UOCR_EINVAL, "moe_shared_forward: T=%lld outside 0..2^24", (long long)T);
    if (T == 0) return ok();
    if (L->n_shared < 1 || L->n_shared > uocr::kDecodeMaxShared)
        return fail(UOCR_EUNSUPPORTED, "moe_shared_forward: n_shared=%d outside 1..8", L->n_shared);
    if (L->hidden < 256 || L->hidden % 256 || L->inter < 128 || L->inter % 128)
        return fail(UOCR_EUNSUPPORTED, "moe_shared_forward: hidden must be a multiple of 256, inter of 128");
    if (!L->w13_shared || !L->w2_shared || !x || !out || !workspace) return fail(UOCR_EINVAL, "moe_shared_forward: null pointer");
    if (!a16(x) || !a16(out) || !a16(L->w13_shared) || !a16(L->w2_shared))
        return fail(UOCR_EINVAL, "moe_shared_forward: pointers must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(UOCR_EINVAL, "moe_shared_forward: workspace must be 256-byte aligned");
    const uocr::PrefillLayout d = uocr::prefill_layout((int)T, L->hidden, L->inter, L->n_routed, L->n_shared, 0, false);
    if (workspace_bytes < d.total)
        return fail(UOCR_EINVAL, "moe_shared_forward: workspace of %zu bytes, need %zu", workspace_bytes, d.total);
    char* ws = reinterpret_cast<char*>(workspace);
    uocr::PrefillArgs a{};
    // no routed entries: the routed tensor maps are sized over the shared weights and never read
    a.T = (int)T; a.H = L->hidden; a.I = L->inter; a.E = L->n_shared; a.S = L->n_shared; a.topk = 0;
    a.G = 128; a.int8 = 0;
    a.route = 0; a.use_shared = 1; a.accumulate = accumulate != 0;
    // this entry point serves the expert-parallel layer, where it runs beside NCCL's exchange
    // kernels: its GEMMs leave 16 SMs free so those kernels are not queued behind them
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) ==
                                                  cudaSuccess && sms > 32)
        a.max_ctas = sms - 16;
    a.x = x;
    a.w13 = L->w13_shared; a.w2 = L->w2_shared;  // no routed groups: the routed maps are never read
    a.w13_shared = L->w13_shared; a.w2_shared = L->w2_shared;
    a.out = out;
    return cuda_status(uocr::launch_prefill(a, ws, d, S(stream)), "moe_shared_forward: launch");
}

// ---------------------------------------------------------------------------------------
// expert-parallel exchange through peer memory
// ---------------------------------------------------------------------------------------

static int check_peers(const uocr_ep_peers* P, const char* who) {
    if (!P) return fail(UOCR_EINVAL, "%s: null peers", who);
    if (P->world < 1 || P->world > uocr::kEpMaxWorld)
        return fail(UOCR_EUNSUPPORTED, "%s: world=%d outside 1..%d", who, P->world, uocr::kEpMaxWorld);
    if (P->rank < 0 || P->rank >= P->world) return fail(UOCR_EINVAL, "%s: rank=%d outside [0, world)", who, P->rank);
    if (P->cap_tokens < 1 || P->cap_tokens > (1 << 22))
        return fail(UOCR_EINVAL, "%s: cap_tokens=%d outside 1..2^22", who, P->cap_tokens);
    if (P->hidden < 256 || P->hidden % 256 || P->hidden > 8192)
        return fail(UOCR_EUNSUPPORTED, "%s: hidden=%d must be a multiple of 256 up to 8192", who, P->hidden);
    if (P->top_k < 1 || P->top_k > uocr::kDecodeMaxTopk) return fail(UOCR_EINVAL, "%s: top_k=%d outside 1..8", who, P->top_k);
    if (P->epoch < 1 || P->epoch > (1ull << 62)) return fail(UOCR_EINVAL, "%s: epoch must be 1..2^62", who);
    if ((int64_t)P->world * P->cap_tokens * P->top_k >= (int64_t(1) << 31))
        return fail(UOCR_EUNSUPPORTED, "%s: world * cap_tokens * top_k exceeds int32", who);
    for (int q = 0; q < P->world; ++q)
        if (!P->buf[q] || (reinterpret_cast<uintptr_t>(P->buf[q]) & 255))
            return fail(UOCR_EINVAL, "%s: buf[%d] null or not 256-byte aligned", who, q);
    return ok();
}

static uocr::EpPeers to_peers(const uocr_ep_peers* P) {
    uocr::EpPeers e{};
    e.world = P->world; e.rank = P->rank; e.cap = P->cap_tokens; e.H = P->hidden; e.k = P->top_k;
    e.epoch = P->epoch;
    for (int q = 0; q < P->world; ++q) e.buf[q] = reinterpret_cast<unsigned char*>(P->buf[q]);
    return e;
}

static uocr::EpPeerScratch peer_scratch(const uocr_moe_layer* L, const uocr_ep_peers* P) {
    const int rows = P->world * P->cap_tokens;
    const size_t pre =
        uocr::prefill_layout(rows, L->hidden, L->inter, L->n_routed, 0, L->top_k, L->int8 != 0).total;
    return uocr::ep_peer_scratch(P->world, P->cap_tokens, L->hidden, L->inter, L->n_routed, L->top_k, L->int8 != 0,
                                 pre);
}

size_t uocr_moe_ep_peer_buffer_bytes(int64_t world, int64_t cap_tokens, int64_t hidden, int64_t top_k) {
    if (world < 1 || world > uocr::kEpMaxWorld || cap_tokens < 1 || cap_tokens > (1 << 22) || hidden < 8 ||
        hidden > 8192 || top_k < 1 || top_k > uocr::kDecodeMaxTopk)
        return 0;
    return uocr::ep_peer_layout((int)world, (int)cap_tokens, (int)hidden, (int)top_k).total;
}

size_t uocr_moe_ep_peer_workspace_bytes(const uocr_moe_layer* L, const uocr_ep_peers* P) {
    if (!L || !P || P->world < 1 || P->world > uocr::kEpMaxWorld || P->cap_tokens < 1) return 0;
    return peer_scratch(L, P).total;
}

int uocr_moe_ep_peer_dispatch(const uocr_ep_peers* P, const float* x, int64_t T, const int32_t* ids,
                              const float* wts, const int32_t* owner, const int32_t* local, int64_t E, int32_t* inv,
                              void* workspace, size_t workspace_bytes, uocr_stream_t stream) {
    int rc = check_peers(P, "moe_ep_peer_dispatch");
    if (rc) return rc;
    if (T < 0 || T > P->cap_tokens)
        return fail(UOCR_EINVAL, "moe_ep_peer_dispatch: T=%lld outside 0..cap_tokens=%d", (long long)T, P->cap_tokens);
    if (E < 1 || E > 4096) return fail(UOCR_EINVAL, "moe_ep_peer_dispatch: E=%lld outside 1..4096", (long long)E);
    if ((T > 0 && (!x || !ids || !wts || !inv)) || !owner || !local || !workspace)
        return fail(UOCR_EINVAL, "moe_ep_peer_dispatch: null pointer");
    if (T > 0 && !a16(x)) return fail(UOCR_EINVAL, "moe_ep_peer_dispatch: x must be 16-byte aligned");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return fail(UOCR_EINVAL, "moe_ep_peer_dispatch: workspace must be 256-byte aligned");
    // the dispatch part of the scratch does not depend on the layer: size it with a stand-in
    const uocr::EpPeerScratch d = uocr::ep_peer_scratch(P->world, P->cap_tokens, P->hidden, 0, 0, P->top_k, false, 0);
    if (workspace_bytes < d.prefill)
        return fail(UOCR_EINVAL, "moe_ep_peer_dispatch: workspace of %zu bytes, need %zu", workspace_bytes, d.prefill);
    return cuda_status(uocr::launch_ep_peer_dispatch(to_peers(P), x, (int)T, ids, wts, owner, local, (int)E, inv,
                                                     reinterpret_cast<char*>(workspace), d, S(stream)),
                       "moe_ep_peer_dispatch: launch");
}

int uocr_moe_ep_peer_experts(const uocr_moe_layer* L, const uocr_ep_peers* P, void* workspace, size_t workspace_bytes,
                             uocr_stream_t stream) {
    int rc = check_layer(L, "moe_ep_peer_experts");
    if (rc) return rc;
    rc = check_peers(P, "moe_ep_peer_experts");
    if (rc) return rc;
    if (P->hidden != L->hidden || P->top_k != L->top_k)
        return fail(UOCR_EINVAL, "moe_ep_peer_experts: peers and layer disagree on hidden or top_k");
    if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 255))
        return fail(UOCR_EINVAL, "moe_ep_peer_experts: workspace null or not 256-byte aligned");
    const uocr::EpPeerScratch d = peer_scratch(L, P);
    if (workspace_bytes < d.total)
        return fail(UOCR_EINVAL, "moe_ep_peer_experts: workspace of %zu bytes, need %zu", workspace_bytes, d.total);
    const int rows = P->world * P->cap_tokens;
    const uocr::EpPeerLayout X = uocr::ep_peer_layout(P->world, P->cap_tokens, P->hidden, P->top_k);
    const uocr::EpPeers peers = to_peers(P);
    char* ws = reinterpret_cast<char*>(workspace);
    cudaError_t err = uocr::launch_ep_peer_wait(peers, ws, d, S(stream));
    if (err != cudaSuccess) return cuda_status(err, "moe_ep_peer_experts: wait");
    unsigned char* own = peers.buf[peers.rank];
    uocr::PrefillArgs a{};
    a.T = rows; a.H = L->hidden; a.I = L->inter; a.E = L->n_routed; a.S = 0; a.topk = L->top_k;
    a.G = L->int8 ? L->group : 128; a.int8 = L->int8;
    a.route = 0; a.use_shared = 0; a.accumulate = 0;
    a.x_bf16 = reinterpret_cast<const uint16_t*>(own + X.rows);
    a.ids = reinterpret_cast<int32_t*>(own + X.eid);
    a.wts = reinterpret_cast<float*>(own + X.w);
    a.w13 = L->w13; a.w2 = L->w2;
    a.peers = &peers;
    a.slot_counts = reinterpret_cast<const int*>(ws + d.hdr + uocr::kEpHdrSlotCounts);
    a.slot_fail = reinterpret_cast<const int*>(ws + d.hdr + uocr::kEpHdrSlotFail);
    a.done = reinterpret_cast<unsigned int*>(ws + d.hdr + uocr::kEpHdrDonePart);
    a.status = reinterpret_cast<uint32_t*>(own + X.status);
    const uocr::PrefillLayout pl =
        uocr::prefill_layout(rows, L->hidden, L->inter, L->n_routed, 0, L->top_k, L->int8 != 0);
    return cuda_status(uocr::launch_prefill(a, ws + d.prefill, pl, S(stream)), "moe_ep_peer_experts: launch");
}

int uocr_moe_ep_peer_combine(const uocr_ep_peers* P, const int32_t* inv, int64_t T, const float* add, float* out,
                             uocr_stream_t stream) {
    int rc = check_peers(P, "moe_ep_peer_combine");
    if (rc) return rc;
    if (T < 0 || T > P->cap_tokens)
        return fail(UOCR_EINVAL, "moe_ep_peer_combine: T=%lld outside 0..cap_tokens=%d", (long long)T, P->cap_tokens);
    if (T > 0 && (!inv || !out)) return fail(UOCR_EINVAL, "moe_ep_peer_combine: null pointer");
    if ((out && !a16(out)) || (add && !a16(add)))
        return fail(UOCR_EINVAL, "moe_ep_peer_combine: add and out must be 16-byte aligned");
    return cuda_status(uocr::launch_ep_peer_combine(to_peers(P), inv, (int)T, add, out, S(stream)),
                       "moe_ep_peer_combine: launch");
}

static PFN_cuMemGetAddressRange_v3020 address_range_fn() {
    static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
    });
    return fn;
}

int uocr_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out) {
    if (!dev_ptr || !handle_out || !offset_out) return fail(UOCR_EINVAL, "ipc_export: null pointer");
    auto range = address_range_fn();
    if (!range) return fail(UOCR_ECUDA, "ipc_export: cuMemGetAddressRange unavailable");
    CUdeviceptr base = 0;
    size_t size = 0;
    if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
        return fail(UOCR_EINVAL, "ipc_export: not a device allocation");
    cudaIpcMemHandle_t h;
    cudaError_t err = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
    if (err != cudaSuccess) return cuda_status(err, "ipc_export: cudaIpcGetMemHandle");
    static_assert(sizeof(h) == UOCR_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle_out, &h, sizeof h);
    *offset_out = reinterpret_cast<uint64_t>(dev_ptr) - (uint64_t)base;
    return ok();
}

int uocr_ipc_import(const void* handle, uint64_t offset, void** dev_ptr_out) {
    if (!handle || !dev_ptr_out) return fail(UOCR_EINVAL, "ipc_import: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    void* base = nullptr;
    cudaError_t err = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) return cuda_status(err, "ipc_import: cudaIpcOpenMemHandle");
    *dev_ptr_out = reinterpret_cast<char*>(base) + offset;
    return ok();
}

int uocr_ipc_close(void* dev_ptr, uint64_t offset) {
    if (!dev_ptr) return fail(UOCR_EINVAL, "ipc_close: null pointer");
    return cuda_status(cudaIpcCloseMemHandle(reinterpret_cast<char*>(dev_ptr) - offset), "ipc_close");
}

int uocr_moe_decode_set_trace(void* device_buffer, size_t bytes) {
    uocr::g_decode_trace = reinterpret_cast<unsigned long long*>(device_buffer);
    uocr::g_decode_trace_bytes = device_buffer ? bytes : 0;
    return ok();
}

int uocr_moe_device_status(const void* workspace, uocr_stream_t stream) {
    if (!workspace) return fail(UOCR_EINVAL, "device_status: null workspace");
    uint32_t code = 0;
    return uocr::read_clear_status(workspace, S(stream), &code);
}

int uocr_moe_test_wait_extra(int extra) {
    if (extra < 0 || extra > 1024) return fail(UOCR_EINVAL, "test_wait_extra: %d outside 0..1024", extra);
    uocr::g_decode_wait_extra = extra;
    return ok();
}

}  // extern "C"
