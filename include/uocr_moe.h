/*
 * uocr_moe.h -- C ABI of libuocr_moe.so, the B200 (sm_100a) implementation of the
 * DeepSeek-V2 mixture-of-experts sublayer of the Unlimited-OCR decoder.
 *
 * Conventions for every entry point:
 *   - all tensor pointers are DEVICE pointers, row-major and packed, owned by the caller;
 *     no entry point allocates device memory;
 *   - bf16 tensors are passed as uint16_t bit patterns;
 *   - work is enqueued asynchronously on `stream` (a cudaStream_t; NULL = legacy default);
 *   - the return value is a status: UOCR_OK (0) or an error code; on error,
 *     uocr_last_error() returns a thread-local message. Shape errors are detected on the
 *     host before anything is launched and carry the reference op's message text;
 *   - out-of-range expert ids are clamped to [0, E) on the device, never faulting
 *     (kernels/moe_routing.mojo:11-16 of the reference).
 */
#ifndef UOCR_MOE_H
#define UOCR_MOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* uocr_stream_t; /* cudaStream_t */

/* Only the functions of this header are exported from libuocr_moe.so. */
#if defined(__GNUC__)
#define UOCR_API __attribute__((visibility("default")))
#else
#define UOCR_API
#endif

enum {
    UOCR_OK = 0,
    UOCR_EINVAL = 1,      /* bad shape or argument (host-side check, nothing launched) */
    UOCR_ECUDA = 2,       /* a CUDA runtime call failed */
    UOCR_EDEVICE = 3,     /* a device-side bounded wait gave up (see uocr_moe_device_status) */
    UOCR_EUNSUPPORTED = 4 /* a configuration this build does not implement */
};

/* Element types of the entry points that take more than one (uocr_quantize_int8_g128). */
enum { UOCR_DTYPE_F32 = 0, UOCR_DTYPE_BF16 = 1 };

/* Thread-local message of the last failed call on this thread ("" if none). */
UOCR_API const char* uocr_last_error(void);
/* ABI version of this header (bumped on any signature change). */
UOCR_API int uocr_abi_version(void);

/* ------------------------------------------------------------------------------------ *
 * The reference's MoE custom ops, 1:1 (same arguments, same shape checks and messages,
 * same clamp and empty-batch behaviour). Each tensor is given with its dims, as the
 * reference op receives whole tensors.
 * ------------------------------------------------------------------------------------ */

/* moe_bf16_qmv: out[s,n] = sum_k f32(w[clamp(ids[s]),n,k]) * x[s,k]   (fp32 accumulate)
 * Replaces @register("moe_bf16_qmv"), unlimited_ocr_max/kernels/moe_bf16.mojo:264-345,
 * staged by StackedExperts._qmv (unlimited_ocr_max/decoder.py:355-366).
 * Every row's bits are independent of the other rows of the call. */
UOCR_API int uocr_moe_bf16_qmv(float* out, int64_t out_rows, int64_t out_cols,
                      const float* x, int64_t x_rows, int64_t x_cols,
                      const int32_t* expert_ids, int64_t ids_len,
                      const uint16_t* w, int64_t w_e, int64_t w_n, int64_t w_k,
                      uocr_stream_t stream);

/* moe_int8_qmv: out[s,n] = sum_g scales[e,n,g] * sum_{k in g} f32(w[e,n,k]) * x[s,k],
 * e = clamp(ids[s]), in the reference's exact fp32 operation order (gsum = fma(q, x, gsum)
 * in ascending k, then acc = fma(scale, gsum, acc)), so the output bits equal the
 * reference op's. Replaces @register("moe_int8_qmv"), kernels/moe_int8.mojo:181-258. */
UOCR_API int uocr_moe_int8_qmv(float* out, int64_t out_rows, int64_t out_cols,
                      const float* x, int64_t x_rows, int64_t x_cols,
                      const int32_t* expert_ids, int64_t ids_len,
                      const int8_t* w, int64_t w_e, int64_t w_n, int64_t w_k,
                      const float* scales, int64_t s_e, int64_t s_n, int64_t s_g,
                      uocr_stream_t stream);

/* int8_dequant_expert: out[n,k] = bf16_rne(f32(w[e,n,k]) * scales[e,n,k/G]), e = clamp(*idx).
 * Bit-exact. Replaces @register("int8_dequant_expert"), kernels/moe_int8.mojo:261-342. */
UOCR_API int uocr_int8_dequant_expert(uint16_t* out, int64_t out_n, int64_t out_k,
                             const int8_t* w, int64_t w_e, int64_t w_n, int64_t w_k,
                             const float* scales, int64_t s_e, int64_t s_n, int64_t s_g,
                             const int32_t* expert_idx, int64_t idx_len,
                             uocr_stream_t stream);

/* dense_bf16_qmv[tile]: out[m,n] = sum_k f32(W[n,k]) * x[m,k] with W held K-blocked as
 * w[k/16, n, k%16]. Replaces @register("dense_bf16_qmv"), kernels/dense_bf16.mojo:119-158
 * (wrapper decoder.py:166-184). `tile` >= 1 is accepted for interface parity; a row's bits
 * do not depend on it. */
UOCR_API int uocr_dense_bf16_qmv(float* out, int64_t out_rows, int64_t out_cols,
                        const float* x, int64_t x_rows, int64_t x_cols,
                        const uint16_t* w, int64_t w_kb, int64_t w_n, int64_t w_blk,
                        int tile, uocr_stream_t stream);

/* Dense bf16 projections of the decode step (attention q/k/v/o, the dense FFN, lm_head) streamed
 * through the tensor cores: replaces dense_bf16_qmv (kernels/dense_bf16.mojo:119-158, decoder.py:
 * 166-184, 236-238) for a weight packed once at load. out[m, n] = sum_k W[n, k] x[m, k], fp32 x
 * and out, the weight read once per 8 rows; x enters the products as two bf16 terms (to ~2^-17 of
 * its magnitude), the products accumulate in fp32.
 *   uocr_dense_packed_bytes(N, K)  size of the packed weight (0 for unsupported dims: N >= 1, K a
 *                                  positive multiple of 16);
 *   uocr_dense_pack                W [N, K] bf16 -> packed; `kblocked` = 1 takes the reference's
 *                                  K-blocked declaration w[k/16, n, k%16] (decoder.py:201-225), 0 a
 *                                  plain row-major [N, K]; 16-byte-aligned pointers;
 *   uocr_dense_stream_workspace_bytes(N, K)  workspace of one call on the current device; the
 *                                  caller zero-fills it once and may reuse it for every later
 *                                  call of the same (N, K); its status word is read and cleared
 *                                  by uocr_moe_device_status;
 *   uocr_dense_stream              x [M, K] fp32 -> out [M, N] fp32, any M >= 0 (8 rows per launch). */
UOCR_API size_t uocr_dense_packed_bytes(int64_t N, int64_t K);
UOCR_API int uocr_dense_pack(const uint16_t* w, int kblocked, int64_t N, int64_t K, void* packed,
                    uocr_stream_t stream);
UOCR_API size_t uocr_dense_stream_workspace_bytes(int64_t N, int64_t K);
UOCR_API int uocr_dense_stream(const void* packed, int64_t N, int64_t K, const float* x, int64_t M,
                      float* out, void* workspace, size_t workspace_bytes, uocr_stream_t stream);

/* Paged decode attention for B requests, one new token each: replaces paged_decode_attention,
 * decoder.py:425-437 (MAX's store_k/v_cache_ragged + flash_attention_ragged, causal) over the page
 * pool of kv_cache.py. Pool kv_pool fp32 [pages][2 (k, v)][layers][128 rows][heads][head_dim]; request
 * b's logical row r is row r % 128 of page lut[b * lut_cols + r / 128]. The call stores k_new[b] /
 * v_new[b] ([B][heads][head_dim], post-RoPE) at row write_index[b] of `layer` and writes out[b] =
 * softmax(q[b] . k^T * scale) v over rows [0, attend_len[b]) (write_index[b] < attend_len[b] <=
 * lut_cols * 128; page ids past the pool read its last page). head_dim 128, heads <= 12. The
 * workspace (uocr_paged_attention_workspace_bytes(B, heads, lut_cols) bytes, 16-byte aligned) is
 * zero-filled once by the caller; its status word is read by uocr_moe_device_status. The result
 * is deterministic (a fixed combine order). */
UOCR_API size_t uocr_paged_attention_workspace_bytes(int64_t B, int64_t heads, int64_t lut_cols);
UOCR_API int uocr_paged_decode_attention(const float* q, const float* k_new, const float* v_new, int64_t B,
                                int64_t heads, int64_t head_dim, float* kv_pool, int64_t pages,
                                int64_t layers, int64_t layer, const uint32_t* lut, int64_t lut_cols,
                                const uint32_t* write_index, const uint32_t* attend_len, float scale,
                                float* out, void* workspace, size_t workspace_bytes, uocr_stream_t stream);

/* RoPE on the decode step's fused q|k|v projection output qkv [B][3 x heads x head_dim] (q, then k,
 * then v, each heads x head_dim): q = x_q cos + rotate_half(x_q) sin, k likewise, v copied, into
 * q, k, v [B][heads][head_dim]; cos, sin [B][head_dim] are the rotary table's rows at each row's
 * position; each product and the sum rounded separately in fp32. Replaces Attention._rope on q and
 * k in Attention.decode, decoder.py:459-462, 478-493. */
UOCR_API int uocr_rope_qkv(const float* qkv, int64_t B, int64_t heads, int64_t head_dim, const float* cos,
                  const float* sin, float* q, float* k, float* v, uocr_stream_t stream);

/* The token embedding of the decode step: out[b] = fp32(table[clamp(ids[b], 0, vocab - 1)]) for a
 * bf16 table [vocab, hidden]. Replaces EmbeddingTable, decoder.py:241-249 (a gather). */
UOCR_API int uocr_embed_rows(const uint16_t* table, int64_t vocab, int64_t hidden, const int32_t* ids, int64_t B,
                    float* out, uocr_stream_t stream);
/* The dense FFN's activation on the fused gate|up output gate_up [B][2 x inter] (gate, then up):
 * out[b][j] = silu(g) * u with silu(g) = g / (1 + e^-g) in fp32. Replaces ops.silu(gate) * up in
 * GatedMlp.decode_rows, decoder.py:276-278. */
UOCR_API int uocr_silu_mul(const float* gate_up, int64_t B, int64_t inter, float* out, uocr_stream_t stream);

/* ngram_block: the no-repeat-n-gram guard on B rows of V fp32 logits. Row b is guarded against
 * row b of history [B, H] int32 (that request's last H token ids, the newest last): every token
 * that would complete a repeat of the last n - 1 ids inside the history is set to -3.0e38 in out,
 * every other logit is copied bit for bit (out may be logits itself). n is read from the device
 * int32 at `ngram` (so one captured launch serves any n); n < 1, or H < n, bans nothing. One row
 * is B = 1. Replaces @register("ngram_block"), kernels/ngram_block.mojo:51-151 (staged by
 * apply_ngram_guard / NgramBlocker, ngram.py:34-104). */
UOCR_API int uocr_ngram_block(const float* logits, int64_t B, int64_t V, const int32_t* history, int64_t H,
                     const int32_t* ngram, float* out, uocr_stream_t stream);

/* The residual add and the RMSNorm around a MoE sublayer of the decode step, fused: h += add
 * (skipped if add is NULL), then y = h / sqrt(mean(h^2) + eps) * gamma per row (skipped if y is
 * NULL); h, add, y fp32 [B, H], gamma fp32 [H] (the bf16 norm weight cast to fp32, as RmsNorm
 * does). Replaces x + mlp.decode_rows(post_attention_layernorm(x)) around the MoE call,
 * decoder.py:709, and RmsNorm, decoder.py:252-261 (MAX's rms_norm). */
UOCR_API int uocr_residual_rmsnorm(float* h, const float* add, const float* gamma, int64_t B, int64_t H,
                          float eps, float* y, uocr_stream_t stream);

/* quantize_per_group: the symmetric per-group int8 format of the int8 checkpoint, on the device.
 * w is [rows, K] row-major, fp32 (w_dtype UOCR_DTYPE_F32) or bf16 (UOCR_DTYPE_BF16), K a multiple
 * of 128; per 128-element group along K: amax = max|w|, scale = amax / 127 in fp32 (1.0 for an
 * all-zero group), q = clip(rint(w / scale), -127, 127) with rint half to even; q int8 [rows, K],
 * scales fp32 [rows, K/128]. Bit-identical to the reference tool's numpy arithmetic. A NaN or Inf
 * element sets *nonfinite (a device int the caller zeroes and reads; the reference refuses such a
 * weight). Replaces quantize_per_group, tools/quantize_int8.py:298-329. */
UOCR_API int uocr_quantize_int8_g128(const void* w, int w_dtype, int64_t rows, int64_t K,
                            int8_t* q, float* scales, int* nonfinite, uocr_stream_t stream);

/* ------------------------------------------------------------------------------------ *
 * The MoE sublayer (MoE.decode_rows / MoE.__call__, unlimited_ocr_max/decoder.py:641-667).
 * ------------------------------------------------------------------------------------ */

/* One layer's device-resident weights, in this library's packed layout (uocr_moe_pack_w13,
 * uocr_moe_pack_w2, uocr_moe_pack_shared). Plain pointers, caller-owned. */
typedef struct uocr_moe_layer {
    int32_t hidden;     /* H (1280), multiple of 128 (of 256 with int8 experts) */
    int32_t inter;      /* I, moe_intermediate_size (896); multiple of 128 */
    int32_t n_routed;   /* E (64), <= 64 */
    int32_t n_shared;   /* S (2): shared_experts_dim = S * I */
    int32_t top_k;      /* k (6) */
    int32_t group;      /* int8 group size along K (128) */
    int32_t int8;       /* 1: routed stacks int8 with fp32 scales inside the blocks; 0: bf16 */
    int32_t reserved;
    const uint16_t* router;     /* bf16 [E, H]  (gate.gate_score.weight) */
    const void* w13;            /* routed gate|up blocks (uocr_moe_pack_w13) */
    const void* w2;             /* routed down blocks (uocr_moe_pack_w2) */
    const uint16_t* w13_shared; /* shared gate|up as S bf16 experts (uocr_moe_pack_shared) */
    const uint16_t* w2_shared;  /* shared down as S bf16 experts (uocr_moe_pack_shared) */
} uocr_moe_layer;

/* Packed layouts (the reference keeps the checkpoint's [E, N, K] stacks, decoder.py:305-313;
 * this library re-lays them out once at load into the shared-memory image the tensor cores
 * read, so that one decode work item is one contiguous block):
 *   atom: 128 rows x 128 bytes of one K range (128 int8 or 64 bf16 elements), byte c of row r
 *         at r * 128 + ((c / 16) ^ (r % 8)) * 16 + c % 16 (the 128-byte swizzle);
 *   item: a row block's atoms over one K range, then for int8 their fp32 scales
 *         [atom][128 rows] (one 128-element group per int8 atom);
 *   w13: per expert, I/64 row blocks of 64 gate/up row pairs (rows 16i..16i+7 gate rows of
 *        pairs 8i..8i+7, rows 16i+8..16i+15 the matching up rows), each row block H/256
 *        (int8) or H/128 (bf16) items of 2 atoms;
 *   w2:  per expert, H/128 row blocks of 128 output rows, each ceil(I/256) (int8, the last
 *        item one atom when I/128 is odd) or I/128 (bf16) items of up to 2 atoms.
 * Sizes in bytes for E experts (0 for unsupported shapes): */
UOCR_API size_t uocr_moe_w13_bytes(int64_t E, int64_t I, int64_t H, int64_t group, int int8);
UOCR_API size_t uocr_moe_w2_bytes(int64_t E, int64_t H, int64_t I, int64_t group, int int8);

/* Pack experts.gate_proj / experts.up_proj [E, I, H] (bf16 or int8; for int8 also their
 * _scales [E, I, H/G] fp32, decoder.py:305-313) into w13_out (uocr_moe_w13_bytes bytes). */
UOCR_API int uocr_moe_pack_w13(const void* gate, const void* up, const float* gate_scales,
                               const float* up_scales, int64_t E, int64_t I, int64_t H, int64_t group,
                               int int8, void* w13_out, uocr_stream_t stream);

/* Pack experts.down_proj [E, H, I] (+ int8 _scales [E, H, I/G]) into w2_out. */
UOCR_API int uocr_moe_pack_w2(const void* down, const float* down_scales, int64_t E, int64_t H, int64_t I,
                              int64_t group, int int8, void* w2_out, uocr_stream_t stream);

/* Pack the shared experts (shared_experts.{gate,up,down}_proj.weight as [S*I, H], [S*I, H],
 * [H, S*I] in plain [out, in] order) into w13_shared (uocr_moe_w13_bytes(S, I, H, 128, 0)
 * bytes) and w2_shared (uocr_moe_w2_bytes(S, H, I, 128, 0) bytes), bf16 layouts as above:
 * shared expert s owns intermediate rows [s*I, (s+1)*I). */
UOCR_API int uocr_moe_pack_shared(const uint16_t* gate, const uint16_t* up, const uint16_t* down,
                         int64_t S, int64_t I, int64_t H,
                         uint16_t* w13_out, uint16_t* w2_out, uocr_stream_t stream);

/* Router: MoEGate.__call__ (decoder.py:509-514): fp32 logits x @ router^T (+ optional
 * per-expert bias, a benchmark input), softmax over all E experts, greedy top-k by
 * (probability desc, expert index asc), no renormalisation. ids [T, k] int32 and
 * weights [T, k] fp32 in score order. Bit-exact with the oracle's stated fp32 order. */
UOCR_API int uocr_moe_route(const float* x, int64_t T, int64_t H, const uint16_t* router, int64_t E,
                   const float* bias, int64_t top_k, int32_t* ids_out, float* wts_out,
                   uocr_stream_t stream);

/* Decode step (MoE.decode_rows, decoder.py:641-655): x [B, H] fp32, 1 <= B <= 8 ->
 * out [B, H] fp32 = routed top-k experts weighted by the router + shared experts.
 * ids_out / wts_out (nullable) receive the routing. `workspace` must hold
 * uocr_moe_decode_workspace_bytes(L, B) bytes (256-byte aligned), zero-filled once before its
 * first use. Two launches: the router logits, then one persistent experts kernel (one CTA per SM,
 * all resident: they wait on each other's units; a kernel of another stream that holds SMs makes
 * the call fail as below, it never hangs). Every device-side wait is bounded: a
 * call in which one gave up writes NaN over `out` and sets the workspace's sticky status; until
 * uocr_moe_device_status has read (and so cleared) it, later calls on that workspace write NaN too. */
UOCR_API size_t uocr_moe_decode_workspace_bytes(const uocr_moe_layer* L, int64_t B);
UOCR_API int uocr_moe_decode(const uocr_moe_layer* L, const float* x, int64_t B, const float* bias,
                    float* out, int32_t* ids_out, float* wts_out,
                    void* workspace, size_t workspace_bytes, uocr_stream_t stream);

/* Prefill (MoE.__call__, decoder.py:657-667, routed part as _routed_native, decoder.py:606-614:
 * moe_create_indices + grouped_matmul_ragged + the weighted mix): x [T, H] fp32, T >= 1 ->
 * out [T, H] fp32. Tokens are permuted into expert-contiguous rows and both expert
 * projections run as grouped bf16 GEMMs on the tensor cores (fp32 accumulate, bf16
 * activations between them); int8 stacks are dequantized to bf16 first with
 * int8_dequant_expert's bits. Needs hidden a multiple of 256. ids_out / wts_out (nullable)
 * receive the routing, bit-identical to uocr_moe_route. `workspace` must hold
 * uocr_moe_prefill_workspace_bytes(L, T) bytes (256-byte aligned; its first word is the
 * device status word: zero-fill it once). */
UOCR_API size_t uocr_moe_prefill_workspace_bytes(const uocr_moe_layer* L, int64_t T);
UOCR_API int uocr_moe_prefill(const uocr_moe_layer* L, const float* x, int64_t T, const float* bias,
                              float* out, int32_t* ids_out, float* wts_out,
                              void* workspace, size_t workspace_bytes, uocr_stream_t stream);

/* Expert-parallel pieces (no counterpart in the reference, which runs on one device; they serve
 * the expert-parallel prefill of configs[4]: tokens routed on their own GPU, rows exchanged with
 * NCCL all-to-all, experts computed where they live).
 *
 * uocr_moe_ep_experts: the routed experts of L (typically a slice of E_local experts) applied to
 * N received bf16 rows: out[n] = sum_s weight[n, s] * expert_{expert_local[n, s]}(rows[n]),
 * s < L->top_k, entries with expert_local < 0 skipped; expert products as in uocr_moe_prefill.
 * L's shared experts are not applied. */
UOCR_API size_t uocr_moe_ep_experts_workspace_bytes(const uocr_moe_layer* L, int64_t N);
UOCR_API int uocr_moe_ep_experts(const uocr_moe_layer* L, const uint16_t* rows, int64_t N,
                                 const int32_t* expert_local, const float* weight, float* out,
                                 void* workspace, size_t workspace_bytes, uocr_stream_t stream);

/* uocr_moe_ep_dispatch: the dispatch plan and row gather of T local tokens routed to ids/wts
 * [T, top_k] (global expert ids, id < 0 = none), for `world` <= 8 ranks with expert e held by rank
 * owner[e] as its local expert local[e] (device int32 [E]). One row per (token, rank holding at
 * least one of its experts), ordered by rank, then token (the row order of the torch bookkeeping
 * in ep.py, bit for bit). Outputs, device memory:
 *   send_counts int64 [world]      rows per destination rank;
 *   rows   bf16  [T * world, H]    x rounded to bf16 (nearest even), first sum(send_counts) used;
 *   meta   int32 [T * world, 2k]   per row the local expert of each slot (-1: another rank's or
 *                                  none), then the slot's routing weight as fp32 bits (0 for -1);
 *   inv    int32 [world, T]        row of (rank p, token t), -1 if t sends p nothing.
 * Two launches; no host synchronisation. */
UOCR_API size_t uocr_moe_ep_dispatch_workspace_bytes(int64_t T, int64_t world);
UOCR_API int uocr_moe_ep_dispatch(const float* x, int64_t T, int64_t H, const int32_t* ids, const float* wts,
                                  int64_t top_k, const int32_t* owner, const int32_t* local, int64_t E,
                                  int64_t world, int64_t* send_counts, uint16_t* rows, int32_t* meta,
                                  int32_t* inv, void* workspace, size_t workspace_bytes, uocr_stream_t stream);

/* uocr_moe_ep_combine: out[t] = (sum over ranks p ascending, from +0, of partials[inv[p, t]] for
 * inv >= 0) + add[t] (when add is not null): the partial rows come back in the dispatch's row
 * order; `add` is typically the shared experts' output. fp32 throughout. */
UOCR_API int uocr_moe_ep_combine(const float* partials, int64_t n_rows, const int32_t* inv, int64_t T,
                                 int64_t world, int64_t H, const float* add, float* out, uocr_stream_t stream);

/* ---- the expert-parallel exchange through peer memory (no counterpart in the reference) ----
 * What ExpertParallelMoE runs: no all-to-all and no host synchronisation. Every rank allocates one
 * exchange buffer of uocr_moe_ep_peer_buffer_bytes (zero-filled, 256-byte aligned, the same size on
 * every rank) and maps every other rank's into its process (uocr_ipc_export / uocr_ipc_import).
 * A forward on every rank, with the same increasing epoch:
 *   1. uocr_moe_ep_peer_dispatch: the plan of uocr_moe_ep_dispatch, but every (token, destination)
 *      row (bf16) and its slot metadata (local expert ids, weights) is stored straight into the
 *      destination's buffer, slot `rank`; then the row count and the epoch are published there.
 *      inv [world, T] receives each token's position in each destination's slot (-1: none).
 *   2. uocr_moe_ep_peer_experts: waits (bounded) for every source's rows of this epoch, applies L's
 *      routed experts (a slice of E_local experts, expert products as in uocr_moe_prefill) to the
 *      received rows, and stores each row's weighted sum as bf16 straight back into its source's
 *      buffer; then flags every source.
 *   3. uocr_moe_ep_peer_combine: waits (bounded) for every expert rank's flag of this epoch, then
 *      out[t] = (sum over ranks p ascending, from +0, of float(partial of (t, p))) + add[t].
 * A wait that gives up (a rank that never comes: 20 s), or a received count above cap_tokens, sets
 * the buffer's status (uocr_moe_device_status(buf[rank]) reports and clears it); the affected
 * sources are flagged and their outputs, and every output while the status is set, are NaN. */
#define UOCR_IPC_HANDLE_BYTES 64
typedef struct uocr_ep_peers {
    int32_t world;       /* ranks, 1..8 */
    int32_t rank;        /* this process's rank */
    int32_t cap_tokens;  /* tokens per rank the slots hold: at least every rank's T */
    int32_t hidden;      /* H, multiple of 256 */
    int32_t top_k;       /* k */
    int32_t reserved;
    uint64_t epoch;      /* this forward's number: 1, 2, ..., the same on every rank */
    void* buf[8];        /* rank p's exchange buffer as mapped in this process (buf[rank]: its own) */
} uocr_ep_peers;
UOCR_API size_t uocr_moe_ep_peer_buffer_bytes(int64_t world, int64_t cap_tokens, int64_t hidden, int64_t top_k);
UOCR_API size_t uocr_moe_ep_peer_workspace_bytes(const uocr_moe_layer* L, const uocr_ep_peers* P);
UOCR_API int uocr_moe_ep_peer_dispatch(const uocr_ep_peers* P, const float* x, int64_t T, const int32_t* ids,
                                       const float* wts, const int32_t* owner, const int32_t* local, int64_t E,
                                       int32_t* inv, void* workspace, size_t workspace_bytes, uocr_stream_t stream);
UOCR_API int uocr_moe_ep_peer_experts(const uocr_moe_layer* L, const uocr_ep_peers* P, void* workspace,
                                      size_t workspace_bytes, uocr_stream_t stream);
UOCR_API int uocr_moe_ep_peer_combine(const uocr_ep_peers* P, const int32_t* inv, int64_t T, const float* add,
                                      float* out, uocr_stream_t stream);
/* CUDA IPC for the exchange buffers: the handle (UOCR_IPC_HANDLE_BYTES) and offset of a device
 * pointer inside its allocation, and the mapping of another process's (current device; peer
 * access enabled on first use). Plain peer loads and stores only: no multicast object is made. */
UOCR_API int uocr_ipc_export(const void* dev_ptr, void* handle_out, uint64_t* offset_out);
UOCR_API int uocr_ipc_import(const void* handle, uint64_t offset, void** dev_ptr_out);
UOCR_API int uocr_ipc_close(void* dev_ptr, uint64_t offset);

/* The shared experts of L alone over x [T, H] fp32 (bf16 products, fp32 out): out = shared(x),
 * or out += shared(x) with accumulate != 0. Meant to run beside the expert-parallel exchanges:
 * its GEMMs leave 16 SMs free for concurrent kernels (NCCL's). */
UOCR_API size_t uocr_moe_shared_workspace_bytes(const uocr_moe_layer* L, int64_t T);
UOCR_API int uocr_moe_shared_forward(const uocr_moe_layer* L, const float* x, int64_t T, float* out,
                                     int accumulate, void* workspace, size_t workspace_bytes,
                                     uocr_stream_t stream);

/* Decode step without a caller workspace. No counterpart in the reference: added for callers
 * that cannot allocate device memory (a plugin host that passes an operator only its inputs
 * and outputs, or a runtime whose device memory is reserved up front). Same computation as
 * uocr_moe_decode; its scratch is a fixed array inside the library, of
 * uocr_moe_decode_noalloc_max_bytes() bytes (1 MiB) on every GPU that loads the library,
 * held until exit. Layers and batches needing more scratch are refused with UOCR_EINVAL.
 * Calls on one device share that array: calls that overlap on the GPU race. The first call
 * on a device looks up the array's address and should come before any stream capture. */
UOCR_API size_t uocr_moe_decode_noalloc_max_bytes(void);
UOCR_API int uocr_moe_decode_noalloc(const uocr_moe_layer* L, const float* x, int64_t B,
                                     const float* bias, float* out, uocr_stream_t stream);
/* The in-library array's status on the current device, as uocr_moe_device_status reports a
 * workspace's: synchronises `stream`, returns UOCR_OK, or UOCR_EDEVICE once after a call whose
 * device-side wait gave up (that call, and every call until this read, wrote NaN over its output),
 * and clears it. No counterpart in the reference. */
UOCR_API int uocr_moe_decode_noalloc_status(uocr_stream_t stream);

/* Diagnostics: record a per-CTA timeline of the work items of subsequent uocr_moe_decode
 * launches into `device_buffer` (zero-filled by the caller; per CTA two halves, gate/up items then
 * down items, per item 8 words: MMA warp wait start, data ready, MMAs issued and committed,
 * slot/rows, producer issue time, accumulator acquired (int8 items), MMAs issued, all in
 * global-timer ns; the last records of each half hold kernel-level events).
 * NULL turns recording off. Not thread-safe; for profiling only. No counterpart in the
 * reference (its profiler is server-level). */
UOCR_API int uocr_moe_decode_set_trace(void* device_buffer, size_t bytes);

/* Status of a decode or prefill workspace after the stream's work finished (synchronises
 * `stream`): UOCR_OK if every device-side bounded wait of the calls since the last read completed,
 * else UOCR_EDEVICE with the code in uocr_last_error(); reading clears it (and the control words
 * a failed call left behind). No counterpart in the reference, whose ops cannot time out. */
UOCR_API int uocr_moe_device_status(const void* workspace, uocr_stream_t stream);

/* Test hook (no counterpart in the reference): the down phase of the next decode launches waits,
 * per slot, for `extra` operand groups that are never written, so its bounded waits run out; used to
 * check that such a failure is reported (NaN output, UOCR_EDEVICE from the status read) and that
 * calls after the status read are correct. 0 turns it off. Not thread-safe; for tests only. */
UOCR_API int uocr_moe_test_wait_extra(int extra);

#ifdef __cplusplus
}
#endif

#endif /* UOCR_MOE_H */
