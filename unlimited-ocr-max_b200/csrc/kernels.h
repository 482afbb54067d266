// Internal launch interface between capi.cu (argument checks, the C ABI) and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace uocr {

// shims.cu
void launch_bf16_qmv(float* out, const float* x, const int32_t* ids, const uint16_t* w, int rows, int E, int N,
                     int K, bool vec, cudaStream_t st);
void launch_int8_qmv(float* out, const float* x, const int32_t* ids, const int8_t* w, const float* scales, int rows,
                     int E, int N, int K, int groups, bool vec, cudaStream_t st);
void launch_int8_dequant(uint16_t* out, const int8_t* w, const float* scales, const int32_t* idx, int E, int N,
                         int K, int groups, cudaStream_t st);
void launch_dense_bf16_qmv(float* out, const float* x, const uint16_t* w, int M, int N, int K, bool vec,
                           cudaStream_t st);

// quant.cu: `groups` consecutive 128-element groups of w (bf16 or fp32) -> int8 q + one fp32 scale per
// group; *nonfinite |= 1 if any element is NaN or Inf. `vec`: w 16-byte and q 8-byte aligned.
cudaError_t launch_quantize_g128(const void* w, bool bf16, long long groups, int8_t* q, float* scales,
                                 int* nonfinite, bool vec, cudaStream_t st);

// dense.cu: dense bf16 projections of the decode step (M <= 8 rows per launch).
// Workspace: a control block of kCtlClearBytes (status word at [0], the split-K row-block counters
// from word kDenseCtlCounters), then the split-K partials [NB][KC][128][8] fp32 when KC > 1.
constexpr int kDenseMaxChunkItems = 12;  // K items (128 elements) of one CTA's x image
constexpr int kDenseMaxSplit = 8;        // K chunks of a row block whose partials one summing pass loads at once
constexpr int kDenseCtlCounters = 16;
struct DensePlan {
    int NB, IPR, KC, IPC, Gp, grid;  // row blocks, items per row block, K chunks, items per chunk, CTAs per chunk
};
DensePlan dense_plan(long long N, long long K, int sms);
cudaError_t launch_dense_pack(const uint16_t* w, bool kblocked, int N, int K, unsigned char* out, cudaStream_t st);
cudaError_t launch_dense_stream(const unsigned char* w, int N, int K, const float* x, int M, float* out,
                                uint32_t* ctl, float* partial, const DensePlan& p, cudaStream_t st);

// attention.cu: paged decode attention. Workspace: a control block of kCtlClearBytes (status word
// at [0], per-request counters from word kAttnCtlCounters), then the partials [B][S][heads][130]
// fp32 (S <= lut_cols x 32 CTAs per request).
constexpr int kAttnCtlCounters = 16;
int paged_attention_ctas(int B, int lut_cols, int sms);  // S: CTAs per request
cudaError_t launch_paged_decode_attention(const float* q, const float* k_new, const float* v_new, float* kv,
                                          int pages, int layers, int layer, const uint32_t* lut, int lut_cols,
                                          const uint32_t* write_index, const uint32_t* attend_len, float* out, int B,
                                          int heads, float scale, uint32_t* ctl, float* partial, int S,
                                          cudaStream_t st);

// rope.cu: RoPE on the fused q|k|v rows [B, 3 x heads x dim] -> q, k (rotated), v, each [B, heads, dim]
cudaError_t launch_rope_qkv(const float* qkv, int B, int heads, int dim, const float* cos, const float* sin, float* q,
                            float* k, float* v, cudaStream_t st);

// step.cu: the token embedding (bf16 table rows -> fp32, ids clamped) and the dense FFN's silu(g) * u
cudaError_t launch_embed_rows(const uint16_t* table, int V, int H, const int32_t* ids, int B, float* out,
                              cudaStream_t st);
cudaError_t launch_silu_mul(const float* gu, int B, int I, float* out, cudaStream_t st);

// ngram.cu: the no-repeat-n-gram guard on B rows of V logits (out may alias logits)
cudaError_t launch_ngram_block(const float* logits, int B, int V, const int32_t* history, int H, const int32_t* ngram,
                               float* out, bool vec, cudaStream_t st);

// norm.cu: h += add (if add), then y = RMSNorm(h) * gamma (if y), one CTA per row
cudaError_t launch_residual_rmsnorm(float* h, const float* add, const float* gamma, int B, int H, float eps, float* y,
                                    cudaStream_t st);

// route.cu
cudaError_t launch_route(const float* x, int T, int H, const uint16_t* wg, int E, const float* bias, int topk,
                         int32_t* ids, float* wts, cudaStream_t st);

// decode.cu
// Control block at the start of a decode workspace, zero-filled once by the caller.
//   status     sticky: the code of the first device-side failure of any call on this workspace,
//              until the host reads and clears it (uocr_moe_device_status, which also zeroes the
//              rest of this block). While it is set, every call writes NaN and touches no counter.
//   call_fail  this call failed somewhere (set before the failing CTA counts its remaining units).
//   hdone[s]   calls with B < 8 (int8) or B < 4 (bf16): gate/up units of slot s finished (4 epilogue
//              warps each: 4 * I/64 per slot); the down phase's stagers then turn the slot's h rows
//              into its operand themselves.
//   gcnt[s][g] the other calls: gate/up arrivals for the 128-group g of slot s's h columns
//              (4 epilogue warps x the group's 2 units); the arrival that completes it hands the
//              group to its CTA's image warp, which writes the group's down-operand image (int8
//              digits and scales, or bf16 terms) and counts it on imgdone[s] (I/128 per slot when
//              done). The down phase copies such a slot's image in bulk.
//   ydone[rb]  down units of output column block rb finished (4 per unit, 4 * slots in all): the
//              arrival that completes a block has its CTA combine it (or write it NaN).
//   cdone      combined column blocks (4 per block); the last resets hdone, gcnt, imgdone, call_fail and
//              itself, so every call starts from zero (ydone[rb] is reset by the block's completing
//              arrival).
constexpr int kDecodeMaxGroups = 16;  // 128-element groups of the intermediate size (I <= 2048)
// floats per row of the decode digit scales (the 128-groups of I, rounded up to 16 bytes)
__host__ __device__ inline int decode_sig_stride(int I) { return ((I / 128 + 3) / 4) * 4; }
struct DecodeCtl {
    uint32_t status;
    uint32_t call_fail;
    uint32_t cdone;
    uint32_t pad0[5];
    uint32_t hdone[72];                       // per slot (small batches): gate/up arrivals (4 per unit)
    uint32_t imgdone[72];                     // per slot (B = 8; bf16 from B = 4): its written 128-group images
    uint32_t ydone[64];                       // per output column block: down units written
    uint32_t gcnt[72 * kDecodeMaxGroups];     // per slot and 128-group (same calls): gate/up arrivals
    uint32_t pad1[2048 - 8 - 72 - 72 - 64 - 72 * kDecodeMaxGroups];
};
// Bytes at the start of a workspace the host clears along with its status word: the whole decode
// control block; prefill and exchange workspaces keep their status word at the start of a status
// region of the same size.
constexpr size_t kCtlClearBytes = 8192;
static_assert(sizeof(DecodeCtl) == kCtlClearBytes, "the decode control block is the cleared region");
constexpr int kDecodeMaxShared = 8;
constexpr int kDecodeMaxTopk = 8;

struct DecodeArgs {
    int B, H, I, E, S, topk, G, int8;
    const float* x;
    const uint16_t* router;
    const float* bias;
    int32_t* ids;
    float* wts;
    const void* w13;   // packed blocks (layout.h), int8 scales inline
    const void* w2;
    const uint16_t* w13_shared;
    const uint16_t* w2_shared;
    float* h;       // [(k+S)*B, I], slot-contiguous rows (shared slot q: rows qB..qB+B-1, routed slots after)
    float* y;       // [(k+S)*B, H], slot-contiguous rows
    // The down operand of each slot, written once per call during the gate/up phase: the slot's
    // image region starts at byte base * I * 4 (base = its first row); int8 slots hold I / 128
    // groups of 3c rows x 128 B (c = the slot's entries), bf16 slots I / 64 atoms of 2c rows x
    // 128 B, rows as in shared memory (decode.cu: put_digits, put_terms)
    unsigned char* himg;
    float* gsig;    // [(k+S)*B, decode_sig_stride(I)]: digit scales of the int8 slots' rows per 128-group
    float* out;     // [B, H]
    DecodeCtl* ctl;
    float* logits;       // [8][64][8] router logit partials (token, expert, segment)
    unsigned char* xd;   // [H / 128][32 rows][128 B]: x as int8 digit planes, the MMA B operand image (K1 -> K2)
    unsigned char* xb;   // [H / 64][16 rows][128 B]: x as two bf16 terms, the MMA B operand image
    float* xsig;         // [8][H / 128] scales of the digit groups
    unsigned long long* trace;  // optional per-CTA item timeline (diagnostics), null = off
    int trace_items;            // items recorded per CTA
    int hold_extra;             // test hook: the down phase waits for this many more operand groups per slot
};
// diagnostics: the trace buffer the next decode launches record into (capi.cu)
extern unsigned long long* g_decode_trace;
extern size_t g_decode_trace_bytes;
// test hook: operand groups per slot the next decode launches' down phase waits for on top of the
// real ones (capi.cu)
extern int g_decode_wait_extra;
cudaError_t launch_decode_layer(const DecodeArgs& a, cudaStream_t st);

// prefill.cu
constexpr int kPrefillMaxGroups = 64 + kDecodeMaxShared;

// One GEMM group: `rows` consecutive rows of A from `a_base`, written to output rows from
// `out_base`, against weight stack `wrow0` of the routed (shared == 0) or shared weights.
struct PrefillGroup {
    int a_base, out_base, rows, wrow0, shared;
};
// The groups with at least one row, and the prefix of their 128-row M tiles.
struct PrefillPlan {
    int ngroups;
    int pad[3];
    int mtile_prefix[kPrefillMaxGroups + 1];
    PrefillGroup g[kPrefillMaxGroups];
};

struct EpPeers;  // ep.cu

struct PrefillArgs {
    int T, H, I, E, S, topk, G, int8;
    int route;       // 1: route x here (ids/wts are outputs); 0: ids/wts given, id < 0 = no expert
    int use_shared;  // add the S shared experts
    int accumulate;  // out += instead of out =
    int max_ctas;    // 0: the GEMMs take one CTA per SM; > 0: at most this many (SMs left to concurrent kernels)
    const float* x;  // [T, H] fp32 (or null with x_bf16)
    const uint16_t* x_bf16;  // [T, H] bf16 rows given directly (or null)
    const uint16_t* router;
    const float* bias;
    int32_t* ids;  // [T, topk]
    float* wts;    // [T, topk]
    const void* w13;
    const void* w2;
    const uint16_t* w13_shared;
    const uint16_t* w2_shared;
    float* out;  // [T, H]
    // expert-parallel peer mode (null peers: off): rows [q cap, q cap + slot_counts[q]) of the T = world
    // cap rows are valid, the others skipped; instead of `out`, row q cap + r goes as bf16 to rank q's
    // partial slot `rank`, row r, and each rank q's part_flag[rank] is set once all rows are stored
    const EpPeers* peers;
    const int* slot_counts;
    const int* slot_fail;
    unsigned int* done;    // local zero word, last-CTA detection of the partials kernel
    uint32_t* status;      // null: the workspace's own status word
};
// Byte offsets of the prefill workspace regions (status word first).
struct PrefillLayout {
    size_t status, n_valid, ids, wts, chunk_counts, chunk_base, plan1, plan2, dest, src_tok, xperm, h, y, w13, w2, total;
};
PrefillLayout prefill_layout(int T, int H, int I, int E, int S, int topk, bool int8);
cudaError_t launch_prefill(const PrefillArgs& a, char* ws, const PrefillLayout& d, cudaStream_t st);

// ep.cu: expert-parallel dispatch plan + bf16 row gather, and the combine of partial rows
constexpr int kEpMaxWorld = 8;
size_t ep_dispatch_workspace_bytes(int T, int world);
cudaError_t launch_ep_dispatch(const float* x, int T, int H, const int32_t* ids, const float* wts, int k,
                               const int32_t* owner, const int32_t* local, int E, int world, long long* send_counts,
                               uint16_t* rows, int32_t* meta, int32_t* inv, void* ws, cudaStream_t st);
cudaError_t launch_ep_combine(const float* part, long long nrows, const int32_t* inv, int T, int world, int H,
                              const float* add, float* out, cudaStream_t st);

// ep.cu: the exchange through peer memory. Every rank holds one exchange buffer of the same layout,
// mapped into every other rank's process (CUDA IPC); a source rank stores its rows and slot
// metadata straight into its slot of each destination's buffer, an expert rank stores the partial
// rows straight back into its slot of each source's buffer, and per-source flags (the forward's
// epoch, written with system-scope release after the data) order the two sides. No host
// synchronisation, no intermediate copies.
struct EpSig {  // per source rank q, in the destination's buffer (64 bytes)
    unsigned long long disp_epoch;  // q's rows / metadata of this epoch are in slot q
    unsigned long long disp_count;  // rows q sent here this epoch
    unsigned long long part_flag;   // (epoch << 1) | fail: q's partial rows for this rank's slot-q rows
    unsigned long long pad[5];
};
struct EpPeerLayout {
    size_t status, sig, eid, w, rows, part, total;
};
EpPeerLayout ep_peer_layout(int world, int cap, int H, int k);
struct EpPeers {
    int world, rank, cap, H, k, pad;
    unsigned long long epoch;
    unsigned char* buf[kEpMaxWorld];  // rank p's exchange buffer as mapped in this process
};
// Local scratch of the peer path: a header (counters, slot counts), the dispatch plan, then the
// expert products of up to world * cap received rows (prefill layout).
struct EpPeerScratch {
    size_t hdr, masks, chunk_counts, order, send_counts, prefill, total;
};
constexpr size_t kEpHdrDoneDispatch = 0, kEpHdrDonePart = 4, kEpHdrSlotCounts = 32, kEpHdrSlotFail = 64;
EpPeerScratch ep_peer_scratch(int world, int cap, int H, int I, int E, int k, bool int8, size_t prefill_bytes);
cudaError_t launch_ep_peer_dispatch(const EpPeers& P, const float* x, int T, const int32_t* ids, const float* wts,
                                    const int32_t* owner, const int32_t* local, int E, int32_t* inv, char* ws,
                                    const EpPeerScratch& d, cudaStream_t st);
// wait for every source's dispatch of this epoch; slot counts and per-slot failures into the header
cudaError_t launch_ep_peer_wait(const EpPeers& P, char* ws, const EpPeerScratch& d, cudaStream_t st);
cudaError_t launch_ep_peer_combine(const EpPeers& P, const int32_t* inv, int T, const float* add, float* out,
                                   cudaStream_t st);

// pack.cu: source rows at (e * estride + row * ld) elements
cudaError_t launch_pack_w13(const void* gate, const void* up, const float* gs, const float* us, int E, int I, int H,
                            bool int8, long estride, long ld, void* out, cudaStream_t st);
cudaError_t launch_pack_w2(const void* down, const float* ds, int E, int H, int I, bool int8, long estride, long ld,
                           void* out, cudaStream_t st);
cudaError_t launch_pack_shared(const uint16_t* gate, const uint16_t* up, const uint16_t* down, long S, long I, long H,
                               uint16_t* w13, uint16_t* w2, cudaStream_t st);

}  // namespace uocr
