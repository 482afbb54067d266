// Thin inline-PTX wrappers for the sm_100a features the kernels use: mbarriers, bulk async
// copies (TMA engine), tensor-map TMA loads, tcgen05 (TMEM alloc, MMA, commit, loads),
// global timer, and bounded waits that give up (status word) instead of hanging.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace uocr {

UOCR_DEV uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

UOCR_DEV uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Budget of every device-side wait: far above any legitimate wait of these kernels (tens of
// microseconds), far below a hang. After it the waiter records kStatusWaitTimeout and the
// kernel winds down without touching the data it was waiting for.
constexpr uint64_t kWaitBudgetNs = 200ull * 1000ull * 1000ull;
// Budget of a wait on another GPU's expert-parallel exchange: the ranks' hosts enqueue their work
// independently and may be far apart in time, so this is long; it only has to end a wait for a
// rank that never comes.
constexpr uint64_t kEpWaitBudgetNs = 20ull * 1000ull * 1000ull * 1000ull;

// ---- mbarrier ------------------------------------------------------------------------------
UOCR_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
UOCR_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
UOCR_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
UOCR_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
// Shared-memory words handed between the warps of a CTA: release stores and adds, acquire loads.
UOCR_DEV void st_release_cta_u32(uint32_t* p, uint32_t v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}
UOCR_DEV void st_release_cta_add(int* p, int v) {
    asm volatile("red.release.cta.shared::cta.add.s32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}
UOCR_DEV uint32_t ld_acquire_cta_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
    return v;
}

UOCR_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar)) : "memory");
}
UOCR_DEV void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
                 "r"(count)
                 : "memory");
}
UOCR_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
UOCR_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of `parity` to complete, at most kWaitBudgetNs. Returns false (and
// records the timeout) if it gave up.
UOCR_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            set_status(status, kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}

// Whole-warp bounded wait (every lane calls it; the result is warp-uniform). mbarrier.try_wait
// itself suspends the warp until the phase completes or a hardware time slice ends, so the
// loop does not sleep; the global timer is read every 32 polls. `abort_flag` (optional) ends
// the wait early.
UOCR_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint32_t* status) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    uint64_t t0 = 0;
    for (uint32_t spin = 1;; ++spin) {
        if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
        if ((spin & 31) == 0) {
            int give_up = 0;
            if ((threadIdx.x & 31) == 0) {
                const uint64_t now = global_timer_ns();
                if (t0 == 0) t0 = now;
                give_up = (abort_flag && *abort_flag) || (now - t0 > kWaitBudgetNs);
                if (give_up) set_status(status, kStatusWaitTimeout);
            }
            if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
        }
    }
}

// ---- bulk async copy global -> shared (no tensor map), completes on an mbarrier ----------
// dst, src 16-byte aligned; bytes a multiple of 16.
UOCR_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// The same with an L2 cache policy (createpolicy): streamed weights marked evict-first leave the
// L2 to the small data every step re-reads (activations, scratch rows, counters, kernel code).
UOCR_DEV uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
UOCR_DEV void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// ---- explicit shared-memory loads (32-bit shared addresses) --------------------------------
// The hot loops read their stages through these so every access is an LDS, never a generic load.
UOCR_DEV uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
UOCR_DEV uint2 lds_u64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
UOCR_DEV float lds_f32(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
UOCR_DEV float4 lds_f128(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}

// ---- global flags with gpu-scope ordering -------------------------------------------------
// Counter arrivals that publish this thread's earlier writes (and those ordered before them, e.g.
// by a __syncwarp): a release reduction, and an acquire-release add that also makes the other
// arrivals' writes visible to the caller.
UOCR_DEV void red_release_gpu_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
UOCR_DEV uint32_t atom_acq_rel_gpu_add(uint32_t* p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
UOCR_DEV uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
UOCR_DEV void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// ---- flags shared with other GPUs (peer memory over NVLink): system-scope ordering --------------
UOCR_DEV unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
UOCR_DEV void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spin until *p >= target (gpu-scope acquire), at most kWaitBudgetNs.
UOCR_DEV bool wait_counter_geq(const uint32_t* p, uint32_t target, uint32_t* status) {
    if (ld_acquire_gpu(p) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_gpu(p) < target) {
        __nanosleep(64);
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            set_status(status, kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}

// Spin until *p != old (gpu-scope acquire), at most kWaitBudgetNs.
UOCR_DEV bool wait_word_ne(const uint32_t* p, uint32_t old, uint32_t* status) {
    if (ld_acquire_gpu(p) != old) return true;
    const uint64_t t0 = global_timer_ns();
    while (ld_acquire_gpu(p) == old) {
        __nanosleep(32);
        if (global_timer_ns() - t0 > kWaitBudgetNs) {
            set_status(status, kStatusWaitTimeout);
            return false;
        }
    }
    return true;
}

// ---- named barriers (a subset of the CTA's warps) ----------------------------------------
UOCR_DEV void named_bar_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- TMA tensor loads (tensor map in kernel-parameter space) --------------------------------
// 2-D tile load: c0 is the innermost (contiguous) coordinate; c0 * element size must be a
// multiple of 16 bytes. Completes on `bar` with the tile's byte count.
UOCR_DEV void tma_load_2d(void* dst, const void* tmap, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(smem_addr(bar))
        : "memory");
}
UOCR_DEV void tma_load_4d(void* dst, const void* tmap, int c0, int c1, int c2, int c3, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}
UOCR_DEV void tma_prefetch_desc(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// ---- tcgen05: tensor memory, MMA, loads --------------------------------------------------------
// Allocate `ncols` (power of two >= 32) TMEM columns; the base address is written to smem.
// Executed by one full warp.
UOCR_DEV void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(smem_dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
UOCR_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
UOCR_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
UOCR_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate); one thread issues.
UOCR_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8 (signed 8-bit inputs, s32 accumulate); one thread issues.
UOCR_DEV void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once all previously issued MMAs of this thread have completed.
UOCR_DEV void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

// Shared-memory matrix descriptor for a K-major tile in the 128-byte-swizzle layout TMA
// writes (rows of 128 bytes, 8-row groups 1024 bytes apart): start >> 4 in bits 0-13, leading
// offset 1 (unused for swizzled K-major), stride offset 1024 >> 4 in bits 32-45, version 1 in
// bits 46-47, layout SWIZZLE_128B (2) in bits 61-63. The tile base is 1024-byte aligned.
UOCR_DEV uint64_t umma_desc_sw128(uint32_t smem_byte_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_byte_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1), B bf16
// (bits 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor, kind::i8: D s32 (bits 4-5 = 2), A and B signed 8-bit (bits 7-9, 10-12
// = 1), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
UOCR_DEV void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
UOCR_DEV void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
        "[%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
UOCR_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.wait::ld that also marks r[] as written by it, so no use of the loaded registers can be
// scheduled before the wait (needed when a later tcgen05.ld is issued before r[] is consumed)
UOCR_DEV void tmem_wait_ld_tie(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                   "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                   "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// ---- CTA pairs (clusters of 2) for tcgen05 cta_group::2 -------------------------------------
UOCR_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// every thread of both CTAs of the cluster: release own prior writes, acquire the peer's
UOCR_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the shared::cluster address of the object at own shared address `a` in CTA `rank`
UOCR_DEV uint32_t mapa_shared(uint32_t a, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    return r;
}
// arrive (release at cluster scope) on an mbarrier given by its shared::cluster address
UOCR_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile loads into own shared memory whose completion is counted on the pair leader's
// mbarrier (`mbar`: a shared::cluster address in CTA 0 of the pair)
UOCR_DEV void tma_load_2d_pair(void* dst, const void* tmap, int c0, int c1, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(mbar)
        : "memory");
}
UOCR_DEV void tma_load_4d_pair(void* dst, const void* tmap, int c0, int c1, int c2, int c3, uint32_t mbar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
        "%5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(mbar)
        : "memory");
}
// TMEM for a CTA pair: one warp of each CTA (the same warp index) allocates / frees the same
// columns in both CTAs' tensor memory
UOCR_DEV void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(smem_dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
UOCR_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair MMA, issued by one thread of CTA 0: D (M = 256: rows 0-127 in CTA 0's TMEM, 128-255 in
// CTA 1's) (+)= A (128 rows from each CTA's shared memory at the descriptor's address) x B (N/2
// rows from each CTA's shared memory)^T, kind::f16.
UOCR_DEV void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on own mbarrier `bar` once every pair MMA issued so far by this thread has completed.
UOCR_DEV void umma_commit_pair_own(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
// Arrive on the mbarrier at own shared address `bar` in both CTAs of the pair (mask 0b11) once
// every pair MMA issued so far by this thread has completed.
UOCR_DEV void umma_commit_pair_both(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
            smem_addr(bar))
        : "memory");
}

// ---- programmatic dependent launch ---------------------------------------------------------
UOCR_DEV void pdl_wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
UOCR_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace uocr
