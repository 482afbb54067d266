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

// ---- mbarrier ------------------------------------------------------------------------------
UOCR_DEV void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
UOCR_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
UOCR_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

UOCR_DEV void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar)) : "memory");
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

// Whole-warp bounded wait (every lane calls it; the result is warp-uniform). Polls with a short
// sleep between tries so waiting warps leave the issue slots to the working ones; the global
// timer is read every 32 polls. `abort_flag` (optional) ends the wait early.
UOCR_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort_flag, uint32_t* status) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    uint64_t t0 = 0;
    for (uint32_t spin = 1;; ++spin) {
        __nanosleep(40);
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
UOCR_DEV uint32_t ld_acquire_gpu(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
UOCR_DEV void st_release_gpu(uint32_t* p, uint32_t v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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

// ---- named barriers (a subset of the CTA's warps) ----------------------------------------
UOCR_DEV void named_bar_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---- programmatic dependent launch ---------------------------------------------------------
UOCR_DEV void pdl_wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
UOCR_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace uocr
