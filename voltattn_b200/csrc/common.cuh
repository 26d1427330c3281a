// Shared device helpers for the sm_100a kernels: shared-memory addresses,
// mbarrier and bulk-copy PTX, bounded waits, the device error word.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace va {

constexpr int kGroup = 64;  // quant group along D (reference src/voltattn.cu:60)

// Device error codes written to g_device_error (first writer wins).
enum DeviceError : int {
    kErrNone = 0,
    kErrFullWait = 1,   // consumer gave up waiting for a stage to land
    kErrEmptyWait = 2,  // producer gave up waiting for a stage to drain
    kErrDrainWait = 3,  // producer gave up waiting for its in-flight copies
    kErrPeerWait = 4,   // split-L exchange gave up waiting for a peer's partial
};

// Wall-clock budget of every spin wait: ~1 s, then the kernel reports an error
// and returns instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 1000000000ull;

// Device error word of this library, defined once (host_util.cu); the
// library is built with relocatable device code so every kernel writes it.
extern __device__ int g_device_error;

__device__ __forceinline__ void report_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---- mbarrier -------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// try_wait suspends the thread until the phase completes or the time hint
// (here 20 us) runs out, so a waiting warp takes no issue slots from the
// warps that compute.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete; false after
// kWaitLimitNs of wall time (the caller reports and bails out).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 7u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// The same wait without the suspend-time hint, for a thread on the critical
// path of a hand-off: with the hint a wait took ~200 cycles even on a
// completed phase (measured on the prefill's issue threads).
__device__ __forceinline__ bool mbar_wait_fast(uint64_t* bar, uint32_t parity) {
    const auto try_once = [&]() {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(smem_u32(bar)), "r"(parity)
            : "memory");
        return ok != 0;
    };
    if (try_once()) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (try_once()) return true;
        if ((i & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

// ---- bulk asynchronous copy (non-tensor TMA), global -> this CTA's smem ----
// Both addresses 16-byte aligned, bytes a multiple of 16. No multicast.

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Brings a kernel-parameter tensor map into the descriptor cache ahead of its
// first tensor copy.
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- named barriers (subset of the CTA's warps) ---------------------------

__device__ __forceinline__ void named_barrier_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Ticket for "the last one finishes the job": a gpu-scope acquire-release
// add by one thread. Callers bracket it with a CTA barrier: the barrier orders
// the other threads' slot writes before the release (cumulativity), and the
// acquire orders the readers after the next barrier behind every earlier
// release on the same counter. One thread fences instead of all of them.
__device__ __forceinline__ unsigned atomic_add_acq_rel_gpu(unsigned* p, unsigned v) {
    unsigned old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

__device__ __forceinline__ void store_relaxed_gpu(unsigned* p, unsigned v) {
    asm volatile("st.relaxed.gpu.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Programmatic dependent launch. wait: block until the preceding grid in the
// stream has completed and its memory is visible (returns at once when the
// launch was not programmatic); launch_dependents: allow the next grid, if
// launched programmatically, to start its prologue.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- misc -----------------------------------------------------------------

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kNegMax = -3.402823466e38f;  // -FLT_MAX: an empty partial's m

}  // namespace va
