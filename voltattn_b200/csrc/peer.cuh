// Split-L exchange over NVLink peer memory (plain stores and flag words in
// buffers mapped into every rank's address space; no TMA, no multicast).
//
// Each rank holds a gather buffer [2][R][H][D+2] floats and flags [2][R][H]
// (double-buffered by epoch parity). For head h, a rank stores its partial
// (m, l, o[D]) into slot [par][rank][h] of every rank's buffer, publishes
// flag[par][rank][h] = epoch on every rank (system-scope release after a
// system fence), waits, bounded, until all R ranks' flags for h carry the
// epoch (system-scope acquire), and merges the R slots with the log-sum-exp
// of the reference's combine (src/voltattn.cu:651-672). A rank publishes
// epoch e+2 only after its merge of e+1 saw every peer's e+1, which each peer
// published after finishing its merge of e, so a parity half is never
// overwritten while it is read. A wait that runs out records kErrPeerWait
// and leaves the head's output untouched.
#pragma once

#include "common.cuh"

namespace va {

constexpr int kMaxRanks = 8;

struct PeerBuffers {
    float* gather[kMaxRanks];    // rank r's gather buffer [2][R][H][D+2]
    unsigned* flags[kMaxRanks];  // rank r's flags [2][R][H]
};

__device__ __forceinline__ void store_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned load_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The exchange of one head by nthr threads of a CTA: thread `tid` holds the
// dims d0 + j * dstride (j < J) of this rank's partial (m in natural-log
// units). `sync` synchronises the nthr threads; `shok` is a shared word;
// wait_ns bounds the wait for the peers' flags.
// Returns the merged output dims in o (normalised), false on a failed wait.
template <int J, class Sync>
__device__ __forceinline__ bool peer_exchange_head(const PeerBuffers& x, int R, int rank, unsigned epoch,
                                                   uint64_t wait_ns, int H, int D, int h, float m, float l,
                                                   float (&o)[J], int d0, int dstride, int tid, Sync sync,
                                                   volatile int* shok) {
    const int par = (int)(epoch & 1u);
    const size_t slot_f = (size_t)(D + 2);
    const size_t buf_f = (size_t)R * H * slot_f;
    for (int r = 0; r < R; ++r) {
        float* dst = x.gather[r] + par * buf_f + ((size_t)rank * H + h) * slot_f;
#pragma unroll
        for (int j = 0; j < J; ++j) dst[2 + d0 + j * dstride] = o[j];
        if (tid == 0) {
            dst[0] = m;
            dst[1] = l;
        }
    }
    if (tid == 0) *shok = 1;
    sync();  // every thread's stores are issued (and shok set)
    if (tid == 0) {
        __threadfence_system();
        for (int r = 0; r < R; ++r) store_release_sys(x.flags[r] + ((size_t)par * R + rank) * H + h, epoch);
    }
    if (tid < R) {
        const unsigned* f = x.flags[rank] + ((size_t)par * R + tid) * H + h;
        bool seen = load_acquire_sys(f) == epoch;
        if (!seen) {
            const uint64_t t0 = global_timer_ns();
            for (uint32_t i = 1; !seen; ++i) {
                seen = load_acquire_sys(f) == epoch;
                if (!seen && (i & 63u) == 0 && global_timer_ns() - t0 > wait_ns) break;
            }
        }
        if (!seen) {
            *shok = 0;
            report_error(kErrPeerWait);
        }
    }
    sync();
    if (!*shok) return false;
    const float* g = x.gather[rank] + par * buf_f;
    float ms = kNegMax;
    for (int r = 0; r < R; ++r) ms = fmaxf(ms, __ldcv(g + ((size_t)r * H + h) * slot_f));
    float ls = 0.f;
#pragma unroll
    for (int j = 0; j < J; ++j) o[j] = 0.f;
    for (int r = 0; r < R; ++r) {
        const float* sp = g + ((size_t)r * H + h) * slot_f;
        const float a = fast_exp2((__ldcv(sp) - ms) * kLog2e);
        ls = fmaf(__ldcv(sp + 1), a, ls);
#pragma unroll
        for (int j = 0; j < J; ++j) o[j] = fmaf(__ldcv(sp + 2 + d0 + j * dstride), a, o[j]);
    }
    const float inv = 1.f / ls;
#pragma unroll
    for (int j = 0; j < J; ++j) o[j] *= inv;
    return true;
}

}  // namespace va
