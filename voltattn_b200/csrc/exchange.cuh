// Split-L partial exchange over NVLink peer memory, fused with the combine.
//
// After each GPU has decoded its range of the KV length into per-head
// partials (m, l, o[D]) (va_decode_partial), one CTA per head on every rank:
//   1. stores its own head-h partial into slot `rank` of every rank's gather
//      buffer (peer pointers mapped into this process; plain stores over
//      NVLink, no TMA, no multicast),
//   2. publishes flag[rank][h] = epoch on every rank (system-scope release
//      after a system fence),
//   3. waits, bounded, until all R ranks' flags for head h carry the epoch
//      (system-scope acquire), then merges the R slots with the log-sum-exp
//      of the reference's combine (src/voltattn.cu:651-672) into fp16 out.
// The gather buffer and flags are double-buffered by epoch parity: a rank can
// only publish epoch e+2 after its combine of e+1 saw every peer's e+1, which
// each peer published after finishing its combine of e.
// A wait that runs out (a peer that never published) records a device error
// and leaves the head's output untouched.
#pragma once

#include "peer.cuh"

namespace va {

__global__ void __launch_bounds__(128) exchange_combine_kernel(const float* __restrict__ partial, int H, int D,
                                                               int R, int rank, PeerBuffers peers, unsigned epoch,
                                                               uint64_t wait_ns, __half* __restrict__ out) {
    const int h = blockIdx.x, tid = threadIdx.x;
    const int par = (int)(epoch & 1u);
    const size_t slot_f = (size_t)(D + 2);
    const size_t buf_f = (size_t)R * H * slot_f;  // floats per parity half
    const float* mine = partial + (size_t)h * slot_f;
    for (int r = 0; r < R; ++r) {
        float* dst = peers.gather[r] + par * buf_f + ((size_t)rank * H + h) * slot_f;
        for (int i = tid; i < D + 2; i += blockDim.x) dst[i] = mine[i];
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence_system();
        for (int r = 0; r < R; ++r) store_release_sys(peers.flags[r] + ((size_t)par * R + rank) * H + h, epoch);
    }
    // wait for every rank's head-h partial of this epoch
    __shared__ int ok;
    if (tid == 0) ok = 1;
    __syncthreads();
    if (tid < R) {
        const unsigned* f = peers.flags[rank] + ((size_t)par * R + tid) * H + h;
        bool seen = load_acquire_sys(f) == epoch;
        if (!seen) {
            const uint64_t t0 = global_timer_ns();
            for (uint32_t i = 1; !seen; ++i) {
                seen = load_acquire_sys(f) == epoch;
                if (!seen && (i & 63u) == 0 && global_timer_ns() - t0 > wait_ns) break;
            }
        }
        if (!seen) {
            ok = 0;
            report_error(kErrPeerWait);
        }
    }
    __syncthreads();
    if (!ok) return;
    const float* g = peers.gather[rank] + par * buf_f;
    float ms = kNegMax;
    for (int r = 0; r < R; ++r) ms = fmaxf(ms, __ldcv(g + ((size_t)r * H + h) * slot_f));
    float ls = 0.f;
    for (int r = 0; r < R; ++r) {
        const float* sp = g + ((size_t)r * H + h) * slot_f;
        ls += __ldcv(sp + 1) * fast_exp2((__ldcv(sp) - ms) * kLog2e);
    }
    for (int d = tid; d < D; d += blockDim.x) {
        float od = 0.f;
        for (int r = 0; r < R; ++r) {
            const float* sp = g + ((size_t)r * H + h) * slot_f;
            od += __ldcv(sp + 2 + d) * fast_exp2((__ldcv(sp) - ms) * kLog2e);
        }
        out[(size_t)h * D + d] = __float2half_rn(od / ls);
    }
}

}  // namespace va
