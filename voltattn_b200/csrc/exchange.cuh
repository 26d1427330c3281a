// Split-L partial exchange over NVLink peer memory, fused with the combine.
//
// After each GPU has decoded its range of the KV length into per-head
// partials (m, l, o[D]) (va_decode_partial), one CTA per head on every rank
// stores its head-h partial as epoch-tagged words into slot `rank` of every
// rank's gather buffer (peer pointers mapped into this process; plain 8-byte
// stores over NVLink, no TMA, no multicast), polls the R slots of its own
// buffer until every word carries the epoch, and merges them with the
// log-sum-exp of the reference's combine (src/voltattn.cu:651-672) into fp16
// out (the protocol: peer.cuh). A wait that runs out (a peer that never
// published) records a device error and leaves the head's output untouched.
#pragma once

#include "peer.cuh"

namespace va {

// One CTA of 128 threads per head; thread t holds dim t (D <= 128).
__global__ void __launch_bounds__(128) exchange_combine_kernel(const float* __restrict__ partial, int H, int D,
                                                               int R, int rank, PeerBuffers peers, unsigned epoch,
                                                               uint64_t wait_ns, __half* __restrict__ out) {
    const int h = blockIdx.x, tid = threadIdx.x;
    __shared__ int ok;
    const float* mine = partial + (size_t)h * (D + 2);
    float o[1] = {tid < D ? mine[2 + tid] : 0.f};
    if (peer_exchange_head<1>(peers, R, rank, epoch, wait_ns, H, D, h, mine[0], mine[1], o, tid, 128, tid,
                              [] { __syncthreads(); }, &ok) &&
        tid < D)
        out[(size_t)h * D + tid] = __float2half_rn(o[0]);
}

}  // namespace va
