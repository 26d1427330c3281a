// HBM read-bandwidth ceiling probe (probe_ceiling / read_kernel,
// src/voltattn.cu:64-78 and :935-957), re-derived for HBM3e: the reference's
// 256 MiB buffer streams in ~35 us on a B200, where launch overhead skews the
// figure, so the buffer is GiB-sized and two read engines are measured:
//   0: wide loads — each thread keeps four 16-byte non-allocating loads in
//      flight per iteration (grid = a multiple of the SM count);
//   1: bulk copies — one warp per CTA streams 32 KiB chunks into a 4-deep
//      shared-memory ring with cp.async.bulk (no multicast), never touching
//      the data in registers, so only DRAM -> SM delivery is measured.
#pragma once

#include "common.cuh"

namespace va {

__device__ __forceinline__ uint4 ld_stream_v4(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__global__ void __launch_bounds__(512) probe_vec_kernel(const uint4* __restrict__ src, size_t n16,
                                                        unsigned* __restrict__ sink) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint32_t acc = 0;
    for (; i + 3 * stride < n16; i += 4 * stride) {
        const uint4 a = ld_stream_v4(src + i);
        const uint4 b = ld_stream_v4(src + i + stride);
        const uint4 c = ld_stream_v4(src + i + 2 * stride);
        const uint4 d = ld_stream_v4(src + i + 3 * stride);
        acc ^= a.x ^ a.y ^ a.z ^ a.w ^ b.x ^ b.y ^ b.z ^ b.w ^ c.x ^ c.y ^ c.z ^ c.w ^ d.x ^ d.y ^ d.z ^ d.w;
    }
    for (; i < n16; i += stride) {
        const uint4 a = ld_stream_v4(src + i);
        acc ^= a.x ^ a.y ^ a.z ^ a.w;
    }
    if (acc == 0x9E3779B9u) sink[0] = acc;  // keeps the loads; the buffer is zero-filled
}

constexpr int kProbeChunk = 32 * 1024;
constexpr int kProbeStages = 4;

__global__ void __launch_bounds__(32) probe_bulk_kernel(const uint8_t* __restrict__ src, size_t nchunks,
                                                        unsigned* __restrict__ sink) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kProbeStages * kProbeChunk);
    if (threadIdx.x != 0) return;
    for (int s = 0; s < kProbeStages; ++s) mbar_init(&full[s], 1);
    fence_mbar_init();
    const uint64_t pol = l2_policy_evict_first();
    int k = 0;
    bool ok = true;
    for (size_t c = blockIdx.x; c < nchunks; c += gridDim.x, ++k) {
        const int stage = k % kProbeStages;
        if (k >= kProbeStages &&
            !mbar_wait_bounded(&full[stage], (uint32_t)((k - kProbeStages) / kProbeStages) & 1u)) {
            report_error(kErrFullWait);
            ok = false;
            break;
        }
        mbar_arrive_expect_tx(&full[stage], kProbeChunk);
        bulk_g2s(smem + (size_t)stage * kProbeChunk, src + c * kProbeChunk, kProbeChunk, &full[stage], pol);
    }
    // wait for the copies still in flight before the CTA exits
    for (int d = 1; d <= kProbeStages && k - d >= 0; ++d) {
        const int kk = k - d;
        if (!mbar_wait_bounded(&full[kk % kProbeStages], (uint32_t)(kk / kProbeStages) & 1u)) ok = false;
    }
    if (!ok) sink[1] = 1u;
}

}  // namespace va
