// Staged streaming decode kernel (the "+" formats: f16+, q8+, q4+, q3+).
//
// Same math as the reference's sub-warp kernels (src/voltattn.cu:364-649):
// per head, score_j = q.K_j/sqrt(D), online softmax, o = sum_j p_j V_j, with
// K/V dequantized in registers and fp32 accumulation. The B200 structure is
// new:
//   * persistent CTAs walk work units (head, split) = (h, s); a producer warp
//     streams each unit's rows as tiles of TR rows through a STAGES-deep ring
//     of shared-memory buffers with bulk asynchronous copies (cp.async.bulk,
//     no multicast) completing on mbarriers, so tens of KB per SM are in
//     flight without holding registers;
//   * tiles start on global row multiples of 8, which makes every copy of
//     codes and scales 16-byte aligned and a multiple of 16 bytes for all
//     formats and D in {64,128}; rows of neighbouring units that a tile
//     covers are read but masked; the last (<8) rows of the whole tensor,
//     which a 16-byte copy could overrun, are fetched with plain loads;
//   * 8 consumer warps split each tile; a warp runs 32/LPR independent
//     softmax chains (LPR lanes per row), each chain takes RPS rows per tile
//     with one max/rescale per batch;
//   * the unit's chains merge in registers (shuffles) then shared memory into
//     one (m, l, o[D]) workspace slot (layout of src/voltattn.cu:92-93); the
//     last CTA to finish a head (atomic ticket, no waiting) merges the head's
//     S slots and writes the fp16 output — the reference's separate combine
//     launch (src/voltattn.cu:651-672) is fused away.
// Every spin wait is bounded (kWaitLimitNs); on expiry the kernel records a
// device error and returns.
#pragma once

#include "formats.cuh"

namespace va {

enum OutMode : int {
    kOutHalf = 0,     // fused combine -> fp16 out[H][D]
    kOutPartial = 1,  // fused combine -> fp32 partial[H][D+2]
    kOutSlots = 2,    // no fused combine: slots only (caller launches combine)
};

struct DecodeParams {
    const uint8_t* K;
    const uint8_t* V;
    const __half* scK;
    const __half* scV;
    const __half* q;
    __half* out;
    float* partial;
    float* ws;
    unsigned* counters;
    int H, L, S;
    int chunk;            // positions per split (multiple of 8)
    long long total_rows; // H * L
    int out_mode;
};

template <Kind K, int D>
struct StreamCfg {
    static constexpr Kind kKind = K;
    static constexpr int kD = D;
    static constexpr int kBits = KindTraits<K>::kBits;
    static constexpr int kDpl = KindTraits<K>::kDpl;
    static constexpr int kLpr = D / kDpl;           // lanes per row
    static constexpr int kNsg = 32 / kLpr;          // chains (sub-groups) per warp
    static constexpr int kRps = (K == Kind::F16) ? 2 : 4;  // rows per chain per tile
    static constexpr int kWarps = 8;                // consumer warps
    static constexpr int kThreads = (kWarps + 1) * 32;
    static constexpr int kTr = kWarps * kNsg * kRps;  // rows per tile
    static constexpr int kRb = D * kBits / 8;         // code bytes per row
    static constexpr int kSb = (K == Kind::F16) ? 0 : 2 * (D / kGroup);  // scale bytes per row
    static constexpr int kBpl = kDpl * kBits / 8;     // code bytes per lane
    static constexpr int kStages = 3;
    static constexpr int kStageBytes = 2 * kTr * kRb + 2 * kTr * kSb;
    static constexpr int kMergeBytes = (kWarps * (D + 2)) * 4 + 16;
    static constexpr int kSmemBytes = kStages * kStageBytes + 2 * kStages * 8 + kMergeBytes;
    static_assert(kTr % 8 == 0, "tiles must be whole 8-row blocks");
    static_assert((kTr * kRb) % 16 == 0 && (kTr * kSb) % 16 == 0, "16-byte stage sections");
    static_assert(kDpl <= kGroup, "a lane's dims must lie in one quant group");
};

struct UnitGeom {
    int h, s;
    long long r0, r1;  // unit's global rows [r0, r1)
    long long a0;      // first tile's first row (r0 rounded down to 8)
    int ntiles;
};

template <class C>
__device__ __forceinline__ UnitGeom unit_geom(const DecodeParams& p, int u) {
    UnitGeom g;
    g.h = u / p.S;
    g.s = u - g.h * p.S;
    const long long j0 = min((long long)p.L, (long long)g.s * p.chunk);
    const long long j1 = min((long long)p.L, j0 + p.chunk);
    g.r0 = (long long)g.h * p.L + j0;
    g.r1 = (long long)g.h * p.L + j1;
    g.a0 = g.r0 & ~7ll;
    g.ntiles = (g.r1 > g.r0) ? (int)((g.r1 - g.a0 + C::kTr - 1) / C::kTr) : 0;
    return g;
}

// ---- producer warp ----------------------------------------------------------

template <class C>
__device__ void stream_producer(const DecodeParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol = l2_policy_evict_first();
    const long long nr8 = p.total_rows & ~7ll;
    const int nunits = p.H * p.S;
    int k = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
        const UnitGeom g = unit_geom<C>(p, u);
        const long long cend = min((g.r1 + 7) & ~7ll, nr8);
        for (int t = 0; t < g.ntiles; ++t, ++k) {
            const int stage = k % C::kStages;
            const uint32_t ph = (uint32_t)(k / C::kStages) & 1u;
            if (!mbar_wait_bounded(&empty[stage], ph ^ 1u)) {
                if (lane == 0) report_error(kErrEmptyWait);
                // drain: wait (bounded) for copies this warp may still have in flight
                for (int d = 1; d <= C::kStages && k - d >= 0; ++d) {
                    const int kk = k - d;
                    mbar_wait_bounded(&full[kk % C::kStages], (uint32_t)(kk / C::kStages) & 1u);
                }
                return;
            }
            uint8_t* sK = smem + (size_t)stage * C::kStageBytes;
            uint8_t* sV = sK + C::kTr * C::kRb;
            uint8_t* sSK = sV + C::kTr * C::kRb;
            uint8_t* sSV = sSK + C::kTr * C::kSb;
            const long long t0 = g.a0 + (long long)t * C::kTr;
            const long long tend = t0 + C::kTr;
            const int brows = (int)max(0ll, min(tend, cend) - t0);
            const long long rg0 = max(t0, nr8), rg1 = min(tend, g.r1);
            if (rg1 > rg0) {
                // tail rows of the whole tensor: plain 8-byte / 2-byte loads
                const int rrows = (int)(rg1 - rg0);
                const int off = (int)(rg0 - t0);
                constexpr int kW8 = C::kRb / 8;
                for (int i = lane; i < rrows * kW8; i += 32) {
                    const int r = i / kW8, w = i % kW8;
                    const size_t src = (size_t)(rg0 + r) * C::kRb + (size_t)w * 8;
                    reinterpret_cast<uint2*>(sK + (size_t)(off + r) * C::kRb)[w] =
                        *reinterpret_cast<const uint2*>(p.K + src);
                    reinterpret_cast<uint2*>(sV + (size_t)(off + r) * C::kRb)[w] =
                        *reinterpret_cast<const uint2*>(p.V + src);
                }
                if constexpr (C::kSb > 0) {
                    constexpr int kG = C::kSb / 2;
                    for (int i = lane; i < rrows * kG; i += 32) {
                        const int r = i / kG, w = i % kG;
                        reinterpret_cast<__half*>(sSK)[(off + r) * kG + w] = p.scK[(size_t)(rg0 + r) * kG + w];
                        reinterpret_cast<__half*>(sSV)[(off + r) * kG + w] = p.scV[(size_t)(rg0 + r) * kG + w];
                    }
                }
                fence_proxy_async_smem();
                __syncwarp();
            }
            if (lane == 0) {
                const uint32_t bytes = (uint32_t)brows * (2u * C::kRb + 2u * C::kSb);
                mbar_arrive_expect_tx(&full[stage], bytes);
                if (brows > 0) {
                    bulk_g2s(sK, p.K + (size_t)t0 * C::kRb, (uint32_t)brows * C::kRb, &full[stage], pol);
                    bulk_g2s(sV, p.V + (size_t)t0 * C::kRb, (uint32_t)brows * C::kRb, &full[stage], pol);
                    if constexpr (C::kSb > 0) {
                        bulk_g2s(sSK, reinterpret_cast<const uint8_t*>(p.scK) + (size_t)t0 * C::kSb,
                                 (uint32_t)brows * C::kSb, &full[stage], pol);
                        bulk_g2s(sSV, reinterpret_cast<const uint8_t*>(p.scV) + (size_t)t0 * C::kSb,
                                 (uint32_t)brows * C::kSb, &full[stage], pol);
                    }
                }
            }
            __syncwarp();
        }
    }
}

// ---- consumer warps ---------------------------------------------------------

template <class C, bool kMasked>
__device__ __forceinline__ void consume_tile(const uint8_t* stage_base, int warp, int sg, int sl, long long t0,
                                             long long r0, long long r1, const float* qf, float& m, float& l,
                                             float* o) {
    const uint8_t* sK = stage_base;
    const uint8_t* sV = sK + C::kTr * C::kRb;
    const __half* sSK = reinterpret_cast<const __half*>(sV + C::kTr * C::kRb);
    const __half* sSV = sSK + C::kTr * (C::kSb / 2);
    constexpr int kG = C::kSb / 2;
    const int g = (sl * C::kDpl) / kGroup;

    float s[C::kRps];
    bool valid[C::kRps];
#pragma unroll
    for (int i = 0; i < C::kRps; ++i) {
        const int lr = (warp * C::kRps + i) * C::kNsg + sg;  // tile-local row
        valid[i] = true;
        if constexpr (kMasked) {
            const long long r = t0 + lr;
            valid[i] = (r >= r0) && (r < r1);
        }
        LaneRaw<C::kKind> kr;
        load_lane<C::kKind>(kr, sK + (size_t)lr * C::kRb + sl * C::kBpl);
        float acc = lane_dot<C::kKind>(kr, qf, 0.f);
        if constexpr (C::kKind != Kind::F16) acc *= __half2float(sSK[lr * kG + g]);
#pragma unroll
        for (int off = C::kLpr / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        s[i] = valid[i] ? acc : -INFINITY;
    }
    float mnew = m;
#pragma unroll
    for (int i = 0; i < C::kRps; ++i) mnew = fmaxf(mnew, s[i]);
    const float c = fast_exp2(m - mnew);
    m = mnew;
    l *= c;
#pragma unroll
    for (int d = 0; d < C::kDpl; ++d) o[d] *= c;
#pragma unroll
    for (int i = 0; i < C::kRps; ++i) {
        const int lr = (warp * C::kRps + i) * C::kNsg + sg;
        const float e = fast_exp2(s[i] - mnew);
        l += e;
        float w = e;
        if constexpr (C::kKind != Kind::F16) w *= __half2float(sSV[lr * kG + g]);
        LaneRaw<C::kKind> vr;
        load_lane<C::kKind>(vr, sV + (size_t)lr * C::kRb + sl * C::kBpl);
        if constexpr (kMasked) {
            if (!valid[i]) {
                w = 0.f;
                zero_lane<C::kKind>(vr);
            }
        }
        lane_axpy<C::kKind>(vr, w, o);
    }
}

template <class C>
__device__ __forceinline__ void merge_chains_in_warp(float& m, float& l, float* o) {
#pragma unroll
    for (int off = C::kLpr; off < 32; off <<= 1) {
        const float mo = __shfl_xor_sync(0xffffffffu, m, off);
        const float lo = __shfl_xor_sync(0xffffffffu, l, off);
        const float ms = fmaxf(m, mo);
        const float a = fast_exp2(m - ms), b = fast_exp2(mo - ms);
        l = l * a + lo * b;
#pragma unroll
        for (int d = 0; d < C::kDpl; ++d) o[d] = o[d] * a + __shfl_xor_sync(0xffffffffu, o[d], off) * b;
        m = ms;
    }
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, 2) decode_stream_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int D = C::kD;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
    uint64_t* empty = full + C::kStages;
    float* shM = reinterpret_cast<float*>(empty + C::kStages);
    float* shL = shM + C::kWarps;
    float* shO = shL + C::kWarps;
    int* shTicket = reinterpret_cast<int*>(shO + C::kWarps * D);
    volatile int* shFail = shTicket + 1;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::kWarps);
        }
        *shFail = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == C::kWarps) {
        stream_producer<C>(p, smem, full, empty);
        return;
    }

    constexpr int kConsumerThreads = C::kWarps * 32;
    const int sg = lane / C::kLpr, sl = lane % C::kLpr;
    const int nunits = p.H * p.S;
    // q scaled by log2(e)/sqrt(D): scores come out in log2 units for exp2
    const float qscale = rsqrtf((float)D) * kLog2e;
    float qf[C::kDpl];
    int cur_h = -1;
    int k = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x) {
        bool failed = false;
        const UnitGeom g = unit_geom<C>(p, u);
        if (g.h != cur_h) {
            const __half* qh = p.q + (size_t)g.h * D + sl * C::kDpl;
#pragma unroll
            for (int d = 0; d < C::kDpl; ++d) qf[d] = __half2float(qh[d]) * qscale;
            cur_h = g.h;
        }
        float m = kNegMax, l = 0.f, o[C::kDpl];
#pragma unroll
        for (int d = 0; d < C::kDpl; ++d) o[d] = 0.f;

        for (int t = 0; t < g.ntiles && !failed; ++t, ++k) {
            const int stage = k % C::kStages;
            const uint32_t ph = (uint32_t)(k / C::kStages) & 1u;
            if (*shFail || !mbar_wait_bounded(&full[stage], ph)) {
                if (lane == 0) {
                    report_error(kErrFullWait);
                    *shFail = 1;
                }
                failed = true;
                break;
            }
            const long long t0 = g.a0 + (long long)t * C::kTr;
            const uint8_t* base = smem + (size_t)stage * C::kStageBytes;
            if (t0 >= g.r0 && t0 + C::kTr <= g.r1)
                consume_tile<C, false>(base, warp, sg, sl, t0, g.r0, g.r1, qf, m, l, o);
            else
                consume_tile<C, true>(base, warp, sg, sl, t0, g.r0, g.r1, qf, m, l, o);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
        }
        // A warp that gave up keeps taking part in this unit's barriers (with
        // whatever partial state it has) so the other warps never block; after
        // the unit all warps see the shared flag and return together. The
        // error is visible through va_device_error.

        merge_chains_in_warp<C>(m, l, o);
        if (lane < C::kLpr) {
#pragma unroll
            for (int d = 0; d < C::kDpl; ++d) shO[warp * D + lane * C::kDpl + d] = o[d];
            if (lane == 0) {
                shM[warp] = m;
                shL[warp] = l;
            }
        }
        named_barrier_sync(1, kConsumerThreads);
        const int tid = threadIdx.x;
        float* slot = p.ws + ((size_t)g.h * p.S + g.s) * (D + 2);
        if (tid < D) {
            float ms = kNegMax;
#pragma unroll
            for (int w = 0; w < C::kWarps; ++w) ms = fmaxf(ms, shM[w]);
            float ls = 0.f, od = 0.f;
#pragma unroll
            for (int w = 0; w < C::kWarps; ++w) {
                const float a = fast_exp2(shM[w] - ms);
                ls += shL[w] * a;
                od += shO[w * D + tid] * a;
            }
            slot[2 + tid] = od;
            if (tid == 0) {
                slot[0] = ms * kLn2;  // natural-log units, as the reference's slots
                slot[1] = ls;
            }
        }
        if (p.out_mode != kOutSlots) {
            __threadfence();
            named_barrier_sync(1, kConsumerThreads);
            if (tid == 0) *shTicket = (int)atomicAdd(&p.counters[g.h], 1u);
            named_barrier_sync(1, kConsumerThreads);
            if (*shTicket == p.S - 1) {
                // last split of head h to finish: merge its S slots
                __threadfence();
                const float* hs = p.ws + (size_t)g.h * p.S * (D + 2);
                float ms = kNegMax;
                for (int s = 0; s < p.S; ++s) ms = fmaxf(ms, __ldcg(hs + (size_t)s * (D + 2)));
                if (tid < D) {
                    float ls = 0.f, od = 0.f;
                    for (int s = 0; s < p.S; ++s) {
                        const float* sp = hs + (size_t)s * (D + 2);
                        const float a = fast_exp2((__ldcg(sp) - ms) * kLog2e);
                        ls += __ldcg(sp + 1) * a;
                        od += __ldcg(sp + 2 + tid) * a;
                    }
                    if (p.out_mode == kOutHalf) {
                        p.out[(size_t)g.h * D + tid] = __float2half_rn(od / ls);
                    } else {
                        float* pp = p.partial + (size_t)g.h * (D + 2);
                        pp[2 + tid] = od;
                        if (tid == 0) {
                            pp[0] = ms;
                            pp[1] = ls;
                        }
                    }
                }
                if (tid == 0) p.counters[g.h] = 0u;  // leave the workspace ready for the next call
            }
        }
        named_barrier_sync(1, kConsumerThreads);
        if (*shFail) break;
    }
}

}  // namespace va
