// Staged streaming decode kernel (the "+" formats: f16+, q8+, q4+, q3+).
//
// Same math as the reference's sub-warp kernels (src/voltattn.cu:364-649):
// per head, score_j = q.K_j/sqrt(D), online softmax, o = sum_j p_j V_j, with
// K/V dequantized in registers. The B200 structure is new:
//
//   * Persistent CTAs (two per SM) walk work units (head, split) = (h, s). A
//     producer warp streams each unit's rows as tiles of TR rows (~32 KB of
//     codes + scales) through a 3-deep ring of shared-memory stages with bulk
//     asynchronous copies (cp.async.bulk, no multicast) completing on
//     mbarriers. Copies are kept at 16 KB or more: small bulk copies (~4 KB)
//     were measured to cap the per-SM stream rate far below HBM bandwidth.
//   * The 8 consumer warps split each tile; a warp runs 32/LPR independent
//     online-softmax chains (LPR lanes per row, 16 dims per lane; 8 for f16),
//     each chain taking RPS rows of the tile with one max/rescale per batch.
//   * Quantized K.q runs on the integer dot-product unit: q is held as 16-bit
//     fixed point split into signed-high / unsigned-low byte planes, and each
//     4-code word of K meets both planes in one dp4a each: exact integer
//     arithmetic, no code is converted to float. (q4: nibbles are masked into
//     even/odd byte lanes with the q planes permuted to match and the +8
//     offset removed with a precomputed sum; q3: 3-bit fields are spread into
//     byte lanes with masks and shifts, offset +4.)
//   * Quantized p.V: the batch's weights e_j * vs_j become 16-bit fixed point
//     relative to the batch maximum; the codes of 4 rows are byte-transposed
//     (8 prmt per 4 words) so that one dp4a accumulates 4 rows of one dim;
//     the integer sums are converted and folded into the fp32 output once
//     per batch. Weight error <= 2^-16 of the batch maximum.
//   * Tiles start on global row multiples of 8, which makes every copy of
//     codes and scales 16-byte aligned and a multiple of 16 bytes for all
//     formats and D in {64,128}; neighbouring rows a tile covers are masked
//     (weight 0, score -inf, even if they hold nan); the last (<8) rows of the
//     tensor, which a 16-byte copy could overrun, come from plain loads.
//   * A unit's chains merge in registers (shuffles) then shared memory into
//     one (m, l, o[D]) workspace slot (layout of src/voltattn.cu:92-93); the
//     last CTA to finish a head (one acquire-release ticket, no waiting)
//     merges the head's S slots and writes the output: the reference's
//     separate combine launch (src/voltattn.cu:651-672) is fused away.
// Every spin wait is bounded (kWaitLimitNs); on expiry the kernel records a
// device error and returns.
#pragma once

#include "formats.cuh"
#include "lse_merge.cuh"
#include "peer.cuh"

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
    int H, L, S;           // H: KV streams (B * Hkv), L: rows per stream (Lmax)
    int chunk;             // positions per split (multiple of 8)
    long long total_rows;  // H * L
    int out_mode;
    int Hkv;               // KV heads per sequence (== H for batch-1 decode)
    const int* lens;       // per-sequence valid lengths (nullptr: all L)
    // paged cache (tile kernels only; page_rows == 0: contiguous streams):
    // row j of KV head hk of sequence b is physical row
    // (block_table[b * max_pages + j / page_rows] * Hkv + hk) * page_rows + j % page_rows
    const int* block_table;
    int max_pages;
    int page_rows;
    int num_pages;
    // multi-query decode (grouped-query tile kernel): the kG query slots of a
    // KV stream are (query head, token) pairs, mq tokens per head; token i of
    // mq sees the stream's rows [0, len - (mq - 1 - i)) (1: plain decode)
    int mq;
    // split-L across GPUs fused into the decode (xR > 0, tile kernel): the
    // head's merged partial is exchanged with the other ranks over peer
    // memory and the R partials merged into out (peer.cuh)
    PeerBuffers x;
    int xR, xrank;
    unsigned xepoch;              // the step's epoch (1, 2, ...), or 0: read from *xepoch_ptr
    unsigned* xepoch_ptr;         // this rank's epoch counter in its peer buffer (device-counted steps)
    unsigned long long xwait_ns;  // bound of the wait for the peers' partials
};

// G = query heads per KV head (1: the reference's batch-1 multi-head decode;
// 2/4/8: grouped-query decode, the G heads share every streamed tile).
template <Kind K, int D, int G = 1>
struct StreamCfg {
    static constexpr Kind kKind = K;
    static constexpr int kD = D;
    static constexpr int kG = G;
    static constexpr int kBits = KindTraits<K>::kBits;
    static constexpr int kDpl = (K == Kind::F16 || K == Kind::BF16) ? 8 : 16;  // dims per lane
    static constexpr int kLpr = D / kDpl;                                  // lanes per row
    static constexpr int kNsg = 32 / kLpr;                                 // chains per warp
    static constexpr int kRps =
        (is_float_kind(K) || K == Kind::Q8) ? 4 : 8;  // rows per chain per tile
    static constexpr int kWarps = 8;                                       // consumer warps
    static constexpr int kThreads = (kWarps + 1) * 32;
    static constexpr int kTr = kWarps * kNsg * kRps;  // rows per tile
    static constexpr int kWpg = kWarps / G;           // warps per query head
    static constexpr int kRb = D * kBits / 8;         // code bytes per row
    static constexpr int kSb = (K == Kind::F16 || K == Kind::BF16) ? 0 : 2 * (D / kGroup);  // scale bytes per row
    static constexpr int kBpl = kDpl * kBits / 8;     // code bytes per lane
    static constexpr int kStages = 3;
    static constexpr int kStageBytes = 2 * kTr * kRb + 2 * kTr * kSb;
    static constexpr int kMergeBytes = (kWarps * (D + 2)) * 4 + 16;
    static constexpr int kSmemBytes = kStages * kStageBytes + 2 * kStages * 8 + kMergeBytes;
    static_assert(kTr % 8 == 0, "tiles must be whole 8-row blocks");
    static_assert((kTr * kRb) % 16 == 0 && (kTr * kSb) % 16 == 0, "16-byte stage sections");
    static_assert(kDpl <= kGroup, "a lane's dims must lie in one quant group");
    static_assert(kRps % 4 == 0, "rows per chain come in groups of 4");
    static_assert(G >= 1 && kWarps % G == 0, "query heads must divide the consumer warps");
    static_assert(kWarps * D >= kWarps * 32 + 64, "merge area doubles as the combine scratch");
};

struct UnitGeom {
    int h, s;          // KV stream (sequence * Hkv + KV head), split
    long long r0, r1;  // unit's global rows [r0, r1)
    long long a0;      // first tile's first row (r0 rounded down to 8)
    int ntiles;
};

// Units of a CTA: with at most one unit per CTA, unit blockIdx.x; with more,
// a contiguous range (same counts as a round robin, +-1), so consecutive
// units share a KV stream and per-stream state (the query's fixed-point
// form) is prepared once per stream instead of once per unit (1.6x on the
// batched grouped-query config).
__device__ __forceinline__ int unit_begin(int nunits, int next = 0) {
    if (nunits <= (int)gridDim.x) return min((int)blockIdx.x + next, nunits);
    return (int)(((long long)nunits * (blockIdx.x + next)) / gridDim.x);
}

template <class C>
__device__ __forceinline__ UnitGeom unit_geom(const DecodeParams& p, int u) {
    UnitGeom g;
    g.h = u / p.S;
    g.s = u - g.h * p.S;
    const long long len = p.lens ? (long long)min(max(__ldg(p.lens + g.h / p.Hkv), 0), p.L) : (long long)p.L;
    const long long j0 = min(len, (long long)g.s * p.chunk);
    const long long j1 = min(len, j0 + p.chunk);
    g.r0 = (long long)g.h * p.L + j0;
    g.r1 = (long long)g.h * p.L + j1;
    g.a0 = g.r0 & ~7ll;
    g.ntiles = (g.r1 > g.r0) ? (int)((g.r1 - g.a0 + C::kTr - 1) / C::kTr) : 0;
    return g;
}

// ---- integer helpers ----------------------------------------------------------

__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {  // a signed, b unsigned
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {  // a unsigned, b signed
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 4x4 byte transpose: byte j of in[i] -> byte i of out[j].
__device__ __forceinline__ void transpose4x4(const uint32_t a, const uint32_t b, const uint32_t c, const uint32_t d,
                                             uint32_t* o) {
    const uint32_t t0 = __byte_perm(a, b, 0x5140), t1 = __byte_perm(a, b, 0x7362);
    const uint32_t t2 = __byte_perm(c, d, 0x5140), t3 = __byte_perm(c, d, 0x7362);
    o[0] = __byte_perm(t0, t2, 0x5410);
    o[1] = __byte_perm(t0, t2, 0x7632);
    o[2] = __byte_perm(t1, t3, 0x5410);
    o[3] = __byte_perm(t1, t3, 0x7632);
}

// q3: fields at bits 0, 6, 12, 18 (3 bits each) -> byte lanes 0..3.
__device__ __forceinline__ uint32_t spread_q3(uint32_t x) {
    x &= 0x1C71C7u;
    x = (x & 0x1C7u) | ((x & 0x1C7000u) << 4);        // -> bits 0, 6, 16, 22
    return (x & 0x70007u) | ((x & 0x1C001C0u) << 2);  // -> bits 0, 8, 16, 24
}

// Exact int <-> float conversions for |x| < 2^22 without the XU pipe: the
// value rides in the mantissa of 1.5 * 2^23 (one integer add + one float
// add), instead of I2F / F2I, which share the transcendental unit with exp2.
__device__ __forceinline__ float small_int_to_float(int x) {
    return __int_as_float(x + 0x4B400000) - 12582912.0f;
}
__device__ __forceinline__ int float_to_small_int_rn(float f) {  // round to nearest even
    return __float_as_int(f + 12582912.0f) - 0x4B400000;
}

// ---- integer lane words -------------------------------------------------------------
// Integer kinds present each lane's 16 codes as 4 words of 4 byte lanes. The
// dim held by byte lane j of word w (word_dim) is a fixed permutation per
// kind; the q planes are built in the same order and V sums are scattered
// back through it, so results come out in natural dim order.
//   q8: word w = dims 4w..4w+3 (signed codes)
//   q4: word 2i = dims {8i, 8i+2, 8i+4, 8i+6}, word 2i+1 = {8i+1, ..., 8i+7}
//       (unsigned v+8)
//   q3: word 2i = fields {0,2,4,6} of granule i, word 2i+1 = fields {1,3,5,7}
//       (unsigned v+4)

template <Kind K>
struct IntWords {
    uint32_t w[4];
};

template <Kind K>
__device__ __forceinline__ void load_int_words(IntWords<K>& r, const uint8_t* p) {
    if constexpr (K == Kind::Q8) {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        r.w[0] = v.x;
        r.w[1] = v.y;
        r.w[2] = v.z;
        r.w[3] = v.w;
    } else if constexpr (K == Kind::Q4) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        r.w[0] = v.x & 0x0F0F0F0Fu;
        r.w[1] = (v.x >> 4) & 0x0F0F0F0Fu;
        r.w[2] = v.y & 0x0F0F0F0Fu;
        r.w[3] = (v.y >> 4) & 0x0F0F0F0Fu;
    } else {
        const uint16_t* p16 = reinterpret_cast<const uint16_t*>(p);
        const uint32_t a = p16[0], b = p16[1], c = p16[2];
        const uint32_t g0 = __byte_perm(a, b, 0x5410);  // bytes 0..2 of the slice
        const uint32_t g1 = __byte_perm(b, c, 0x0541);  // bytes 3..5
        r.w[0] = spread_q3(g0);
        r.w[1] = spread_q3(g0 >> 3);
        r.w[2] = spread_q3(g1);
        r.w[3] = spread_q3(g1 >> 3);
    }
}

template <Kind K>
__host__ __device__ constexpr int word_dim(int w, int j) {
    return K == Kind::Q8 ? 4 * w + j : 8 * (w / 2) + 2 * j + (w % 2);
}

// ---- f16 lane (fp32 math) ------------------------------------------------------------

template <Kind K>
struct FloatLane {
    float v[(K == Kind::F8) ? 16 : 8];
};

// One lane's 16 bytes as floats: 8 fp16 values, 8 bf16 values (the upper
// half of an fp32), or 16 e4m3 codes (CUDA's fp8 -> fp16 conversion, exact).
template <Kind K>
__device__ __forceinline__ void load_float_lane(FloatLane<K>& r, const uint8_t* p) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        if constexpr (K == Kind::F16) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            r.v[2 * i] = f.x;
            r.v[2 * i + 1] = f.y;
        } else if constexpr (K == Kind::BF16) {
            r.v[2 * i] = __uint_as_float(w[i] << 16);
            r.v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        } else {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const __half2_raw hr =
                    __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> (16 * j)), __NV_E4M3);
                const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hr));
                r.v[4 * i + 2 * j] = f.x;
                r.v[4 * i + 2 * j + 1] = f.y;
            }
        }
    }
}

// ---- producer warp ----------------------------------------------------------

template <class C>
__device__ void stream_producer(const DecodeParams& p, uint8_t* smem, uint64_t* full, uint64_t* empty) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol = l2_policy_evict_first();
    const long long nr8 = p.total_rows & ~7ll;
    const int nunits = p.H * p.S;
    int k = 0;
    const bool paged = p.page_rows > 0;
    for (int u = unit_begin(nunits), ue = unit_begin(nunits, 1); u < ue; ++u) {
        const UnitGeom g = unit_geom<C>(p, u);
        // paged cache: logical rows of whole 8-row blocks are copied (a page
        // holds whole blocks), so no row needs a plain load
        const long long cend = paged ? (g.r1 + 7) & ~7ll : min((g.r1 + 7) & ~7ll, nr8);
        for (int t = 0; t < g.ntiles; ++t, ++k) {
            const int stage = k % C::kStages;
            const uint32_t ph = (uint32_t)(k / C::kStages) & 1u;
            if (!mbar_wait_bounded(&empty[stage], ph ^ 1u)) {
                if (lane == 0) report_error(kErrEmptyWait);
                for (int d = 1; d <= C::kStages && k - d >= 0; ++d) {  // drain own copies
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
            if (paged) {
                // the tile's logical rows, one bulk copy per matrix and run of
                // rows inside one page (rows and pages are whole 8-row
                // blocks: every copy is 16-byte aligned and sized)
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[stage], (uint32_t)brows * (2u * C::kRb + 2u * C::kSb));
                    const int b = g.h / p.Hkv, hk = g.h - b * p.Hkv;
                    int j = (int)(t0 - (long long)g.h * p.L);  // sequence position (below 2^31)
                    for (int dr = 0; dr < brows;) {
                        const int pi = j / p.page_rows, in = j - pi * p.page_rows;
                        const int n = min(brows - dr, p.page_rows - in);
                        int pg = pi < p.max_pages ? __ldg(p.block_table + (size_t)b * p.max_pages + pi) : 0;
                        pg = (pg >= 0 && pg < p.num_pages) ? pg : 0;
                        const size_t ph = ((size_t)pg * p.Hkv + hk) * p.page_rows + in;
                        bulk_g2s(sK + (size_t)dr * C::kRb, p.K + ph * C::kRb, (uint32_t)n * C::kRb, &full[stage], pol);
                        bulk_g2s(sV + (size_t)dr * C::kRb, p.V + ph * C::kRb, (uint32_t)n * C::kRb, &full[stage], pol);
                        if constexpr (C::kSb > 0) {
                            bulk_g2s(sSK + (size_t)dr * C::kSb, reinterpret_cast<const uint8_t*>(p.scK) + ph * C::kSb,
                                     (uint32_t)n * C::kSb, &full[stage], pol);
                            bulk_g2s(sSV + (size_t)dr * C::kSb, reinterpret_cast<const uint8_t*>(p.scV) + ph * C::kSb,
                                     (uint32_t)n * C::kSb, &full[stage], pol);
                        }
                        dr += n;
                        j += n;
                    }
                }
                __syncwarp();
                continue;
            }
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

// ---- consumer: per-head query state ---------------------------------------------

template <class C>
struct QState {
    float qf[C::kDpl];  // float kinds: q * log2(e)/sqrt(D)
    uint32_t qp[8];     // integer kinds: q as 16-bit pairs, qp[2w] = byte lanes 0,1 of word w, qp[2w+1] = 2,3
    int qbias;          // q4 / q3: code offset * sum of this lane's fixed-point q
    float qscale;       // 2^-e * log2(e) / sqrt(D)
};

template <class C>
__device__ __forceinline__ void load_q(QState<C>& qs, const __half* qh, int sl) {
    constexpr int D = C::kD;
    const float base = rsqrtf((float)D) * kLog2e;
    float x[C::kDpl];
#pragma unroll
    for (int d = 0; d < C::kDpl; ++d) x[d] = __half2float(qh[sl * C::kDpl + d]);
    if constexpr (is_float_kind(C::kKind)) {
#pragma unroll
        for (int d = 0; d < C::kDpl; ++d) qs.qf[d] = x[d] * base;
    } else {
        // per-head 16-bit fixed point with |q| * 2^e < 2^14 over the whole head
        float amax = 0.f;
#pragma unroll
        for (int d = 0; d < C::kDpl; ++d) amax = fmaxf(amax, fabsf(x[d]));
#pragma unroll
        for (int off = 1; off < C::kLpr; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        int e = 0;
        if (amax > 0.f) {
            int ex;
            frexpf(amax, &ex);  // amax < 2^ex
            e = 14 - ex;
        }
        int qi[16];
        int sum = 0;
#pragma unroll
        for (int d = 0; d < 16; ++d) {
            qi[d] = __float2int_rn(ldexpf(x[d], e));
            sum += qi[d];
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const auto pair = [&](int j) {
                return ((uint32_t)qi[word_dim<C::kKind>(w, j)] & 0xFFFFu) |
                       ((uint32_t)qi[word_dim<C::kKind>(w, j + 1)] << 16);
            };
            qs.qp[2 * w] = pair(0);
            qs.qp[2 * w + 1] = pair(2);
        }
        qs.qbias = (C::kKind == Kind::Q4) ? 8 * sum : (C::kKind == Kind::Q3) ? 4 * sum : 0;
        qs.qscale = ldexpf(base, -e);
    }
}

// dp2a: c + a.h0 * b.b(0|2) + a.h1 * b.b(1|3); a = two 16-bit values, b = four bytes
template <bool kHi, bool kASigned, bool kBSigned>
__device__ __forceinline__ int dp2a(uint32_t a, uint32_t b, int c) {
    int d;
    if constexpr (kHi) {
        if constexpr (kASigned && kBSigned) asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        else if constexpr (kASigned) asm("dp2a.hi.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        else if constexpr (kBSigned) asm("dp2a.hi.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        else asm("dp2a.hi.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    } else {
        if constexpr (kASigned && kBSigned) asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        else if constexpr (kASigned) asm("dp2a.lo.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        else if constexpr (kBSigned) asm("dp2a.lo.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
        else asm("dp2a.lo.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    }
    return d;
}

// Dot of one lane slice with q (before the group scale), in log2 units.
template <class C>
__device__ __forceinline__ float lane_score(const QState<C>& qs, const uint8_t* kp) {
    if constexpr (is_float_kind(C::kKind)) {
        FloatLane<C::kKind> r;
        load_float_lane<C::kKind>(r, kp);
        float acc = 0.f;
#pragma unroll
        for (int d = 0; d < C::kDpl; ++d) acc = fmaf(qs.qf[d], r.v[d], acc);
        return acc;
    } else {
        IntWords<C::kKind> r;
        load_int_words<C::kKind>(r, kp);
        constexpr bool kSignedCodes = C::kKind == Kind::Q8;
        int x = -qs.qbias;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            x = dp2a<false, true, kSignedCodes>(qs.qp[2 * w], r.w[w], x);
            x = dp2a<true, true, kSignedCodes>(qs.qp[2 * w + 1], r.w[w], x);
        }
        // |x| < 2^22 for q4 / q3 (|q| < 2^14, |v| <= 7, 16 dims); q8 sums can
        // reach 2^25 and use the hardware converter
        if constexpr (C::kKind == Kind::Q8) return (float)x * qs.qscale;
        else return small_int_to_float(x) * qs.qscale;
    }
}

// ---- consumer: one tile --------------------------------------------------------

template <class C, bool kMasked>
__device__ __forceinline__ void consume_tile(const uint8_t* stage_base, int rb, int sg, int sl, long long t0,
                                             long long r0, long long r1, const QState<C>& qs, float& m, float& l,
                                             float* o) {
    constexpr int kG = C::kSb / 2;
    constexpr int R = C::kRps;
    const uint8_t* sK = stage_base;
    const uint8_t* sV = sK + C::kTr * C::kRb;
    const __half* sSK = reinterpret_cast<const __half*>(sV + C::kTr * C::kRb);
    const __half* sSV = sSK + C::kTr * kG;
    const int g = (sl * C::kDpl) / kGroup;

    // scores of this chain's R rows: tile rows (rb*R + i)*Nsg + sg of row
    // block rb, so at each step i the warp reads Nsg consecutive rows,
    // lane-contiguous
    float s[R];
    bool valid[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int lr = (rb * R + i) * C::kNsg + sg;
        valid[i] = true;
        if constexpr (kMasked) {
            const long long r = t0 + lr;
            valid[i] = (r >= r0) && (r < r1);
        }
        float acc = lane_score<C>(qs, sK + (size_t)lr * C::kRb + sl * C::kBpl);
        if constexpr (C::kSb > 0) acc *= __half2float(sSK[lr * kG + g]);
#pragma unroll
        for (int off = C::kLpr / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        s[i] = valid[i] ? acc : -INFINITY;
    }
    float mnew = m;
#pragma unroll
    for (int i = 0; i < R; ++i) mnew = fmaxf(mnew, s[i]);
    const float c = fast_exp2(m - mnew);
    m = mnew;
    float e[R];
    float esum = 0.f;
#pragma unroll
    for (int i = 0; i < R; ++i) {
        e[i] = fast_exp2(s[i] - mnew);
        esum += e[i];
    }
    l = l * c + esum;

    if constexpr (is_float_kind(C::kKind)) {
#pragma unroll
        for (int d = 0; d < C::kDpl; ++d) o[d] *= c;
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const int lr = (rb * R + i) * C::kNsg + sg;
            FloatLane<C::kKind> r;
            load_float_lane<C::kKind>(r, sV + (size_t)lr * C::kRb + sl * C::kBpl);
            float wi = e[i];
            if constexpr (C::kSb > 0) wi *= __half2float(sSV[lr * kG + g]);  // fp8: the group scale
            if constexpr (kMasked) {
                if (!valid[i]) {
                    wi = 0.f;
#pragma unroll
                    for (int d = 0; d < C::kDpl; ++d) r.v[d] = 0.f;
                }
            }
#pragma unroll
            for (int d = 0; d < C::kDpl; ++d) o[d] = fmaf(wi, r.v[d], o[d]);
        }
    } else {
        // weights e_i * vs_i as fixed point relative to the batch max: 15 bits
        // (q4 / q3) or 13 bits (q8, keeps every 4-row group sum below 2^22)
        constexpr float kPmax = (C::kKind == Kind::Q8) ? 8191.f : 32767.f;
        float w[R];
        float wmax = 0.f;
#pragma unroll
        for (int i = 0; i < R; ++i) {
            const int lr = (rb * R + i) * C::kNsg + sg;
            w[i] = e[i] * __half2float(sSV[lr * kG + g]);
            if constexpr (kMasked) w[i] = valid[i] ? w[i] : 0.f;
            wmax = fmaxf(wmax, w[i]);
        }
        const float inv = wmax > 0.f ? kPmax / wmax : 0.f;
        // p_i rides in the low bits of 1.5 * 2^23: the float's bit pattern is
        // 0x4B400000 + p_i, so its low half is p_i
        uint32_t pb[R];
        uint32_t psum_u = 0;
#pragma unroll
        for (int i = 0; i < R; ++i) {
            pb[i] = __float_as_uint(fmaf(w[i], inv, 12582912.0f));
            psum_u += pb[i] - 0x4B400000u;
        }
        const int psum = (int)psum_u;
        constexpr bool kSignedCodes = C::kKind == Kind::Q8;
        if constexpr (C::kKind == Kind::Q4) {
            // raw bytes (two nibbles) transposed once; per byte the dot with the
            // full byte and with its low nibble give both dims:
            // hi = (full - lo) / 16
            int af[8], al[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) af[k] = al[k] = 0;
#pragma unroll
            for (int g4 = 0; g4 < R / 4; ++g4) {
                const uint32_t p01 = __byte_perm(pb[4 * g4], pb[4 * g4 + 1], 0x5410);
                const uint32_t p23 = __byte_perm(pb[4 * g4 + 2], pb[4 * g4 + 3], 0x5410);
                uint2 raw[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int lr = (rb * R + 4 * g4 + j) * C::kNsg + sg;
                    raw[j] = *reinterpret_cast<const uint2*>(sV + (size_t)lr * C::kRb + sl * C::kBpl);
                }
                uint32_t t[8];
                transpose4x4(raw[0].x, raw[1].x, raw[2].x, raw[3].x, t);
                transpose4x4(raw[0].y, raw[1].y, raw[2].y, raw[3].y, t + 4);
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    const uint32_t tl = t[k] & 0x0F0F0F0Fu;
                    af[k] = dp2a<false, false, false>(p01, t[k], af[k]);
                    af[k] = dp2a<true, false, false>(p23, t[k], af[k]);
                    al[k] = dp2a<false, false, false>(p01, tl, al[k]);
                    al[k] = dp2a<true, false, false>(p23, tl, al[k]);
                }
            }
            const float wscale = wmax * (1.f / kPmax);
            // the running max rarely moves once a chain is warm: skip the
            // rescale when no chain of the warp needs it
            if (__any_sync(0xffffffffu, c != 1.f)) {
#pragma unroll
                for (int d = 0; d < 16; ++d) o[d] *= c;
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int xlo = al[k] - 8 * psum;
                const int xhi16 = af[k] - al[k] - 128 * psum;  // 16 * (sum of p * hi-nibble value)
                o[2 * k] = fmaf((float)xlo, wscale, o[2 * k]);
                o[2 * k + 1] = fmaf((float)xhi16, wscale * 0.0625f, o[2 * k + 1]);
            }
        } else {
            int acc[16];
#pragma unroll
            for (int d = 0; d < 16; ++d) acc[d] = 0;
#pragma unroll
            for (int g4 = 0; g4 < R / 4; ++g4) {
                const uint32_t p01 = __byte_perm(pb[4 * g4], pb[4 * g4 + 1], 0x5410);
                const uint32_t p23 = __byte_perm(pb[4 * g4 + 2], pb[4 * g4 + 3], 0x5410);
                IntWords<C::kKind> rw[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int lr = (rb * R + 4 * g4 + j) * C::kNsg + sg;
                    load_int_words<C::kKind>(rw[j], sV + (size_t)lr * C::kRb + sl * C::kBpl);
                }
#pragma unroll
                for (int wi = 0; wi < 4; ++wi) {
                    uint32_t t[4];  // t[j]: byte lane j of word wi for rows 0..3
                    transpose4x4(rw[0].w[wi], rw[1].w[wi], rw[2].w[wi], rw[3].w[wi], t);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int d = word_dim<C::kKind>(wi, j);
                        acc[d] = dp2a<false, false, kSignedCodes>(p01, t[j], acc[d]);
                        acc[d] = dp2a<true, false, kSignedCodes>(p23, t[j], acc[d]);
                    }
                }
            }
            const int bias = (C::kKind == Kind::Q3) ? 4 * psum : 0;
            const float wscale = wmax * (1.f / kPmax);
#pragma unroll
            if (__any_sync(0xffffffffu, c != 1.f)) {
#pragma unroll
                for (int d = 0; d < 16; ++d) o[d] *= c;
            }
#pragma unroll
            for (int d = 0; d < 16; ++d) {
                // q3: |x| <= 8 * 32767 * 3 < 2^22; q8: |x| <= 4 * 8191 * 127 < 2^22
                o[d] = fmaf(small_int_to_float(acc[d] - bias), wscale, o[d]);
            }
        }
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
    // Everything above touches only shared memory. Nothing below reads or
    // writes global memory before the preceding grid has fully completed, so
    // results equal plain stream order; the early trigger lets the next
    // decode's CTAs be resident and initialised as soon as ours exit.
    grid_dependency_wait();
    if (threadIdx.x == 0) grid_launch_dependents();

    if (warp == C::kWarps) {
        stream_producer<C>(p, smem, full, empty);
        return;
    }

    constexpr int kConsumerThreads = C::kWarps * 32;
    const int sg = lane / C::kLpr, sl = lane % C::kLpr;
    const int hk = warp / C::kWpg;   // this warp's query head within the group
    const int wig = warp % C::kWpg;  // and its index among that head's warps
    const int nunits = p.H * p.S;
    QState<C> qs;
    int cur_h = -1;
    int k = 0;  // CTA tile counter (the producer's sequence)
    for (int u = unit_begin(nunits), ue = unit_begin(nunits, 1); u < ue; ++u) {
        bool failed = false;
        const UnitGeom g = unit_geom<C>(p, u);
        if (g.h != cur_h) {
            load_q<C>(qs, p.q + ((size_t)g.h * C::kG + hk) * D, sl);
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
            const bool interior = t0 >= g.r0 && t0 + C::kTr <= g.r1;
            // the head's kWpg warps split the tile; each takes G row blocks
#pragma unroll
            for (int j = 0; j < C::kG; ++j) {
                const int rb = wig * C::kG + j;
                if (interior)
                    consume_tile<C, false>(base, rb, sg, sl, t0, g.r0, g.r1, qs, m, l, o);
                else
                    consume_tile<C, true>(base, rb, sg, sl, t0, g.r0, g.r1, qs, m, l, o);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
        }
        // A warp that gave up keeps taking part in this unit's barriers so the
        // others never block; after the unit all warps see the shared flag and
        // return together. The error is visible through va_device_error.

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
        if (tid < D) {
#pragma unroll
            for (int kq = 0; kq < C::kG; ++kq) {
                const int w0 = kq * C::kWpg;
                float ms = kNegMax;
#pragma unroll
                for (int w = 0; w < C::kWpg; ++w) ms = fmaxf(ms, shM[w0 + w]);
                float ls = 0.f, od = 0.f;
#pragma unroll
                for (int w = 0; w < C::kWpg; ++w) {
                    const float a = fast_exp2(shM[w0 + w] - ms);
                    ls += shL[w0 + w] * a;
                    od += shO[(w0 + w) * D + tid] * a;
                }
                float* slot = p.ws + (((size_t)g.h * C::kG + kq) * p.S + g.s) * (D + 2);
                slot[2 + tid] = od;
                if (tid == 0) {
                    slot[0] = ms * kLn2;  // natural-log units, as the reference's slots
                    slot[1] = ls;
                }
            }
        }
        if (p.out_mode != kOutSlots) {
            named_barrier_sync(1, kConsumerThreads);
            if (tid == 0) *shTicket = (int)atomic_add_acq_rel_gpu(&p.counters[g.h], 1u);
            named_barrier_sync(1, kConsumerThreads);
            if (*shTicket == p.S - 1) {
                // last split of this KV stream to finish: merge the S slots of
                // each of its query heads (the merge area is free again after
                // the ticket barrier)
                for (int kq = 0; kq < C::kG; ++kq) {
                    const size_t hq = (size_t)g.h * C::kG + kq;
                    const float* hs = p.ws + hq * p.S * (D + 2);
                    float ms, ls, od;
                    lse_merge([&](int i) { return hs + (size_t)i * (D + 2); }, p.S, D, tid, kConsumerThreads,
                              LseScratch{shO, shO + kConsumerThreads},
                              [] { named_barrier_sync(1, kConsumerThreads); }, ms, ls, od);
                    if (tid < D) {
                        if (p.out_mode == kOutHalf) {
                            p.out[hq * D + tid] = __float2half_rn(od / ls);
                        } else {
                            float* pp = p.partial + hq * (D + 2);
                            pp[2 + tid] = od;
                            if (tid == 0) {
                                pp[0] = ms;
                                pp[1] = ls;
                            }
                        }
                    }
                }
                if (tid == 0) store_relaxed_gpu(&p.counters[g.h], 0u);  // ready for the next call
            }
        }
        named_barrier_sync(1, kConsumerThreads);
        if (*shFail) break;
    }
}

}  // namespace va
