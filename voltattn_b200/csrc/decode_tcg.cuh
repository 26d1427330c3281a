// Tensor-core tile kernel for grouped-query decode with G = 4 query heads per
// KV head (q4+, D = 128): every streamed K/V row serves 4 query heads.
//
// Front end, schedule, ticket warp and head merge are those of the batch-1
// tile kernel (decode_tc.cuh): 2-D tensor copies with the 64-byte swizzle into
// a 3-deep ring of 256-row tiles, a head's splits taking interleaved tiles,
// dynamic units, per-stage headers. The consumer is laid out by head instead
// of by quant group: with g = lane / 4 and t = lane % 4, lane (g, t) works for
// query head t of the group.
//
//   scores  per 16-row block, per quant group gi and kind: one m16n8k32 per
//           half chunk, A = K rows (lane t reads chunk t of rows A(g), B(g)),
//           B = the 4 heads' q (16-bit fixed point, signed byte planes) in
//           columns (head, plane). Kinds: low nibbles x even-dim q (LE), low
//           nibbles x odd-dim q (LO), raw bytes x odd-dim q (RO); 16 LE + RO -
//           LO = 16 x (the group's dot), exactly. B is zero outside the
//           group's chunks, so each accumulator holds one group's sum and
//           lane t gets head t's score of its two rows with no reduction.
//   softmax per head over the warp's 64 rows (8 per lane; reductions over
//           the 8 lanes of a head), weights e * vs per quant group as 15-bit
//           fixed point relative to the tile's maximum.
//   output  O^T += V^T . P per chunk: A = V^T by ldmatrix.m16n16.trans.b8, k =
//           32 rows of two blocks, B = weight planes of the 4 heads in columns
//           (head, plane), staged per warp; raw-byte and low-nibble mmas as
//           in the batch-1 kernel.
// Rows are placed in each block so that a quad's four rows of a k-step are
// distinct modulo 8 and each ldmatrix phase reads 8 distinct residues (the
// swizzle period), and the 128-bit K loads of quads 2i, 2i+1 hit rows of
// different parity: all shared-memory reads of the tiles are conflict-free.
#pragma once

#include "decode_tc.cuh"

namespace va {

template <Kind K, int D, int G>
struct TcgCfg {
    static constexpr Kind kKind = K;
    static constexpr int kD = D;
    static constexpr int kG = G;
    static constexpr int kBits = KindTraits<K>::kBits;
    static constexpr int kRb = D * kBits / 8;
    static constexpr int kRbT = kRb;  // compute-tile row bytes (the swizzle span)
    static constexpr int kChunks = kRb / 16;
    static constexpr int kNgrp = D / kGroup;
    static constexpr int kSb = 2 * kNgrp;
    static constexpr bool kChan = false;  // group scales on every K and V row
    static constexpr int kSbK = kSb, kSbV = kSb;
    static constexpr int kHg = G < 4 ? 1 : G / 4;  // head groups: 4 query head slots per consumer warp
    static constexpr int kRowWarps = 4;      // warps splitting a tile's rows
    static constexpr int kWarps = kRowWarps * kHg;
    static constexpr int kRpw = 64;
    static constexpr int kTr = kRowWarps * kRpw;
    static constexpr int kBox = 32;
    // rows per tensor copy of a contiguous cache: 128 (config 5: 0.266 -> 0.260 ms against 32)
    static constexpr int kBoxC = 128;
    static constexpr int kThreads = (kWarps + 2) * 32;
    static constexpr int kMinBlocks = kHg == 1 ? 2 : 1;  // CTAs per SM the smem budget is cut for
    static constexpr int kStages = kHg == 1 ? 3 : 5;
    static constexpr int kTRing = 4;
    static constexpr int kStageBytes = (2 * kTr * kRb + 2 * kTr * kSb + 1023) & ~1023;
    static constexpr int kQBytes = G * D * 2;
    // per warp: weight B fragments [k-step][group][lane] (8 bytes); also the
    // merge area at a unit's end (per head group: 2 warps x 32 lanes x 18 floats)
    static constexpr int kPWarp = 2 * 2 * 32 * 8;
    static constexpr int kMergeBytes = kHg * 2 * 32 * 18 * 4;
    static constexpr int kPArea = (kWarps * kPWarp > kMergeBytes) ? kWarps * kPWarp : kMergeBytes;
    static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 2 * kStages * 8 + kStages * 16 +
                                      kStages * kQBytes + kPArea + 2 * kTRing * 8 + kTRing * 4 + 16 + 16 +
                                      kQBytes;
    static_assert(K == Kind::Q4 && D == 128 && (G == 2 || G == 4 || G == 8),
                  "q4+, D = 128, 2, 4 or 8 query heads per KV head (G = 2 leaves 2 of 4 head slots idle)");
    static_assert(kRb == 64, "64-byte swizzle");
    static_assert((kStages * kStageBytes + 2 * kStages * 8 + kStages * 16) % 16 == 0, "query ring");
    static_assert((kStages * kQBytes + kPArea + 2 * kTRing * 8 + kTRing * 4 + 16) % 16 == 0, "first query");
    static_assert(kSmemBytes <= 227 * 1024, "shared memory");
};

// Row of 16-row block `blk` held by mma row g (A) and g + 8 (B).
__host__ __device__ constexpr int tcg_row_a(int blk, int q) { return (blk & 1) ? (q ^ 2) : q; }
__host__ __device__ constexpr int tcg_row_b(int blk, int q) { return 8 + ((blk & 1) ? (q ^ 3) : (q ^ 1)); }

// Per-stream query state of a lane: B fragments for its column (head g/2,
// plane g%2) and the bias / scale of its own head t.
struct TcgQ {
    uint32_t be[2][2][2];  // even-dim q [group][half][reg]
    uint32_t bo[2][2][2];  // odd-dim q
    int bias[2];           // -8 * sum(q over the group) for head t (low-nibble column start)
    float qs;              // 2^-e * log2(e)/sqrt(D) / 16 for head t
};

template <class C>
__device__ __forceinline__ void tcg_load_q(TcgQ& tq, const __half* qs, int g, int t, int lane) {
    constexpr int D = C::kD, G = 4;                      // the warp's head slots
    constexpr int kActive = C::kG < 4 ? C::kG : 4;       // slots holding a query head (rest: q = 0)
    // per-head exponent and group sums: lane L holds dims 4L..4L+3 of each head
    int e[G];
    float x[G][4];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const uint2 w4 = h < kActive ? reinterpret_cast<const uint2*>(qs + h * D)[lane] : make_uint2(0u, 0u);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w4.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w4.y));
        x[h][0] = a.x;
        x[h][1] = a.y;
        x[h][2] = b.x;
        x[h][3] = b.y;
        float amax = fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(b.x), fabsf(b.y)));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        e[h] = amax > 0.f ? 14 - (((__float_as_int(amax) >> 23) & 0xFF) - 126) : 0;
    }
    int s[G];  // lanes 0-15: group 0 sums, lanes 16-31: group 1 sums
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const float sc = __int_as_float((127 + e[h]) << 23);
        s[h] = __float2int_rn(x[h][0] * sc) + __float2int_rn(x[h][1] * sc) + __float2int_rn(x[h][2] * sc) +
               __float2int_rn(x[h][3] * sc);
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) s[h] += __shfl_xor_sync(0xffffffffu, s[h], off);
    }
    int st0 = 0, st1 = 0, et = 0;
#pragma unroll
    for (int h = 0; h < G; ++h) {
        const int a = __shfl_sync(0xffffffffu, s[h], 0), b = __shfl_sync(0xffffffffu, s[h], 16);
        if (h == t) {
            st0 = a;
            st1 = b;
            et = e[h];
        }
    }
    tq.bias[0] = -8 * st0;
    tq.bias[1] = -8 * st1;
    tq.qs = rsqrtf((float)D) * kLog2e * 0.0625f / __int_as_float((127 + et) << 23);
    // B fragment bytes of column (head hc = g/2, plane g%2): chunk t (dims 32t..32t+31), group t/2
    const int hc = g >> 1, plane = g & 1;
    int ec = 0;
#pragma unroll
    for (int h = 0; h < G; ++h)
        if (h == hc) ec = e[h];
    const float scc = __int_as_float((127 + ec) << 23);
    const uint4* src = reinterpret_cast<const uint4*>(qs + (hc < kActive ? hc : 0) * D + 32 * t);
    uint32_t we[4], wo[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {  // 8 dims = 4 bytes per 16-byte load
        const uint4 h = hc < kActive ? src[c] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
        uint32_t ae = 0, ao = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hw[j]));
            ae |= tc_plane_byte(f.x, scc, plane) << (8 * j);
            ao |= tc_plane_byte(f.y, scc, plane) << (8 * j);
        }
        we[c] = ae;
        wo[c] = ao;
    }
    const int gt = t >> 1;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                tq.be[gi][hf][r] = gi == gt ? we[2 * hf + r] : 0u;
                tq.bo[gi][hf][r] = gi == gt ? wo[2 * hf + r] : 0u;
            }
}

template <class C>
struct TcgState {
    float m, l;
    float o[4][4];  // head t: chunk c, byte g (lo, hi dim), byte g + 8 (lo, hi dim)
};

template <class C, bool kMasked>
__device__ __forceinline__ void tcg_tile(uint32_t sK, uint32_t sV, const __half* sSK, const __half* sSV, uint8_t* sp,
                                         int wrow, int g, int t, long long t0, long long r0, long long r1,
                                         const TcgQ& tq, const uint32_t* voff, TcgState<C>& st) {
    constexpr int kRb = C::kRb;
    const uint32_t m4 = 0x0F0F0F0Fu;
    // ---- scores of head t, rows A / B of blocks 0..3 ----------------------------------------
    float s[4][2];
    bool valid[4][2];
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const int ra = tcg_row_a(blk, g), rbw = tcg_row_b(blk, g);
        const uint32_t base = sK + (uint32_t)((wrow + 16 * blk) * kRb);
        const uint4 wa = lds128(base + (uint32_t)tc_swz<C>(ra, t));
        const uint4 wb = lds128(base + (uint32_t)tc_swz<C>(rbw, t));
        const uint32_t la[4] = {wa.x & m4, wa.y & m4, wa.z & m4, wa.w & m4};
        const uint32_t lb[4] = {wb.x & m4, wb.y & m4, wb.z & m4, wb.w & m4};
        int v[2][2];  // [group][row]
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            int le[4] = {0, tq.bias[gi], 0, tq.bias[gi]}, lo[4] = {0, 0, 0, 0}, ro[4] = {0, 0, 0, 0};
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                mma_k32<false, true>(le, la[2 * hf], lb[2 * hf], la[2 * hf + 1], lb[2 * hf + 1], tq.be[gi][hf][0],
                                     tq.be[gi][hf][1]);
                mma_k32<false, true>(lo, la[2 * hf], lb[2 * hf], la[2 * hf + 1], lb[2 * hf + 1], tq.bo[gi][hf][0],
                                     tq.bo[gi][hf][1]);
            }
            const uint32_t ra4[4] = {wa.x, wa.y, wa.z, wa.w}, rb4[4] = {wb.x, wb.y, wb.z, wb.w};
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
                mma_k32<false, true>(ro, ra4[2 * hf], rb4[2 * hf], ra4[2 * hf + 1], rb4[2 * hf + 1],
                                     tq.bo[gi][hf][0], tq.bo[gi][hf][1]);
            // columns 2t (high plane), 2t+1 (low plane) of head t
            v[gi][0] = 16 * (256 * le[0] + le[1]) + (256 * ro[0] + ro[1]) - (256 * lo[0] + lo[1]);
            v[gi][1] = 16 * (256 * le[2] + le[3]) + (256 * ro[2] + ro[3]) - (256 * lo[2] + lo[3]);
        }
        const float2 ka = __half22float2(*reinterpret_cast<const __half2*>(sSK + (wrow + 16 * blk + ra) * 2));
        const float2 kb = __half22float2(*reinterpret_cast<const __half2*>(sSK + (wrow + 16 * blk + rbw) * 2));
        s[blk][0] = ((float)v[0][0] * ka.x + (float)v[1][0] * ka.y) * tq.qs;
        s[blk][1] = ((float)v[0][1] * kb.x + (float)v[1][1] * kb.y) * tq.qs;
        valid[blk][0] = valid[blk][1] = true;
        if constexpr (kMasked) {
            const long long xa = t0 + wrow + 16 * blk + ra, xb = t0 + wrow + 16 * blk + rbw;
            valid[blk][0] = xa >= r0 && xa < r1;
            valid[blk][1] = xb >= r0 && xb < r1;
            s[blk][0] = valid[blk][0] ? s[blk][0] : -INFINITY;
            s[blk][1] = valid[blk][1] ? s[blk][1] : -INFINITY;
        }
    }

    // ---- online softmax of head t over the warp's 64 rows (lanes t, t+4, ..., t+28) ----------
    float bm = s[0][0];
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) bm = fmaxf(bm, fmaxf(s[blk][0], s[blk][1]));
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
    const float mnew = fmaxf(st.m, bm);
    const float c = fast_exp2(st.m - mnew);
    st.m = mnew;
    float w[4][2][2];  // [blk][row][group]
    float wm[2] = {0.f, 0.f};
    float esum = 0.f;
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const int rr[2] = {tcg_row_a(blk, g), tcg_row_b(blk, g)};
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float e = fast_exp2(s[blk][r] - mnew);
            esum += e;
            const float2 vs =
                __half22float2(*reinterpret_cast<const __half2*>(sSV + (wrow + 16 * blk + rr[r]) * 2));
            w[blk][r][0] = e * vs.x;
            w[blk][r][1] = e * vs.y;
            if constexpr (kMasked) {
                w[blk][r][0] = valid[blk][r] ? w[blk][r][0] : 0.f;
                w[blk][r][1] = valid[blk][r] ? w[blk][r][1] : 0.f;
            }
            wm[0] = fmaxf(wm[0], w[blk][r][0]);
            wm[1] = fmaxf(wm[1], w[blk][r][1]);
        }
    }
    st.l = st.l * c + esum;
    float wscale[2];
    int psum[2];
    uint32_t pb[4][2][2];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) wm[gi] = fmaxf(wm[gi], __shfl_xor_sync(0xffffffffu, wm[gi], off));
        const float inv = wm[gi] > 0.f ? 32767.f / wm[gi] : 0.f;
        wscale[gi] = wm[gi] * (1.f / 32767.f);
        int ps = 0;
#pragma unroll
        for (int blk = 0; blk < 4; ++blk)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                pb[blk][r][gi] = __float_as_uint(fmaf(w[blk][r][gi], inv, 12582912.0f));
                ps += (int)(pb[blk][r][gi] - 0x4B400000u);
            }
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
        psum[gi] = ps;
    }
    // stage the weight planes as B fragments: k-step ks (blocks 2ks, 2ks+1), owner
    // quad g -> dest lanes (column 2t / 2t+1, t' of g), half (g >> 1) & 1
    {
        const int tp = ((g & 1) << 1) | (g >> 2), half = (g >> 1) & 1;
#pragma unroll
        for (int ks = 0; ks < 2; ++ks)
#pragma unroll
            for (int gi = 0; gi < 2; ++gi) {
                const uint32_t a = __byte_perm(pb[2 * ks][0][gi], pb[2 * ks][1][gi], 0x5140);
                const uint32_t b = __byte_perm(pb[2 * ks + 1][0][gi], pb[2 * ks + 1][1][gi], 0x5140);
                const uint32_t lo_w = __byte_perm(a, b, 0x5410), hi_w = __byte_perm(a, b, 0x7632);
                uint32_t* area = reinterpret_cast<uint32_t*>(sp + (ks * 2 + gi) * 32 * 8);
                area[(4 * (2 * t) + tp) * 2 + half] = hi_w;      // column 2t: high plane
                area[(4 * (2 * t + 1) + tp) * 2 + half] = lo_w;  // column 2t+1: low plane
            }
    }
    __syncwarp();

    // ---- output: O^T += V^T . P per chunk ------------------------------------------------------
    if (__any_sync(0xffffffffu, c != 1.f)) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch)
#pragma unroll
            for (int x = 0; x < 4; ++x) st.o[ch][x] *= c;
    }
    const int lane = 4 * g + t;
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
        uint2 bf[2];
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) bf[ks] = reinterpret_cast<const uint2*>(sp + (ks * 2 + gi) * 32 * 8)[lane];
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
            const int ch = 2 * gi + cc;
            int aR[4] = {0, -136 * psum[gi], 0, -136 * psum[gi]}, aL[4] = {0, -8 * psum[gi], 0, -8 * psum[gi]};
#pragma unroll
            for (int ks = 0; ks < 2; ++ks) {
                const uint4 a = ldsm_x2_trans_b8(sV + (uint32_t)((wrow + 32 * ks) * kRb) + voff[ch]);
                mma_k32<false, false>(aR, a.x, a.y, a.z, a.w, bf[ks].x, bf[ks].y);
                mma_k32<false, false>(aL, a.x & m4, a.y & m4, a.z & m4, a.w & m4, bf[ks].x, bf[ks].y);
            }
            const int xl0 = 256 * aL[0] + aL[1], xl1 = 256 * aL[2] + aL[3];
            const int xr0 = 256 * aR[0] + aR[1], xr1 = 256 * aR[2] + aR[3];
            const float ws = wscale[gi], ws16 = wscale[gi] * 0.0625f;
            st.o[ch][0] = fmaf((float)xl0, ws, st.o[ch][0]);
            st.o[ch][1] = fmaf((float)(xr0 - xl0), ws16, st.o[ch][1]);
            st.o[ch][2] = fmaf((float)xl1, ws, st.o[ch][2]);
            st.o[ch][3] = fmaf((float)(xr1 - xl1), ws16, st.o[ch][3]);
        }
    }
    __syncwarp();
}

template <class C, bool kPaged>
__global__ void __launch_bounds__(C::kThreads, C::kMinBlocks)
    decode_tcg_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    constexpr int D = C::kD, G = C::kG;
    uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(stages + C::kStages * C::kStageBytes);
    uint64_t* empty = full + C::kStages;
    TcHeader* hdr = reinterpret_cast<TcHeader*>(empty + C::kStages);
    uint8_t* qring = reinterpret_cast<uint8_t*>(hdr + C::kStages);
    uint8_t* shP = qring + C::kStages * C::kQBytes;  // weight staging; merge area at unit end
    uint64_t* tdone = reinterpret_cast<uint64_t*>(shP + C::kPArea);
    uint64_t* tfree = tdone + C::kTRing;
    int* th = reinterpret_cast<int*>(tfree + C::kTRing);
    volatile int* shFail = th + C::kTRing;
    uint64_t* qbar = reinterpret_cast<uint64_t*>(th + C::kTRing + 4);
    uint8_t* qfirst = reinterpret_cast<uint8_t*>(qbar + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::kWarps);
        }
        for (int e = 0; e < C::kTRing; ++e) {
            mbar_init(&tdone[e], C::kWarps);
            mbar_init(&tfree[e], 1);
        }
        mbar_init(qbar, 1);
        *shFail = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // programmatic dependent launch: as in decode_tc_kernel
    if (warp != C::kWarps || !kTcEarlyKv) grid_dependency_wait();
    if (threadIdx.x == 0) grid_launch_dependents();

    const int h0 = (int)blockIdx.x / p.S;
    if (warp == C::kWarps) {
        if (lane == 0) {
            prefetch_tensormap(&tmK);
            prefetch_tensormap(&tmV);
        }
        tc_producer<C, kPaged>(p, &tmK, &tmV, stages, hdr, qring, full, empty, qfirst, qbar,
                       reinterpret_cast<volatile unsigned*>(shFail + 2));
        return;
    }
    if (warp == C::kWarps + 1) {
        if (p.out_mode != kOutSlots)
            tc_ticket_warp<C>(p, th, tdone, tfree, shFail + 1, reinterpret_cast<volatile unsigned*>(shFail + 2));
        return;
    }

    constexpr int kConsumerThreads = C::kWarps * 32;
    const int g = lane >> 2, t = lane & 3, tid = threadIdx.x;
    uint8_t* sp = shP + warp * C::kPWarp;
    const int rw = warp % C::kRowWarps, hg = warp / C::kRowWarps;  // rows of the tile, head group
    const int wrow = rw * C::kRpw;
    // ldmatrix row of this lane in a 32-row k-step: k = lane (rows of blocks 2ks, 2ks+1)
    uint32_t voff[4];
    {
        const int k = lane & 15, hi = lane >> 4;
        const int q = tc_q1(k >> 2) + 2 * hi, j = k & 3;
        const int blk = j >> 1;
        const int row = 16 * blk + ((j & 1) ? tcg_row_b(blk, q) : tcg_row_a(blk, q));
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) voff[ch] = (uint32_t)tc_swz<C>(row, ch);
    }
    TcgQ tq;
    TcgState<C> st;
    TcUnit gm;
    int cur_h = -1;
    if (mbar_wait_bounded(qbar, 0)) {
        tcg_load_q<C>(tq, reinterpret_cast<const __half*>(qfirst) + hg * 4 * D, g, t, lane);
        cur_h = h0;
    } else if (lane == 0) {
        report_error(kErrFullWait);
    }
    const bool tickets = p.out_mode != kOutSlots;
    int nu = 0;
    const auto hand_over = [&](int h) {
        const int e = nu % C::kTRing;
        if (tid == 0) th[e] = h;
        named_barrier_sync(1, kConsumerThreads);
        __syncwarp();
        if (lane == 0) mbar_arrive(&tdone[e]);
        ++nu;
    };
    const auto ring_slot_free = [&]() -> bool {
        return mbar_wait_bounded(&tfree[nu % C::kTRing], ((uint32_t)(nu / C::kTRing) & 1u) ^ 1u);
    };
    for (int k = 0;; ++k) {
        const int stage = k % C::kStages;
        const uint32_t ph = (uint32_t)(k / C::kStages) & 1u;
        if (*shFail || !mbar_wait_bounded(&full[stage], ph)) {
            if (lane == 0) {
                report_error(kErrFullWait);
                *shFail = 1;
            }
            break;
        }
        const TcHeader h = hdr[stage];
        if (h.unit < 0) break;
        uint8_t* base = stages + (size_t)stage * C::kStageBytes;
        if (h.tile == 0) {
            gm = tc_unit_geom<C>(p, h.unit);
            if (gm.h != cur_h && h.ntiles > 0) {
                tcg_load_q<C>(tq, reinterpret_cast<const __half*>(qring + stage * C::kQBytes) + hg * 4 * D, g, t,
                              lane);
                cur_h = gm.h;
            }
            st.m = kNegMax;
            st.l = 0.f;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
#pragma unroll
                for (int x = 0; x < 4; ++x) st.o[ch][x] = 0.f;
        }
        if (h.ntiles > 0) {
            const long long t0 = tc_tile_row<C>(gm, h.trow);
            const uint32_t sK = smem_u32(base), sV = sK + C::kTr * C::kRb;
            const __half* sSK = reinterpret_cast<const __half*>(base + 2 * C::kTr * C::kRb);
            const __half* sSV = sSK + C::kTr * C::kNgrp;
            const long long w0 = t0 + wrow;
            // multi-query: this lane's slot is token (4 hg + t) % mq, which sees
            // mq - 1 - token fewer rows; no masking only where every slot sees the warp's rows
            const long long r1l = gm.r1 - (p.mq - 1 - (4 * hg + t) % p.mq);
            if (w0 >= gm.r0 && w0 + C::kRpw <= gm.r1 - (p.mq - 1))
                tcg_tile<C, false>(sK, sV, sSK, sSV, sp, wrow, g, t, t0, gm.r0, r1l, tq, voff, st);
            else
                tcg_tile<C, true>(sK, sV, sSK, sSV, sp, wrow, g, t, t0, gm.r0, r1l, tq, voff, st);
        }
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (h.tile < h.ntiles - 1) continue;

        // ---- unit epilogue: head-t partials of the 4 warps merged lane by lane in
        // two rounds through the staging area, then written to head t's slot
        float l = st.l;
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        float m = st.m;
        float* area = reinterpret_cast<float*>(shP) + hg * 2 * 32 * 18;  // the head group's [2][32][18]
        const auto put = [&](int slot) {
            float* a = area + (slot * 32 + lane) * 18;
            a[0] = m;
            a[1] = l;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
#pragma unroll
                for (int x = 0; x < 4; ++x) a[2 + 4 * ch + x] = st.o[ch][x];
        };
        const auto take = [&](int slot) {
            const float* a = area + (slot * 32 + lane) * 18;
            const float mo = a[0], lo = a[1];
            const float ms = fmaxf(m, mo);
            const float fa = fast_exp2(m - ms), fb = fast_exp2(mo - ms);
            l = l * fa + lo * fb;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch)
#pragma unroll
                for (int x = 0; x < 4; ++x) st.o[ch][x] = st.o[ch][x] * fa + a[2 + 4 * ch + x] * fb;
            m = ms;
        };
        named_barrier_sync(1, kConsumerThreads);  // all warps done with their staging
        if (rw >= 2) put(rw - 2);
        named_barrier_sync(1, kConsumerThreads);
        if (rw < 2) take(rw);
        named_barrier_sync(1, kConsumerThreads);
        if (rw == 1) put(0);
        named_barrier_sync(1, kConsumerThreads);
        if (rw == 0 && 4 * hg + t < G) {  // idle head slots (G = 2) write nothing
            take(0);
            float* slot = p.ws + (((size_t)gm.h * G + 4 * hg + t) * p.S + gm.s) * (D + 2);
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                const int d0 = 2 * (16 * ch + g), d1 = 2 * (16 * ch + g + 8);
                *reinterpret_cast<float2*>(slot + 2 + d0) = make_float2(st.o[ch][0], st.o[ch][1]);
                *reinterpret_cast<float2*>(slot + 2 + d1) = make_float2(st.o[ch][2], st.o[ch][3]);
            }
            if (g == 0) {
                slot[0] = m * kLn2;  // natural-log units, as the reference's slots
                slot[1] = l;
            }
        }
        if (tickets) {
            if (!ring_slot_free()) {
                if (lane == 0) {
                    report_error(kErrFullWait);
                    *shFail = 1;
                }
            }
            hand_over(gm.h);
        } else {
            named_barrier_sync(1, kConsumerThreads);
        }
    }
    if (tickets && ring_slot_free()) hand_over(-1);
}

}  // namespace va
