// Tensor-core decode kernel for the quantized "+" formats (q8+, q4+, q3+),
// batch-1 multi-head (G = 1) and grouped-query (G = 2, 4, 8).
//
// Same math and the same streaming front end as decode_stream.cuh (persistent
// CTAs over (KV stream, split) units, producer warp, cp.async.bulk ring on
// mbarriers, fused last-CTA combine); the consumer warps instead run the two
// contractions on the tensor cores with integer mma.sync (m16n8k32, int32
// accumulation, exact):
//
//   scores  S[16 rows x 8] = K[16 rows x 32 dims] . Q[32 dims x 8]
//           Q's 8 columns are (query head, byte plane) pairs: q is 16-bit
//           fixed point split into two signed byte planes (q = 256 hi + lo),
//           so one mma scores 16 rows for 4 query heads at once.
//   output  O^T[16 dims x 8] += V^T[16 dims x 32 rows] . P[32 rows x 8]
//           P's columns are (query head, byte plane) pairs of the softmax
//           weights e_j * vs_j as 15-bit fixed point relative to the 32-row
//           block's maximum (per head and quant group).
//
// Fragment mapping (g = lane / 4, t = lane % 4):
//   * K operand: row g and g+8 of a 16-row group; the 32 dims of k-step
//     s = 2*gi + h are 64*gi + 16*t + word_dim(2h (+1), j): each thread
//     reads one 16-dim slice of a row per quant group (the integer lane
//     words of decode_stream.cuh), and a k-step never crosses a quant group,
//     so every scores accumulator has one K scale per row.
//   * V operand: m-tile mt of quant group gi = mt / 4 holds dims
//     64*gi + 8*g + 2*(mt%4) (row g) and the next dim (row g+8): each
//     thread reads one 8-dim chunk of 4 rows and byte-transposes it (prmt),
//     which turns row-major V into the k-major A fragment without a
//     shared-memory round trip.
//   * P operand: written per warp to a 512-byte staging area by the threads
//     that own the scores (thread t owns head t [+4]) and read back as 4-row
//     words.
// With G <= 4 every head of a group is handled in the same instructions
// (thread t carries head t), so the per-row cost does not grow with G.
#pragma once

#include "decode_stream.cuh"

namespace va {

template <Kind K, int D, int G>
struct MmaCfg {
    static constexpr Kind kKind = K;
    static constexpr int kD = D;
    static constexpr int kG = G;
    static constexpr int kBits = KindTraits<K>::kBits;
    static constexpr int kNgrp = D / kGroup;                       // quant groups per row
    static constexpr int kNq = (G + 3) / 4;                        // n-blocks of 4 heads
    static constexpr int kWarps = (K == Kind::Q8 && D == 128) ? 4 : 8;
    static constexpr int kBpw = (K != Kind::Q8 && D == 64) ? 2 : 1;  // 32-row blocks per warp per tile
    static constexpr int kThreads = (kWarps + 1) * 32;
    static constexpr int kTr = kWarps * kBpw * 32;
    static constexpr int kRb = D * kBits / 8;
    static constexpr int kSb = 2 * kNgrp;
    static constexpr int kStages = 3;
    static constexpr int kStageBytes = 2 * kTr * kRb + 2 * kTr * kSb;
    static constexpr int kMergeFloats = kWarps * (D + 2);
    static constexpr int kPStage = kNq * kNgrp * 8 * 32;  // bytes per warp: [nq][gi][col][32 rows]
    static constexpr int kSmemBytes =
        kStages * kStageBytes + 2 * kStages * 8 + kMergeFloats * 4 + kWarps * kPStage + 16;
    // (kTr, kRb, kSb, kStages, kStageBytes are what the shared producer uses)
    static_assert(kTr % 8 == 0 && (kTr * kRb) % 16 == 0 && (kTr * kSb) % 16 == 0, "aligned stages");
    static_assert(kMergeFloats >= kWarps * 32 + 64, "merge area doubles as combine scratch");
};

// ---- mma.sync wrappers (m16n8k32, int8 x int8 -> int32) -------------------------

template <bool kASigned, bool kBSigned>
__device__ __forceinline__ void mma_k32(int* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
#define VA_MMA(TA, TB)                                                                                        \
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." TA "." TB                                         \
                 ".s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"                                 \
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])                                            \
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1))
    if constexpr (kASigned && kBSigned) VA_MMA("s8", "s8");
    else if constexpr (kASigned) VA_MMA("s8", "u8");
    else if constexpr (kBSigned) VA_MMA("u8", "s8");
    else VA_MMA("u8", "u8");
#undef VA_MMA
}

template <class C>
struct MmaQ {
    uint32_t b[C::kNq][2 * C::kNgrp][2];  // K-step B fragments (q planes) of this thread's column
    int bias[C::kNq][C::kNgrp];           // code offset * sum of q over the group (thread's head t)
    float qscale[C::kNq];                 // 2^-e * log2(e)/sqrt(D) of the thread's head
};

// Per-unit query preparation, per warp (no CTA barrier): each warp derives
// the per-head exponent (|q| * 2^e < 2^14 over the head) of the group's
// heads with shuffles, then every thread builds the B fragments of its column
// (head 4*nq + g/2, byte plane g%2) and the bias / scale of its own head
// (4*nq + t) straight from the fp16 query (L1-resident after the first warp).
template <class C>
__device__ __forceinline__ void mma_load_q(MmaQ<C>& mq, const __half* q, int h, int g, int t, int lane) {
    constexpr int D = C::kD, G = C::kG, H4 = 4 * C::kNq;
    const float base = rsqrtf((float)D) * kLog2e;
    const __half* qh = q + (size_t)h * G * D;
    int ex[H4];
    int gs[H4][C::kNgrp];
#pragma unroll
    for (int hq = 0; hq < H4; ++hq) {
        float amax = 0.f;
        if (hq < G) {
#pragma unroll
            for (int d = lane; d < D; d += 32) amax = fmaxf(amax, fabsf(__half2float(qh[hq * D + d])));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        int e = 0;
        if (amax > 0.f) {
            int x;
            frexpf(amax, &x);
            e = 14 - x;
        }
        ex[hq] = e;
#pragma unroll
        for (int gi = 0; gi < C::kNgrp; ++gi) {
            int sum = 0;
            if (hq < G) {
#pragma unroll
                for (int d = lane; d < kGroup; d += 32)
                    sum += __float2int_rn(ldexpf(__half2float(qh[hq * D + 64 * gi + d]), e));
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            gs[hq][gi] = sum;
        }
    }
    const int offv = (C::kKind == Kind::Q4) ? 8 : (C::kKind == Kind::Q3) ? 4 : 0;
#pragma unroll
    for (int nq = 0; nq < C::kNq; ++nq) {
        // the thread's column head (4nq + g/2) and its own head (4nq + t), by selection
        int ec = 0, eo = 0;
        int bo[C::kNgrp];
#pragma unroll
        for (int gi = 0; gi < C::kNgrp; ++gi) bo[gi] = 0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if ((g >> 1) == k) ec = ex[4 * nq + k];
            if (t == k) {
                eo = ex[4 * nq + k];
#pragma unroll
                for (int gi = 0; gi < C::kNgrp; ++gi) bo[gi] = gs[4 * nq + k][gi];
            }
        }
        const int hc = 4 * nq + (g >> 1), plane = g & 1;
#pragma unroll
        for (int gi = 0; gi < C::kNgrp; ++gi) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t w = 0;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int d = 64 * gi + 16 * t + word_dim<C::kKind>(2 * hh + half, j);
                        const int v = hc < G ? __float2int_rn(ldexpf(__half2float(qh[hc * D + d]), ec)) : 0;
                        const int hi = (v + 128) >> 8;  // balanced split: v = 256 hi + lo, lo in [-128, 127]
                        const int lo = v - 256 * hi;
                        w |= (uint32_t)((plane ? lo : hi) & 0xFF) << (8 * j);
                    }
                    mq.b[nq][2 * gi + hh][half] = w;
                }
            }
            mq.bias[nq][gi] = offv * bo[gi];
        }
        mq.qscale[nq] = ldexpf(base, -eo);
    }
}

// q3: the 24-bit granule starting at byte p (any alignment) as a word.
__device__ __forceinline__ uint32_t load_granule(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16);
}

// V operand words of one thread for one quant group and the 4 rows
// rowq + r*rstride: out[2*j] / out[2*j+1] = dims 8g+2j / 8g+2j+1 of the 4 rows
// (byte lane r = row r).
template <class C>
__device__ __forceinline__ void mma_v_words(const uint8_t* sV, int rowq, int rstride, int gi, int g,
                                            uint32_t* out) {
    constexpr int kRb = C::kRb;
    if constexpr (C::kKind == Kind::Q8) {
        uint2 c[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            c[r] = *reinterpret_cast<const uint2*>(sV + (size_t)(rowq + r * rstride) * kRb + 64 * gi + 8 * g);
        uint32_t t0[4], t1[4];
        transpose4x4(c[0].x, c[1].x, c[2].x, c[3].x, t0);
        transpose4x4(c[0].y, c[1].y, c[2].y, c[3].y, t1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            out[j] = t0[j];
            out[4 + j] = t1[j];
        }
    } else if constexpr (C::kKind == Kind::Q4) {
        uint32_t c[4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
            c[r] = *reinterpret_cast<const uint32_t*>(sV + (size_t)(rowq + r * rstride) * kRb + 32 * gi + 4 * g);
        uint32_t tt[4];
        transpose4x4(c[0], c[1], c[2], c[3], tt);  // tt[j] = byte j (dims 2j, 2j+1) of the 4 rows
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            out[2 * j] = tt[j] & 0x0F0F0F0Fu;
            out[2 * j + 1] = (tt[j] >> 4) & 0x0F0F0F0Fu;
        }
    } else {
        uint32_t e[4], o[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t gr = load_granule(sV + (size_t)(rowq + r * rstride) * kRb + 24 * gi + 3 * g);
            e[r] = spread_q3(gr);       // fields 0, 2, 4, 6
            o[r] = spread_q3(gr >> 3);  // fields 1, 3, 5, 7
        }
        uint32_t te[4], to[4];
        transpose4x4(e[0], e[1], e[2], e[3], te);
        transpose4x4(o[0], o[1], o[2], o[3], to);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            out[2 * j] = te[j];
            out[2 * j + 1] = to[j];
        }
    }
}

template <class C>
struct MmaState {
    float m[C::kNq], l[C::kNq];
    float o[C::kNq][2 * C::kNgrp * 8];  // dims (mt, g) and (mt, g+8) for the m-tiles of each group
};

// One 32-row block (tile rows rb*32 .. rb*32+31) of the thread's heads.
template <class C, bool kMasked>
__device__ __forceinline__ void mma_block(const uint8_t* stage, int rb, int g, int t, long long t0, long long r0,
                                          long long r1, const MmaQ<C>& mq, MmaState<C>& st, uint8_t* sp) {
    constexpr int kG2 = C::kNgrp;
    constexpr bool kSignedCodes = C::kKind == Kind::Q8;
    const uint8_t* sK = stage;
    const uint8_t* sV = sK + C::kTr * C::kRb;
    const __half* sSK = reinterpret_cast<const __half*>(sV + C::kTr * C::kRb);
    const __half* sSV = sSK + C::kTr * kG2;
    const int row0 = rb * 32;

    // ---- scores: rows row0 + 16*i + g (+8) -----------------------------------------
    float s[C::kNq][4];  // [nq][i*2 + (0: row g, 1: row g+8)]
    bool valid[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int ra = row0 + 16 * i + g, rbw = ra + 8;
        valid[2 * i] = true;
        valid[2 * i + 1] = true;
        if constexpr (kMasked) {
            valid[2 * i] = (t0 + ra >= r0) && (t0 + ra < r1);
            valid[2 * i + 1] = (t0 + rbw >= r0) && (t0 + rbw < r1);
        }
        int acc[C::kNq][kG2][4];
#pragma unroll
        for (int nq = 0; nq < C::kNq; ++nq)
#pragma unroll
            for (int gi = 0; gi < kG2; ++gi)
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[nq][gi][k] = 0;
#pragma unroll
        for (int gi = 0; gi < kG2; ++gi) {
            IntWords<C::kKind> wa, wb;
            const int sliceb = (64 * gi + 16 * t) * C::kBits / 8;
            load_int_words<C::kKind>(wa, sK + (size_t)ra * C::kRb + sliceb);
            load_int_words<C::kKind>(wb, sK + (size_t)rbw * C::kRb + sliceb);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                for (int nq = 0; nq < C::kNq; ++nq)
                    mma_k32<kSignedCodes, true>(acc[nq][gi], wa.w[2 * hh], wb.w[2 * hh], wa.w[2 * hh + 1],
                                                wb.w[2 * hh + 1], mq.b[nq][2 * gi + hh][0], mq.b[nq][2 * gi + hh][1]);
            }
        }
        float ks[2][kG2];
#pragma unroll
        for (int gi = 0; gi < kG2; ++gi) {
            ks[0][gi] = __half2float(sSK[ra * kG2 + gi]);
            ks[1][gi] = __half2float(sSK[rbw * kG2 + gi]);
        }
#pragma unroll
        for (int nq = 0; nq < C::kNq; ++nq) {
            float sa = 0.f, sb = 0.f;
#pragma unroll
            for (int gi = 0; gi < kG2; ++gi) {
                // columns 2t (hi plane), 2t+1 (lo plane) of head 4*nq + t
                const int xa = acc[nq][gi][0] * 256 + acc[nq][gi][1] - mq.bias[nq][gi];
                const int xb = acc[nq][gi][2] * 256 + acc[nq][gi][3] - mq.bias[nq][gi];
                sa = fmaf((float)xa, ks[0][gi], sa);
                sb = fmaf((float)xb, ks[1][gi], sb);
            }
            s[nq][2 * i] = valid[2 * i] ? sa * mq.qscale[nq] : -INFINITY;
            s[nq][2 * i + 1] = valid[2 * i + 1] ? sb * mq.qscale[nq] : -INFINITY;
        }
    }

    // ---- online softmax over the block, per head ----------------------------------------
    float vs[4][kG2];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int row = row0 + 16 * (r >> 1) + g + 8 * (r & 1);
#pragma unroll
        for (int gi = 0; gi < kG2; ++gi) vs[r][gi] = __half2float(sSV[row * kG2 + gi]);
    }
    float c[C::kNq];
    int psum[C::kNq][kG2];
    float wscale[C::kNq][kG2];
#pragma unroll
    for (int nq = 0; nq < C::kNq; ++nq) {
        float bm = fmaxf(fmaxf(s[nq][0], s[nq][1]), fmaxf(s[nq][2], s[nq][3]));
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, off));
        const float mnew = fmaxf(st.m[nq], bm);
        c[nq] = fast_exp2(st.m[nq] - mnew);
        st.m[nq] = mnew;
        float e[4], esum = 0.f;
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            e[r] = fast_exp2(s[nq][r] - mnew);
            esum += e[r];
        }
        st.l[nq] = st.l[nq] * c[nq] + esum;
#pragma unroll
        for (int gi = 0; gi < kG2; ++gi) {
            float w[4], wm = 0.f;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                w[r] = e[r] * vs[r][gi];
                if constexpr (kMasked) w[r] = valid[r] ? w[r] : 0.f;
                wm = fmaxf(wm, w[r]);
            }
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, off));
            const float inv = wm > 0.f ? 32767.f / wm : 0.f;
            wscale[nq][gi] = wm * (1.f / 32767.f);
            int ps = 0;
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int p = float_to_small_int_rn(w[r] * inv);  // 0..32767
                ps += p;
                const int row = 16 * (r >> 1) + g + 8 * (r & 1);
                uint8_t* col = sp + ((nq * kG2 + gi) * 8 + 2 * t) * 32;  // column 2t (hi), 2t+1 (lo)
                const int kp = (row & 16) | (4 * (row & 3) + ((row >> 2) & 3));  // k position of this row
                col[kp] = (uint8_t)(p >> 8);
                col[32 + kp] = (uint8_t)(p & 0xFF);
            }
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            psum[nq][gi] = ps;
        }
    }
    __syncwarp();

    // ---- output: O^T += V^T . P per quant group -------------------------------------------
#pragma unroll
    for (int gi = 0; gi < kG2; ++gi) {
        uint32_t pb[C::kNq][2];
#pragma unroll
        for (int nq = 0; nq < C::kNq; ++nq) {
            const uint8_t* col = sp + ((nq * kG2 + gi) * 8 + g) * 32;
            pb[nq][0] = *reinterpret_cast<const uint32_t*>(col + 4 * t);
            pb[nq][1] = *reinterpret_cast<const uint32_t*>(col + 16 + 4 * t);
        }
        uint32_t va_[8], vb_[8];  // rows 4t..4t+3 and 16+4t..16+4t+3
        // k = 4t + r of each 16-row half is tile row 4r + t: for a fixed r the
        // 4 values of t read 4 consecutive rows, which halves the bank
        // conflicts of 64-byte rows against a stride of 4 rows
        mma_v_words<C>(sV, row0 + t, 4, gi, g, va_);
        mma_v_words<C>(sV, row0 + 16 + t, 4, gi, g, vb_);
        const int offv = (C::kKind == Kind::Q4) ? 8 : (C::kKind == Kind::Q3) ? 4 : 0;
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
            for (int nq = 0; nq < C::kNq; ++nq) {
                int acc[4] = {0, 0, 0, 0};
                mma_k32<kSignedCodes, false>(acc, va_[2 * mt], va_[2 * mt + 1], vb_[2 * mt], vb_[2 * mt + 1],
                                             pb[nq][0], pb[nq][1]);
                // rows g (dim 64gi + 8g + 2mt) / g+8 (next dim); cols 2t, 2t+1 = head t planes
                const int xa = acc[0] * 256 + acc[1] - offv * psum[nq][gi];
                const int xb = acc[2] * 256 + acc[3] - offv * psum[nq][gi];
                float* o = &st.o[nq][gi * 8 + 2 * mt];
                o[0] = fmaf((float)xa, wscale[nq][gi], o[0] * c[nq]);
                o[1] = fmaf((float)xb, wscale[nq][gi], o[1] * c[nq]);
            }
        }
    }
    __syncwarp();
}

template <class C>
__global__ void __launch_bounds__(C::kThreads, 2) decode_mma_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int D = C::kD;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
    uint64_t* empty = full + C::kStages;
    float* shMerge = reinterpret_cast<float*>(empty + C::kStages);  // [warps][D+2]
    uint8_t* shP = reinterpret_cast<uint8_t*>(shMerge + C::kMergeFloats);
    int* shTicket = reinterpret_cast<int*>(shP + C::kWarps * C::kPStage);
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
    grid_dependency_wait();
    if (threadIdx.x == 0) grid_launch_dependents();

    if (warp == C::kWarps) {
        stream_producer<C>(p, smem, full, empty);
        return;
    }

    constexpr int kConsumerThreads = C::kWarps * 32;
    const int g = lane >> 2, t = lane & 3, tid = threadIdx.x;
    const int nunits = p.H * p.S;
    uint8_t* sp = shP + warp * C::kPStage;
    MmaQ<C> mq;
    int cur_h = -1;
    int k = 0;
    for (int u = unit_begin(nunits), ue = unit_begin(nunits, 1); u < ue; ++u) {
        bool failed = false;
        const UnitGeom gm = unit_geom<C>(p, u);
        if (gm.h != cur_h) {
            mma_load_q<C>(mq, p.q, gm.h, g, t, lane);
            cur_h = gm.h;
        }
        MmaState<C> st;
#pragma unroll
        for (int nq = 0; nq < C::kNq; ++nq) {
            st.m[nq] = kNegMax;
            st.l[nq] = 0.f;
#pragma unroll
            for (int d = 0; d < 16 * C::kNgrp; ++d) st.o[nq][d] = 0.f;
        }
        for (int ti = 0; ti < gm.ntiles && !failed; ++ti, ++k) {
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
            const long long t0 = gm.a0 + (long long)ti * C::kTr;
            const uint8_t* base = smem + (size_t)stage * C::kStageBytes;
            const bool interior = t0 >= gm.r0 && t0 + C::kTr <= gm.r1;
#pragma unroll
            for (int j = 0; j < C::kBpw; ++j) {
                const int rb = warp * C::kBpw + j;
                if (interior)
                    mma_block<C, false>(base, rb, g, t, t0, gm.r0, gm.r1, mq, st, sp);
                else
                    mma_block<C, true>(base, rb, g, t, t0, gm.r0, gm.r1, mq, st, sp);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
        }

        // ---- merge: per query head, warps -> slot ----------------------------------------
        for (int hq = 0; hq < C::kG; ++hq) {
            const int nq = hq >> 2;
            float lw = st.l[nq];
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) lw += __shfl_xor_sync(0xffffffffu, lw, off);
            if (t == (hq & 3)) {
                float* row = shMerge + warp * (D + 2);
#pragma unroll
                for (int gi = 0; gi < C::kNgrp; ++gi)
#pragma unroll
                    for (int mt = 0; mt < 4; ++mt) {
                        const int d0 = 64 * gi + 8 * g + 2 * mt;
                        row[2 + d0] = st.o[nq][gi * 8 + 2 * mt];
                        row[2 + d0 + 1] = st.o[nq][gi * 8 + 2 * mt + 1];
                    }
                if (g == 0) {
                    row[0] = st.m[nq];
                    row[1] = lw;
                }
            }
            named_barrier_sync(1, kConsumerThreads);
            if (tid < D) {
                float ms = kNegMax;
                for (int w = 0; w < C::kWarps; ++w) ms = fmaxf(ms, shMerge[w * (D + 2)]);
                float ls = 0.f, od = 0.f;
                for (int w = 0; w < C::kWarps; ++w) {
                    const float a = fast_exp2(shMerge[w * (D + 2)] - ms);
                    ls += shMerge[w * (D + 2) + 1] * a;
                    od += shMerge[w * (D + 2) + 2 + tid] * a;
                }
                float* slot = p.ws + (((size_t)gm.h * C::kG + hq) * p.S + gm.s) * (D + 2);
                slot[2 + tid] = od;
                if (tid == 0) {
                    slot[0] = ms * kLn2;
                    slot[1] = ls;
                }
            }
            named_barrier_sync(1, kConsumerThreads);
        }
        if (p.out_mode != kOutSlots) {
            if (tid == 0) *shTicket = (int)atomic_add_acq_rel_gpu(&p.counters[gm.h], 1u);
            named_barrier_sync(1, kConsumerThreads);
            if (*shTicket == p.S - 1) {
                for (int hq = 0; hq < C::kG; ++hq) {
                    const size_t hg = (size_t)gm.h * C::kG + hq;
                    const float* hs = p.ws + hg * p.S * (D + 2);
                    float ms, ls, od;
                    lse_merge([&](int i) { return hs + (size_t)i * (D + 2); }, p.S, D, tid, kConsumerThreads,
                              LseScratch{shMerge, shMerge + kConsumerThreads},
                              [] { named_barrier_sync(1, kConsumerThreads); }, ms, ls, od);
                    if (tid < D) {
                        if (p.out_mode == kOutHalf) {
                            p.out[hg * D + tid] = __float2half_rn(od / ls);
                        } else {
                            float* pp = p.partial + hg * (D + 2);
                            pp[2 + tid] = od;
                            if (tid == 0) {
                                pp[0] = ms;
                                pp[1] = ls;
                            }
                        }
                    }
                }
                if (tid == 0) store_relaxed_gpu(&p.counters[gm.h], 0u);
            }
        }
        named_barrier_sync(1, kConsumerThreads);
        if (*shFail) break;
    }
}

}  // namespace va
