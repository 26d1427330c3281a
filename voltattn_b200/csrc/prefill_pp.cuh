// Staged prefill, ping-pong form: two query tiles per CTA whose softmax
// phases alternate against one tensor-core issuer, so the tensor pipe works on
// one tile while the other tile's softmax runs.
//
// Same problem and math as prefill_tc.cuh (the reference's per-row
// attention, src/voltattn.cu:769-794, over the dequantized cache,
// src/voltattn.cu:747-767), over the fp16 staging rows that
// prefill_stage_kernel writes once per call.
//
// One CTA per (query head, pair of 128-token tiles), 1 CTA per SM, 10 warps:
//   warps 0-3  softmax of tile 0, warps 4-7 softmax of tile 1: thread r of a
//              warpgroup owns token row r (TMEM lane r) of its tile, so the
//              row maximum needs no exchange between threads;
//   warp 8     one thread issues every tcgen05.mma;
//   warp 9     one thread issues every tensor copy.
// (Three warps per SM sub-partition cap registers at 168 per thread; a whole
// row of S, 128 values, stays in registers.)
// Tensor memory (512 columns, the whole SM's): S0 [0,128), S1 [128,256),
// O0 [256,384), O1 [384,512); P(kb) of tile w overlays the first 64 columns
// of S_w as fp16 pairs (column c = keys 2c, 2c+1) and is the A operand of
// O_w += P V read from TMEM.
// Shared memory: Q0, Q1 and a ring of 5 K/V tiles (items K(0), V(0), K(1),
// V(1), ... in order), each a 128 x 128 fp16 tile in the canonical 128-byte
// swizzled layout (two 64-dim panels), 224 KB in all.
// MMA order: S0(0) S1(0), then per block kb: PV0(kb) S0(kb+1) PV1(kb)
// S1(kb+1). PV_w(kb) waits for tile w's P(kb); S_w(kb+1) overwrites the
// columns PV_w(kb) reads, which is safe because the MMAs of one thread execute
// in issue order. A K tile is free once S1 has read it, a V tile once PV1 has.
// The softmax of tile w at block kb runs after S_w(kb) completed, and with it
// every earlier MMA (PV_w(kb-1) included), so it may rescale O_w in TMEM
// without a race. Every mbarrier wait is bounded (va_device_error on expiry).
#pragma once

#include "prefill_tc.cuh"

namespace va {

// Development builds (-DPF_TIMELINE): per-CTA cycle totals of the phases below
// into g_pf_tl (read back by va_debug_pf_timeline); absent in the product.
#ifdef PF_TIMELINE
extern __device__ unsigned long long g_pf_tl[4096 * 8];
#define PP_T(v) v = clock64()
// event log of CTA (0, 0): region r (0: tile 0 softmax, 1: tile 1, 2: MMA
// thread) of 8192 words: kind << 56 | kb << 40 | cycles since the start
#define PP_EV(r, kind, kb)                                                                          \
    do {                                                                                            \
        if (blockIdx.x == 0 && blockIdx.y == 0 && pp_nev < 8192)                                   \
            g_pf_tl[(r) * 8192 + pp_nev++] = ((unsigned long long)(kind) << 56) |                   \
                                             ((unsigned long long)(kb) << 40) |                     \
                                             (unsigned long long)(clock64() - tstart);              \
    } while (0)
#define PP_ACC(slot, a, b) do { pp_acc[slot] += (unsigned long long)((b) - (a)); } while (0)
#else
#define PP_T(v) do { } while (0)
#define PP_EV(r, kind, kb) do { } while (0)
#define PP_ACC(slot, a, b) do { } while (0)
#endif

struct PpCfg {
    static constexpr int kD = 128;
    static constexpr int kBq = 128;  // tokens per tile (MMA M)
    static constexpr int kBk = 128;  // cache rows per block
    static constexpr int kTile = kBq * kD * 2;
    static constexpr int kRing = 5;  // K/V tiles in flight
    static constexpr int kThreads = 10 * 32;
    static constexpr int kBars = 2 * kRing + 2 + 2 + 2 + 1;
    static constexpr int kSmemBytes = 1024 + (2 + kRing) * kTile + kBars * 8 + 16;
    static constexpr int kTmemCols = 512;
    static_assert(kSmemBytes <= 227 * 1024, "one CTA per SM");
};

__device__ __forceinline__ void tmem_st16_u(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// 8 consecutive fp32 columns of this thread's TMEM lane (with the wait), and
// the store back.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
                 "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7]))
                 : "memory");
}

// Bounded wait of the issue threads, which sit on the critical path of every
// hand-off: try_wait without a suspend-time hint. (With the 20 us hint of
// mbar_wait_bounded a wait took ~200 cycles even on a completed phase: 808
// against 867 TFLOP/s; a test_wait spin took issue slots from the softmax
// warps: 839.)
__device__ __forceinline__ bool pp_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool pp_wait(uint64_t* bar, uint32_t parity) {
    if (pp_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t i = 1;; ++i) {
        if (pp_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__global__ void __launch_bounds__(PpCfg::kThreads, 1)
    prefill_pp_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV, int Lpad) {
    using C = PpCfg;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* sQ = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sKV = sQ + 2 * C::kTile;
    uint64_t* full = reinterpret_cast<uint64_t*>(sKV + C::kRing * C::kTile);
    uint64_t* freeb = full + C::kRing;
    uint64_t* sfull = freeb + C::kRing;
    uint64_t* pready = sfull + 2;
    uint64_t* odone = pready + 2;
    uint64_t* fin = odone + 2;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(fin + 1);

    constexpr int D = C::kD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npair = (int)gridDim.x;
    const int qp = npair - 1 - (int)blockIdx.x;  // the longest (last) token pairs start first
    const int h = (int)blockIdx.y;
    const int hk = h / (p.Hq / p.Hkv);
    const int q0 = qp * 2 * C::kBq;
    const long long off0 = (long long)p.L - p.Lq;  // cache row of token 0
    // blocks of cache rows each tile sees (tile 1's tokens come later)
    const int nkb0 = (int)(min((long long)p.L - 1, off0 + q0 + C::kBq - 1) / C::kBk) + 1;
    const int nkb1 = (int)(min((long long)p.L - 1, off0 + q0 + 2 * C::kBq - 1) / C::kBk) + 1;
    const int ybase = hk * Lpad;  // staging row of the KV head's row 0
    const uint32_t sQa = smem_u32(sQ), sKVa = smem_u32(sKV);
    constexpr uint32_t kTileBytes = (uint32_t)C::kTile;

    if (warp == 0) tmem_alloc(tslot, C::kTmemCols);
    if (tid == 0) {
        for (int i = 0; i < C::kRing; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&freeb[i], 1);
        }
        for (int w = 0; w < 2; ++w) {
            mbar_init(&sfull[w], 1);
            mbar_init(&pready[w], 128);
            mbar_init(&odone[w], 1);
        }
        mbar_init(fin, 1);
        fence_mbar_init();
    }
    // the pair's query tokens -> sQ (rows past Lq are zero)
    for (int i = tid; i < 2 * C::kBq * 16; i += C::kThreads) {
        const int tile = i >> 11, r = (i >> 4) & 127, c = i & 15;
        const int tok = q0 + tile * C::kBq + r;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (tok < p.Lq) v = __ldg(reinterpret_cast<const uint4*>(p.q + ((size_t)h * p.Lq + tok) * D) + c);
        sts128_generic(sQ + tile * C::kTile, pf_off(r, c), v);
    }
    fence_proxy_async_smem();
    tc05_fence_before();
    __syncthreads();
    tc05_fence_after();
    const uint32_t tbase = *tslot;
#ifdef PF_TIMELINE
    unsigned long long pp_acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    long long t0, t1, t2, t3, t4;
    const long long tstart = clock64();
    int pp_nev = 0;
#endif

    if (warp == 9) {
        // ---- tensor copies: item n = K(n/2) (n even) or V(n/2) into ring slot n % kRing ----
        if (lane == 0) {
            prefetch_tensormap(&tmK);
            prefetch_tensormap(&tmV);
            const int nitems = 2 * nkb1;
            int n = 0;
            for (; n < nitems; ++n) {
                const int slot = n % C::kRing;
                if (n >= C::kRing && !pp_wait(&freeb[slot], (uint32_t)(n / C::kRing - 1) & 1u)) {
                    report_error(kErrEmptyWait);
                    break;
                }
                const CUtensorMap* map = (n & 1) ? &tmV : &tmK;
                const uint32_t dst = sKVa + (uint32_t)slot * kTileBytes;
                const int y = ybase + (n >> 1) * C::kBk;
                mbar_arrive_expect_tx(&full[slot], kTileBytes);
                pf_tma_2d(dst, map, 0, y, &full[slot]);
                pf_tma_2d(dst + 16384u, map, 64, y, &full[slot]);
            }
            // no copy may still be writing shared memory when the CTA exits
            for (int d = 1; d <= C::kRing && n - d >= 0; ++d) {
                const int m = n - d;
                mbar_wait_bounded(&full[m % C::kRing], (uint32_t)(m / C::kRing) & 1u);
            }
        }
    } else if (warp == 8) {
        // ---- tensor-core issue ----
        if (lane == 0) {
            constexpr uint32_t kIdescS = umma_idesc_f16(128, 128, false);
            constexpr uint32_t kIdescO = umma_idesc_f16(128, 128, true);
            bool ok = true;
            const auto wait_item = [&](int n) {
                PP_T(t2);
                const bool got = ok && pp_wait(&full[n % C::kRing], (uint32_t)(n / C::kRing) & 1u);
                PP_T(t3);
                PP_ACC(6, t2, t3);
                if (ok && !got) {
                    report_error(kErrFullWait);
                    ok = false;
                }
                return ok;
            };
            const auto issue_s = [&](int w, int kb) {  // S_w = Q_w K(kb)^T
                const uint32_t sKa = sKVa + (uint32_t)((2 * kb) % C::kRing) * kTileBytes;
                const uint32_t qa = sQa + (uint32_t)w * kTileBytes;
#pragma unroll
                for (int kk = 0; kk < D / 16; ++kk) {
                    const uint32_t o = (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32);
                    umma_f16(tbase + 128u * w, umma_desc_sw128(qa + o, 16, 1024), umma_desc_sw128(sKa + o, 16, 1024),
                             kIdescS, kk > 0);
                }
                umma_commit(&sfull[w]);
            };
            const auto issue_pv = [&](int w, int kb) {  // O_w += P_w V(kb)
                const uint32_t sVa = sKVa + (uint32_t)((2 * kb + 1) % C::kRing) * kTileBytes;
#pragma unroll
                for (int kk = 0; kk < C::kBk / 16; ++kk)
                    umma_f16_ts(tbase + 256u + 128u * w, tbase + 128u * w + 8u * kk,
                                umma_desc_sw128(sVa + (uint32_t)(kk * 16 * 128), 16384, 1024), kIdescO,
                                kb > 0 || kk > 0);
            };
            const auto wait_p = [&](int w, int kb) {
                PP_T(t0);
                const bool got = ok && pp_wait(&pready[w], (uint32_t)kb & 1u);
                PP_T(t1);
                PP_ACC(4 + w, t0, t1);
                if (ok && !got) {
                    report_error(kErrFullWait);
                    ok = false;
                }
                tc05_fence_after();
                return ok;
            };
            if (wait_item(0)) {
                issue_s(0, 0);
                issue_s(1, 0);
                umma_commit(&freeb[0]);
            }
            for (int kb = 0; ok && kb < nkb1; ++kb) {
                bool v_waited = false, k_waited = false;
                if (kb < nkb0) {
                    if (!wait_p(0, kb)) break;
                    PP_EV(2, 11, kb);
                    if (!wait_item(2 * kb + 1)) break;
                    v_waited = true;
                    PP_EV(2, 5, kb);
                    issue_pv(0, kb);
                    if (kb == nkb0 - 1) umma_commit(&odone[0]);
                    if (kb + 1 < nkb0) {
                        PP_EV(2, 12, kb);
                        if (!wait_item(2 * kb + 2)) break;
                        PP_EV(2, 13, kb);
                        k_waited = true;
                        issue_s(0, kb + 1);
                        PP_EV(2, 7, kb);
                    }
                }
                if (!wait_p(1, kb)) break;
                if (!v_waited && !wait_item(2 * kb + 1)) break;
                PP_EV(2, 8, kb);
                issue_pv(1, kb);
                umma_commit(&freeb[(2 * kb + 1) % C::kRing]);
                if (kb == nkb1 - 1) umma_commit(&odone[1]);
                if (kb + 1 < nkb1) {
                    if (!k_waited && !wait_item(2 * kb + 2)) break;
                    issue_s(1, kb + 1);
                    PP_EV(2, 10, kb);
                    umma_commit(&freeb[(2 * kb + 2) % C::kRing]);
                }
            }
            // every MMA issued has completed before the CTA frees tensor memory
            umma_commit(fin);
            mbar_wait_bounded(fin, 0);
#ifdef PF_TIMELINE
            const int cta = (int)(blockIdx.y * gridDim.x + blockIdx.x);
            (void)cta;
#endif
        }
    } else {
        // ---- softmax of tile w, token row r ----
        const int w = warp >> 2;
        const int r = tid & 127;
        const uint32_t lane_addr = (uint32_t)((warp & 3) * 32) << 16;
        const uint32_t tS = tbase + 128u * w + lane_addr, tO = tbase + 256u + 128u * w + lane_addr;
        const int tok = q0 + w * C::kBq + r;
        const long long vis = min(off0 + tok, (long long)p.L - 1);  // last visible cache row
        const float qk_scale = rsqrtf((float)D) * kLog2e;
        float m = kNegMax, l = 0.f;
        bool ok = true;
        const int nk = w ? nkb1 : nkb0;
        for (int kb = 0; kb < nk; ++kb) {
            PP_T(t0);
            const bool got_s = mbar_wait_bounded(&sfull[w], (uint32_t)kb & 1u);
            PP_T(t1);
            PP_ACC(0, t0, t1);
            PP_EV(w, 1, kb);
            if (!got_s) {
                if (lane == 0) report_error(kErrFullWait);
                ok = false;
                break;
            }
            tc05_fence_after();
            uint32_t s[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32_nowait(tS + 32u * c, s[c]);
            tmem_wait_ld_only();
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_tie32(s[c]);
            // last visible key of the block (negative: none)
            const int lim = (int)max(-1ll, min(vis - (long long)kb * C::kBk, (long long)C::kBk - 1));
            const bool fullrow = lim >= C::kBk - 1;
            PP_T(t2);
            PP_ACC(1, t1, t2);
            // keys past the last visible one: -inf, whose weight is exactly 0
            // (diagonal blocks only; the loops below are the same for all)
            if (!fullrow) {
#pragma unroll
                for (int j = 0; j < C::kBk; ++j)
                    if (j > lim) s[j >> 5][j & 31] = 0xFF800000u;
            }
            float bm0 = kNegMax, bm1 = kNegMax;
#pragma unroll
            for (int j = 0; j < C::kBk; j += 4) {
                bm0 = fmax3f(bm0, __uint_as_float(s[j >> 5][j & 31]), __uint_as_float(s[j >> 5][(j & 31) + 1]));
                bm1 = fmax3f(bm1, __uint_as_float(s[j >> 5][(j & 31) + 2]), __uint_as_float(s[j >> 5][(j & 31) + 3]));
            }
            // lazy rescaling: the reference maximum moves only when the block
            // exceeds it by more than 8 (log2 units), so weights stay <= 256
            const float bms = fmaxf(bm0, bm1) * qk_scale;
            const float mnew = bms > m + 8.f ? bms : m;
            const float corr = fast_exp2(m - mnew);
            m = mnew;
            // O_w has no MMA in flight here (S_w(kb) completed after PV_w(kb-1)):
            // rescale it before P(kb) lets PV start
            if (kb > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll 1
                for (int c = 0; c < 16; ++c) {
                    float o[8];
                    tmem_ld8(tO + 8u * c, o);
#pragma unroll
                    for (int i = 0; i < 8; ++i) o[i] *= corr;
                    tmem_st8(tO + 8u * c, o);
                }
            }
            float2 sum2[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                              make_float2(0.f, 0.f)};  // 4 chains: the adds do not serialize
            const float2 sc2 = make_float2(qk_scale, qk_scale), nm2 = make_float2(-mnew, -mnew);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t pw[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float2 x =
                        ffma2(make_float2(__uint_as_float(s[c][2 * i]), __uint_as_float(s[c][2 * i + 1])), sc2, nm2);
                    const float a = fast_exp2(x.x);
                    const float b = fast_exp2(x.y);
                    sum2[i & 3] = fadd2(sum2[i & 3], make_float2(a, b));
                    const __half2 hp = __floats2half2_rn(a, b);
                    pw[i] = *reinterpret_cast<const uint32_t*>(&hp);
                }
                tmem_st16_u(tS + 16u * c, pw);
            }
            // P(kb) written: this tile's PV may start
            tmem_wait_st();
            tc05_fence_before();
            mbar_arrive(&pready[w]);
            if ((tid & 127) == 0) PP_EV(w, 2, kb);
            const float2 sa = fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3]));
            l = l * corr + (sa.x + sa.y);
            PP_T(t3);
            PP_ACC(2, t2, t3);
            PP_T(t4);
            PP_ACC(3, t3, t4);
        }
#ifdef PF_TIMELINE
        if (tid == 0) {
            const int cta = (int)(blockIdx.y * gridDim.x + blockIdx.x);
            (void)cta;
        }
#endif
        // epilogue: O_w / l -> out once the tile's last PV completed
        if (ok && mbar_wait_bounded(&odone[w], 0u)) {
            tc05_fence_after();
            const float inv = 1.f / l;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                float o[32];
                tmem_ld32(tO + 32u * c, o);
                if (tok < p.Lq) {
                    uint4* dst = reinterpret_cast<uint4*>(p.out + ((size_t)h * p.Lq + tok) * D + 32 * c);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        uint32_t wv[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const __half2 hp = __floats2half2_rn(o[8 * q + 2 * i] * inv, o[8 * q + 2 * i + 1] * inv);
                            wv[i] = *reinterpret_cast<const uint32_t*>(&hp);
                        }
                        dst[q] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
                    }
                }
            }
        } else if (ok && lane == 0) {
            report_error(kErrFullWait);
        }
    }
    __syncwarp();
    tc05_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc05_fence_after();
        tmem_dealloc(tbase, C::kTmemCols);
    }
}

}  // namespace va
