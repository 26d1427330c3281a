// Block-wide log-sum-exp merge of n partial slots (m, l, o[D]) — the
// reference's combine (src/voltattn.cu:651-672) — parallel over slots:
//   m* = max_i m_i, l* = sum_i l_i e^(m_i - m*), o*[d] = sum_i o_i[d] e^(m_i - m*)
// Pass 1 reduces m* over all threads; pass 2 walks the slots in chunks of
// `nt`: each thread computes one slot's weight into shared memory, then the
// threads of dim d (two per dim when nt >= 2D) sum over the chunk with
// independent, coalesced loads. The reference loops over the slots serially,
// which costs one L2 round trip per slot.
#pragma once

#include "common.cuh"

namespace va {

struct LseScratch {
    float* a;    // nt floats: the chunk's slot weights
    float* red;  // 64 floats: reductions
};

// slot(i) returns a pointer to slot i (m in natural-log units). Returns the
// merged (m*, l*, o*[tid % D]) to every thread; o* is valid for tid < D.
template <class SlotFn, class Barrier>
__device__ __forceinline__ void lse_merge(SlotFn slot, int n, int D, int tid, int nt, LseScratch sc, Barrier bar,
                                          float& ms_out, float& ls_out, float& od_out) {
    const int lane = tid & 31, wid = tid >> 5, nw = nt >> 5;
    float ms = kNegMax;
    for (int i = tid; i < n; i += nt) ms = fmaxf(ms, __ldcg(slot(i)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ms = fmaxf(ms, __shfl_xor_sync(0xffffffffu, ms, off));
    if (lane == 0) sc.red[wid] = ms;
    bar();
    ms = kNegMax;
    for (int w = 0; w < nw; ++w) ms = fmaxf(ms, sc.red[w]);
    bar();

    const int halves = (nt >= 2 * D) ? 2 : 1;
    const int d = tid % D, part = tid / D;
    float ls = 0.f, od = 0.f;
    for (int c = 0; c < n; c += nt) {
        const int i = c + tid;
        float a = 0.f;
        if (i < n) {
            const float* sp = slot(i);
            a = fast_exp2((__ldcg(sp) - ms) * kLog2e);
            ls += __ldcg(sp + 1) * a;
        }
        sc.a[tid] = a;
        bar();
        if (part < halves) {
            const int cnt = min(nt, n - c);
#pragma unroll 4
            for (int j = part; j < cnt; j += halves) od += __ldcg(slot(c + j) + 2 + d) * sc.a[j];
        }
        bar();
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
    if (lane == 0) sc.red[wid] = ls;
    if (halves == 2 && part == 1) sc.a[d] = od;
    bar();
    ls = 0.f;
    for (int w = 0; w < nw; ++w) ls += sc.red[w];
    if (halves == 2 && part == 0) od += sc.a[d];
    bar();
    ms_out = ms;
    ls_out = ls;
    od_out = od;
}

}  // namespace va
