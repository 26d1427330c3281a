// Split-L exchange over NVLink peer memory (plain 8-byte stores into buffers
// mapped into every rank's address space; no TMA, no multicast, no fences).
//
// Each rank holds a gather buffer of tagged words [2][R][H][D+2] (double-
// buffered by epoch parity). A tagged word is 64 bits: the low half a float
// of a partial (m, l, o[0..D)), the high half the epoch that wrote it. For
// head h, a rank stores its partial into slot [par][rank][h] of every rank's
// buffer, one 64-bit store per value; a reader polls each word of the R slots
// of its own buffer until the tag equals the step's epoch. An aligned 64-bit
// store is performed as one access, so a word whose tag matches carries that
// step's value: no flag, no fence and no acquire are needed (the flag-in-the-
// data idea of low-latency collective protocols). The merge is the
// log-sum-exp of the reference's combine (src/voltattn.cu:651-672), applied
// rank by rank as an online rescale.
//
// A rank writes epoch e+2 into a parity half only after its merge of e+1 saw
// every peer's e+1 words, which each peer wrote after finishing its merge of
// e, so a half is never overwritten while it is read. Epochs start at 1 and
// the buffers are zeroed once, so a word never carries a tag it was not
// written with. A wait that runs out records kErrPeerWait and leaves the
// head's output untouched.
#pragma once

#include "common.cuh"

namespace va {

constexpr int kMaxRanks = 8;

struct PeerBuffers {
    unsigned long long* gather[kMaxRanks];  // rank r's tagged words [2][R][H][D+2]
};

__device__ __forceinline__ void store_tagged_sys(unsigned long long* p, float v, unsigned tag) {
    const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long load_tagged_sys(const unsigned long long* p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Polls one tagged word until its tag is `tag`; false once the wall-clock
// budget that started at the first miss (t0, 0 = not started) runs out.
__device__ __forceinline__ bool poll_tagged(const unsigned long long* p, unsigned tag, uint64_t wait_ns,
                                            uint64_t& t0, float& v) {
    unsigned long long w = load_tagged_sys(p);
    for (uint32_t i = 1; (unsigned)(w >> 32) != tag; ++i) {
        if ((i & 63u) == 0) {
            const uint64_t now = global_timer_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > wait_ns) return false;
        }
        w = load_tagged_sys(p);
    }
    v = __uint_as_float((unsigned)w);
    return true;
}

// The exchange of one head by nthr threads of a CTA: thread `tid` holds the
// dims d0 + j * dstride (j < J; dims >= D are not held) of this rank's
// partial (m in natural-log units). `sync` synchronises the nthr threads;
// `shok` is a shared word; wait_ns bounds the wait for the peers' words.
// Returns the merged output dims in o (normalised), false on a failed wait.
template <int J, class Sync>
__device__ __forceinline__ bool peer_exchange_head(const PeerBuffers& x, int R, int rank, unsigned epoch,
                                                   uint64_t wait_ns, int H, int D, int h, float m, float l,
                                                   float (&o)[J], int d0, int dstride, int tid, Sync sync,
                                                   volatile int* shok) {
    const int par = (int)(epoch & 1u);
    const size_t slot_w = (size_t)(D + 2);
    const size_t buf_w = (size_t)R * H * slot_w;
    if (tid == 0) *shok = 1;
    sync();
    for (int r = 0; r < R; ++r) {
        unsigned long long* dst = x.gather[r] + par * buf_w + ((size_t)rank * H + h) * slot_w;
#pragma unroll
        for (int j = 0; j < J; ++j)
            if (d0 + j * dstride < D) store_tagged_sys(dst + 2 + d0 + j * dstride, o[j], epoch);
        if (tid == 0) {
            store_tagged_sys(dst, m, epoch);
            store_tagged_sys(dst + 1, l, epoch);
        }
    }
    const unsigned long long* g = x.gather[rank] + par * buf_w;
    float ms = kNegMax, ls = 0.f, acc[J];
#pragma unroll
    for (int j = 0; j < J; ++j) acc[j] = 0.f;
    uint64_t t0 = 0;
    bool ok = true;
    for (int r = 0; r < R && ok; ++r) {
        const unsigned long long* sp = g + ((size_t)r * H + h) * slot_w;
        float mr, lr, orr[J];
        ok = poll_tagged(sp, epoch, wait_ns, t0, mr) && poll_tagged(sp + 1, epoch, wait_ns, t0, lr);
#pragma unroll
        for (int j = 0; j < J; ++j) {
            orr[j] = 0.f;
            if (ok && d0 + j * dstride < D) ok = poll_tagged(sp + 2 + d0 + j * dstride, epoch, wait_ns, t0, orr[j]);
        }
        if (!ok) break;
        const float nm = fmaxf(ms, mr);
        const float c = fast_exp2((ms - nm) * kLog2e);  // 0 while ms is the empty -FLT_MAX
        const float a = fast_exp2((mr - nm) * kLog2e);
        ls = fmaf(lr, a, ls * c);
#pragma unroll
        for (int j = 0; j < J; ++j) acc[j] = fmaf(orr[j], a, acc[j] * c);
        ms = nm;
    }
    if (!ok) {
        *shok = 0;
        report_error(kErrPeerWait);
    }
    sync();
    if (!*shok) return false;
    const float inv = 1.f / ls;
#pragma unroll
    for (int j = 0; j < J; ++j) o[j] = acc[j] * inv;
    return true;
}

}  // namespace va
