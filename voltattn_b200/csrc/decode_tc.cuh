// Tensor-core decode kernel for batch-1 multi-head decode (G = 1) of the
// quantized "+" formats at D = 128 (q4+, q8+).
//
// Same math as the reference's sub-warp kernels (src/voltattn.cu:425-561):
// per head, score_j = q.K_j/sqrt(D), online softmax, o = sum_j p_j V_j. The
// integer dot-product consumer (decode_stream.cuh) spends ~720 thread
// instructions per row on q4+, which makes it issue-bound below the HBM
// rate. This kernel moves both contractions onto int8 mma.sync and spreads
// the per-row softmax work over the lanes, for ~150 instructions per row.
//
// Front end. A producer warp takes (head, split) units from a global counter
// (dynamic schedule) and streams each as tiles of 256 rows through a 3-deep
// ring of shared-memory stages, telling the consumers which unit and tile a
// stage holds in a per-stage header: the unit's query, K and V codes by 2-D
// tensor copies (cp.async.bulk.tensor, 32-row boxes, no multicast) with the
// 64-/128-byte swizzle (the 16-byte chunk index of a row is XORed with bits
// 7.. of its shared-memory offset), scales by plain bulk copies, completing on
// mbarriers. Rows past the tensor's end come back as zeros from the tensor
// copy; the scale rows of the tensor's last partial 8-row block come from
// plain loads. The swizzle makes both access patterns below conflict-free.
//
// Consumers: 4 warps, 64 rows each per tile, in 4 blocks of 16 rows. With
// g = lane / 4 and t = lane % 4 (the mma fragment coordinates):
//
//   scores  one m16n8k32 per 32 codes: A = K rows (row g and g+8 of the
//           block; lane t reads the row's 16-byte chunk t (q4) or chunks t,
//           t+4 (q8) with one 128-bit load each), B = q as 16-bit fixed point
//           in two signed byte planes, columns arranged so that lane t of the
//           accumulator gets one (quant group, part) sum of the row. q4 codes
//           are two nibbles per byte: one mma takes the low nibbles
//           (raw & 0x0F0F0F0F) against q of the even dims and of the odd
//           dims, a second takes the raw bytes against q of the odd dims;
//           raw - lo = 16 * hi gives the odd dims' sum exactly.
//           A reduce-scatter over the 4 lanes of each quad (integer adds in
//           a group, then the two groups after their fp16 scales) leaves
//           lane t with the final scores of block t's two rows.
//   softmax per warp and tile (64 rows, 2 per lane): one max, exponentials,
//           the weights e_j * vs_j per quant group as 15-bit fixed point
//           relative to the tile's maximum (byte planes p = 256 hi + lo),
//           staged per warp as the B fragments of the output mma.
//   output  one m16n8k32 per 16 rows x chunk pair: A = V^T from
//           ldmatrix.m16n16.trans.b8 (k = row, m = byte), the two k-halves
//           taking two chunks of the same 16 rows, B = the weight planes in
//           columns 0,1 (first chunk) and 2,3 (second chunk); q4 again runs
//           a raw-byte and a low-nibble mma. Integer sums over the tile are
//           folded into the fp32 output once per tile.
//
// The last CTA to finish a head's splits (acquire-release ticket) merges the
// head's slots in one pass; every spin wait is bounded, as in the streaming
// kernel.
#pragma once

#include <cuda.h>

#include "decode_mma.cuh"
#include "decode_stream.cuh"

namespace va {

// Per-CTA event timeline for development builds (-DVA_TC_TIMELINE): eight
// %globaltimer words per CTA (16 slots), see VA_TL below; the array is defined in
// launch_tc.cu and read back by va_debug_tc_timeline. Absent in the product.
#ifdef VA_TC_TIMELINE
constexpr int kTlCtas = 1024;
extern __device__ unsigned long long g_tc_timeline[kTlCtas * 16];
#define VA_TL(slot, v) \
    do { if (blockIdx.x < kTlCtas) g_tc_timeline[blockIdx.x * 16 + (slot)] = (unsigned long long)(v); } while (0)
#else
#define VA_TL(slot, v) do { } while (0)
#endif

// kChan: K codes with static per-channel scales per head ([H][D], folded into
// the query once per unit) and V codes with one scale per row ([H][L]);
// otherwise fp16 scales per 64-element group of every K and V row.
template <Kind K, int D, bool kChanScales = false>
struct TcCfg {
    static constexpr Kind kKind = K;
    static constexpr int kD = D;
    static constexpr int kG = 1;
    static constexpr bool kChan = kChanScales;
    static constexpr int kBits = KindTraits<K>::kBits;
    // q3 and q4 codes both run the two-field-per-byte path (kNib): q4 bytes
    // hold two nibbles, q3 granules are widened to two 3-bit fields per byte
    static constexpr bool kNib = K == Kind::Q4 || K == Kind::Q3;
    static constexpr int kRb = D * kBits / 8;  // code bytes per row (global rows, stages)
    // bytes per row of the swizzled compute tile: the stage itself, or for q3
    // the per-warp V buffer of widened rows (K is widened in registers)
    static constexpr int kRbT = K == Kind::Q3 ? D / 2 : kRb;
    static constexpr int kChunks = kRbT / 16;  // 16-byte chunks per compute row
    static constexpr int kPairs = kChunks / 2;
    static constexpr int kNgrp = D / kGroup;
    static constexpr int kSbK = kChan ? 0 : 2 * kNgrp;  // K scale bytes per row
    static constexpr int kSbV = kChan ? 2 : 2 * kNgrp;  // V scale bytes per row
    static constexpr int kSb = kSbV;
    // 4 consumer warps (q8+ with 2 warps and 128-row tiles at 2 CTAs per SM
    // measured slower: 26.1 against 24.5 us at L=16384)
    static constexpr int kWarps = 4;
    static constexpr int kRpw = 64;  // rows per warp per tile
    static constexpr int kTr = kWarps * kRpw;
    static constexpr int kBox = 32;  // rows per tensor copy
    // rows per tensor copy of a contiguous cache (64 and 128 measured
    // slower for batch-1 q4+ / q8+: 17.09 -> 17.29 / 17.34 us at L=16384)
    static constexpr int kBoxC = 32;
    static constexpr int kThreads = (kWarps + 2) * 32;  // consumers, producer, ticket warp
    static constexpr int kStages = 3;
    static constexpr int kTRing = 4;  // finished units handed to the ticket warp
    static constexpr int kStageBytes = (2 * kTr * kRb + kTr * (kSbK + kSbV) + 1023) & ~1023;
    static constexpr int kPStage = 4 * 2 * 5 * 4 * 8;  // per warp: [block][group][slot][t'] 8-byte B fragments
    static constexpr int kMergeFloats = kWarps * (D + 2);
    static constexpr int kQBytes = (kChan ? 2 : 1) * D * 2;  // the head's fp16 query (+ K channel scales)
    static constexpr int kVBuf = K == Kind::Q3 ? kWarps * kRpw * kRbT : 0;  // q3: widened V rows per warp
    static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kVBuf + 2 * kStages * 8 + kStages * 16 +
                                      kStages * kQBytes + kMergeFloats * 4 + kWarps * kPStage + 2 * kTRing * 8 +
                                      kTRing * 4 + 16 + 16 + kQBytes;
    static_assert(K == Kind::Q3 || K == Kind::Q4 || K == Kind::Q8, "integer 3-, 4- and 8-bit codes");
    static_assert(D == 128, "two quant groups per row");
    static_assert(kRbT == 64 || kRbT == 128, "swizzle span = row");
    static_assert(K != Kind::Q3 || !kChan, "q3 codes: per-group scales");
    static_assert(kMergeFloats >= kWarps * 32 + 64, "merge area doubles as combine scratch");
    static_assert(kTr % kBox == 0 && kBox % 8 == 0, "whole boxes of 8-row blocks");
    // 16-byte alignment of the bulk-copy targets carved after the stages
    static_assert((kStages * kStageBytes + kVBuf + 2 * kStages * 8 + kStages * 16) % 16 == 0, "query ring");
    static_assert(kVBuf % 1024 == 0, "stage alignment after the V buffers");
    static_assert((kStages * kQBytes + kMergeFloats * 4 + kWarps * kPStage + 2 * kTRing * 8 + kTRing * 4 + 16) %
                      16 == 0,
                  "first-unit query");
};

// ---- row placement --------------------------------------------------------------
// Row of a 16-row block held by mma row g (A) and g + 8 (B). Chosen so that the
// 128-bit K loads of quads (2i, 2i+1) hit different bank groups, and the rows
// one ldmatrix phase reads (k = 0..7 and 8..15 below) are distinct modulo 8
// (the swizzle period).
template <class C>
__host__ __device__ constexpr int tc_row_a(int q) {
    return C::kKind != Kind::Q8 ? q : ((q >> 1) | ((q & 1) << 2));
}
template <class C>
__host__ __device__ constexpr int tc_row_b(int q) {
    return 8 + tc_row_a<C>(q ^ 1);
}
// Output-mma k index k = 4t' + j (j = 0..3) of a 16-row block is row A (j even)
// or B (j odd) of quad q1(t') (j < 2) or q1(t') + 2 (j >= 2).
__host__ __device__ constexpr int tc_q1(int tp) { return 4 * (tp & 1) + (tp >> 1); }

// Byte offset of (row, 16-byte chunk) in a swizzled tile whose base is
// 1024-byte aligned: chunk bits 4.. XOR offset bits 7.. (span = row bytes).
template <class C>
__host__ __device__ constexpr int tc_swz(int row, int chunk) {
    return row * C::kRbT + 16 * (chunk ^ ((row * C::kRbT >> 7) & (C::kRbT / 16 - 1)));
}

// One 12-byte q3 granule (32 fields, field i at bits 3i..3i+2 of the
// little-endian stream) widened to the 16-byte chunk layout of q4: byte b
// holds fields 2b (bits 0..2) and 2b+1 (bits 3..5), so raw & 7 is the even
// field and raw - (raw & 7) = 8 * the odd field. Per 24-bit segment (bits
// above 24 are ignored): 12-bit halves to 16-bit halves, 6-bit pairs to
// bytes, each a shift and a bit select that leaves stray bits only in bits
// 6..7 of the bytes, then one mask clears those.
__device__ __forceinline__ uint32_t tc_widen_q3_seg(uint32_t s) {
    const uint32_t x = (s & 0x0000FFFFu) | ((s << 4) & 0xFFFF0000u);
    const uint32_t y = (x & 0x00FF00FFu) | ((x << 2) & 0xFF00FF00u);
    return y & 0x3F3F3F3Fu;
}
__device__ __forceinline__ uint4 tc_widen_q3(uint32_t w0, uint32_t w1, uint32_t w2) {
    uint4 r;
    r.x = tc_widen_q3_seg(w0);                         // stream bits 0..23
    r.y = tc_widen_q3_seg(__funnelshift_r(w0, w1, 24));  // 24..47
    r.z = tc_widen_q3_seg(__funnelshift_r(w1, w2, 16));  // 48..71
    r.w = tc_widen_q3_seg(w2 >> 8);                    // 72..95
    return r;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}


// ---- PTX wrappers -----------------------------------------------------------------

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}


__device__ __forceinline__ uint4 ldsm_x2_trans_b8(uint32_t addr) {
    uint4 r;
    asm volatile("ldmatrix.sync.aligned.m16n16.x2.trans.shared.b8 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(addr));
    return r;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr));
    return r;
}

// ---- producer: dynamic unit schedule ------------------------------------------------------
// Units (head, split) are handed out by a global counter, so a CTA that gets
// less bandwidth simply takes fewer units (static shares finished up to 15 %
// apart). The producer tells the consumers which unit and tile each stage
// holds through a per-stage header; a unit's first tile also carries the
// head's query (bulk copy into the stage's query slot). A header with
// unit = -1 ends the consumers' loop. Scheduler words (after the per-head
// tickets): next unit, CTAs finished; the last CTA to finish resets both.

// unit; tile = sequence number of the stage within the unit (0 = first);
// ntiles = 0 for an empty unit, tile + 1 on the unit's last tile, larger
// otherwise; trow = the tile's index in its stream (rows a0 + trow * kTr).
struct TcHeader {
    int unit, tile, ntiles, trow;
};

// Unit (head h, split s) of the tile kernel: the head's rows [r0, r1) are cut
// into T tiles of kTr rows starting at the 8-row block of r0 (a0), and split
// s takes tiles s, s + S, s + 2S, ...: a head's splits sweep its rows side by
// side (the online softmax needs no contiguity), which keeps the copies of
// all CTAs in a narrow window of the cache like one sequential stream.
// Tile i of the stream starts at row a0 + i * kTr; rows outside [r0, r1) are
// masked.
struct TcUnit {
    int h, s, S;
    long long r0, r1, a0;
    int T;       // tiles of the stream
    int ntiles;  // tiles of this split under the static pattern
    int b, hk;   // sequence and KV head (paged cache)
};

// Contiguous streams: rows are the flat rows of [H][L]. Paged cache: rows
// are the sequence's logical positions [0, len); the producer maps each copy
// box through the block table.
template <class C>
__device__ __forceinline__ TcUnit tc_unit_geom(const DecodeParams& p, int u) {
    TcUnit g;
    g.h = u / p.S;
    g.s = u - g.h * p.S;
    g.S = p.S;
    g.b = g.h / p.Hkv;
    g.hk = g.h - g.b * p.Hkv;
    long long len = p.lens ? (long long)min(max(__ldg(p.lens + g.b), 0), p.L) : (long long)p.L;
    if (p.page_rows > 0) {
        g.r0 = 0;
    } else {
        g.r0 = (long long)g.h * p.L;
    }
    g.r1 = g.r0 + len;
    g.a0 = g.r0 & ~7ll;
    g.T = len > 0 ? (int)((g.r1 - g.a0 + C::kTr - 1) / C::kTr) : 0;
    g.ntiles = g.T > g.s ? (g.T - g.s + p.S - 1) / p.S : 0;
    return g;
}

// First row of tile i of the unit's stream.
template <class C>
__device__ __forceinline__ long long tc_tile_row(const TcUnit& g, int i) {
    return g.a0 + (long long)i * C::kTr;
}

#ifdef VA_TC_EARLY_KV
constexpr bool kTcEarlyKv = true;
#else
constexpr bool kTcEarlyKv = false;
#endif

// Rows per tensor copy of a contiguous cache (the paged path copies kBox-row
// boxes, each inside one page; q3 rows move as flat byte ranges).
template <class C>
__host__ __device__ constexpr int tc_box_rows() {
    return C::kKind == Kind::Q3 ? C::kBox : (C::kBoxC < C::kTr ? C::kBoxC : C::kTr);
}

// kPaged: the cache is a page pool (block table); a template parameter so
// that each instantiation carries only one copy path: the producer's code
// per tile is on the critical path of every stage (measured: contiguous rows
// issued through the paged path took 17.3 -> 18.9 us for q4+ at L=16384).
template <class C, bool kPaged>
__device__ void tc_producer(const DecodeParams& p, const CUtensorMap* tmK, const CUtensorMap* tmV, uint8_t* stages,
                            TcHeader* hdr, uint8_t* qring, uint64_t* full, uint64_t* empty, uint8_t* qfirst,
                            uint64_t* qbar, volatile unsigned* shep) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol = l2_policy_evict_first();
    // the first unit's query goes to its own buffer ahead of the tiles, so the
    // consumers prepare it while the tiles are in flight
    const auto first_query = [&]() {
        if (lane == 0) {
            const int h0 = (int)blockIdx.x / p.S;
            mbar_arrive_expect_tx(qbar, (uint32_t)C::kQBytes);
            if constexpr (C::kChan) {
                bulk_g2s(qfirst, p.q + (size_t)h0 * C::kD, C::kD * 2, qbar, pol);
                bulk_g2s(qfirst + C::kD * 2, p.scK + (size_t)h0 * C::kD, C::kD * 2, qbar, pol);
            } else {
                bulk_g2s(qfirst, p.q + (size_t)h0 * C::kG * C::kD, (uint32_t)C::kQBytes, qbar, pol);
            }
        }
        __syncwarp();
    };
    // split-L across GPUs: the step's epoch, read once (after the grid
    // dependency: the previous step's last CTA advanced the counter) and kept
    // in shared memory for the ticket warp; the early-copy variant waits first
    const auto read_epoch = [&]() {
        if (p.xR > 0 && lane == 0)
            *shep = p.xepoch_ptr ? *reinterpret_cast<volatile unsigned*>(p.xepoch_ptr) + 1u : p.xepoch;
    };
    bool waited = !kTcEarlyKv || p.xR > 0;
    if (waited) {
        read_epoch();
        first_query();
    }
    const auto ensure_wait = [&]() {
        if (!waited) {
            grid_dependency_wait();
            VA_TL(12, global_timer_ns());
            first_query();
            waited = true;
        }
    };
    if (lane == 0) VA_TL(11, global_timer_ns());
    const long long nr8 = p.total_rows & ~7ll;
    // q3 rows (48 bytes) are copied as flat byte ranges: a tensor copy issues
    // one request per row, and 48-byte rows straddle 32-byte sectors (about
    // twice the L2 requests of the data, measured)
    constexpr bool kFlatRows = C::kKind == Kind::Q3;
    const int nunits = p.H * p.S;
    unsigned* sched = p.counters + p.H;
    // First unit: blockIdx.x. Later units come from the counter (offset by
    // the grid); a unit's successor is requested when two of its tiles are
    // left to issue, late enough not to reserve work a faster CTA could take,
    // early enough to hide the atomic's round trip.
    int u = blockIdx.x;
    int k = 0;
    bool ok = true;
    // waits for stage k to be free; on expiry reports, drains own copies, stops
    const auto acquire = [&](int kk) -> bool {
        const int stage = kk % C::kStages;
#ifdef VA_TC_FAST_ACQUIRE
        if (mbar_wait_fast(&empty[stage], ((uint32_t)(kk / C::kStages) & 1u) ^ 1u)) return true;
#else
        if (mbar_wait_bounded(&empty[stage], ((uint32_t)(kk / C::kStages) & 1u) ^ 1u)) return true;
#endif
        if (lane == 0) report_error(kErrEmptyWait);
        for (int d = 1; d <= C::kStages && kk - d >= 0; ++d) {
            const int k2 = kk - d;
            mbar_wait_bounded(&full[k2 % C::kStages], (uint32_t)(k2 / C::kStages) & 1u);
        }
        return false;
    };
    // Paged cache: physical first row of box `lane` of tile t, through the block
    // table (a page index outside the pool reads page 0: no wild access).
    const auto paged_row = [&](const TcUnit& g, int t) -> int {
        if (!kPaged || g.T <= 0) return 0;
        const long long pt0 = tc_tile_row<C>(g, t);
        const int pneed = (int)(min(pt0 + C::kTr, (g.r1 + 7) & ~7ll) - pt0);
        if (lane * C::kBox >= pneed) return 0;
        // sequence positions are below 2^31 (checked on the host): 32-bit
        // division, far cheaper than the emulated 64-bit one
        const int yl = (int)(pt0 + (long long)lane * C::kBox);
        const int pg = yl / p.page_rows;
        int pp = pg < p.max_pages ? __ldg(p.block_table + (size_t)g.b * p.max_pages + pg) : 0;
        pp = (pp >= 0 && pp < p.num_pages) ? pp : 0;
        return (pp * p.Hkv + g.hk) * p.page_rows + (yl - pg * p.page_rows);
    };
    // a unit index from the schedule counter, nunits when none is left (also
    // for any counter value, so a workspace that was not zeroed cannot send
    // the producer outside the streams)
    const auto next_unit = [&](unsigned* c, int n) -> int {
        const unsigned v = atomicAdd(c, 1u);
        return v < (unsigned)(n - (int)gridDim.x) ? (int)gridDim.x + (int)v : n;
    };
    while (ok && u < nunits) {
        int unext = nunits;
        bool asked = false;
        const TcUnit g = tc_unit_geom<C>(p, u);
        const long long r1b = (g.r1 + 7) & ~7ll;
        const long long cend = min(r1b, nr8);
        // tile j of the unit: s + j S, -1 past the stream's end
        const auto static_tile = [&](int j) -> int {
            const long long v = (long long)g.s + (long long)j * g.S;
            return v < g.T ? (int)v : -1;
        };
        int cur = static_tile(0);
        int nxt = -1;
        int py_next = cur >= 0 ? paged_row(g, cur) : 0;
        if (cur < 0) {  // empty split: the header alone (slot and ticket still count)
            if (!waited && (k >= C::kStages || !asked)) ensure_wait();
            if (!asked) {
                if (lane == 0) unext = next_unit(sched, nunits);
                asked = true;
            }
            if (!acquire(k)) {
                ok = false;
                break;
            }
            if (lane == 0) {
                hdr[k % C::kStages] = TcHeader{u, 0, 0, 0};
                mbar_arrive(&full[k % C::kStages]);
            }
            __syncwarp();
            ++k;
        }
        for (int t = 0; cur >= 0; ++t, ++k) {
            if (!waited && (k >= C::kStages || (!asked && t >= g.ntiles - 2))) ensure_wait();
            if (!asked && t >= g.ntiles - 2) {
                if (lane == 0) unext = next_unit(sched, nunits);
                asked = true;
            }
            if (!acquire(k)) {
                ok = false;
                break;
            }
            nxt = static_tile(t + 1);
            // paged cache: the next tile's block-table entries are loaded now,
            // one tile ahead of their use
            const int py = py_next;
            py_next = nxt >= 0 ? paged_row(g, nxt) : 0;
            const int stage = k % C::kStages;
            const int hnt = nxt < 0 ? t + 1 : 0x7FFFFFFF;  // header ntiles: marks the unit's last tile
            uint8_t* sK = stages + (size_t)stage * C::kStageBytes;
            uint8_t* sV = sK + C::kTr * C::kRb;
            uint8_t* sSK = sV + C::kTr * C::kRb;
            uint8_t* sSV = sSK + C::kTr * C::kSbK;
            const long long t0 = tc_tile_row<C>(g, cur);
            const long long tend = t0 + C::kTr;
            const int need = (int)(min(tend, r1b) - t0);
            const int nbox = (need + C::kBox - 1) / C::kBox;
            const int brows = (int)max(0ll, min(tend, cend) - t0);
            const long long rg0 = max(t0, nr8), rg1 = min(tend, g.r1);
            // a unit's first tile also carries the stream's query (and, with
            // per-channel K scales, the head's channel scales right after it);
            // the CTA's first unit has its query in its own buffer
            const uint32_t qb = t == 0 && u != (int)blockIdx.x ? (uint32_t)C::kQBytes : 0u;
            const auto copy_query = [&]() {
                if constexpr (C::kChan) {
                    bulk_g2s(qring + stage * C::kQBytes, p.q + (size_t)g.h * C::kD, C::kD * 2, &full[stage], pol);
                    bulk_g2s(qring + stage * C::kQBytes + C::kD * 2, p.scK + (size_t)g.h * C::kD, C::kD * 2,
                             &full[stage], pol);
                } else {  // the stream's kG query heads, contiguous
                    bulk_g2s(qring + stage * C::kQBytes, p.q + (size_t)g.h * C::kG * C::kD, qb, &full[stage], pol);
                }
            };
            if (!kPaged && rg1 > rg0) {
                // scales of the tensor's last partial 8-row block: plain loads
                const int off = (int)(rg0 - t0);
                const int rrows = (int)(rg1 - rg0);
                if constexpr (C::kSbK > 0) {
                    constexpr int kG = C::kSbK / 2;
                    for (int i = lane; i < rrows * kG; i += 32) {
                        const int r = i / kG, w = i % kG;
                        reinterpret_cast<__half*>(sSK)[(off + r) * kG + w] = p.scK[(size_t)(rg0 + r) * kG + w];
                    }
                }
                constexpr int kGv = C::kSbV / 2;
                for (int i = lane; i < rrows * kGv; i += 32) {
                    const int r = i / kGv, w = i % kGv;
                    reinterpret_cast<__half*>(sSV)[(off + r) * kGv + w] = p.scV[(size_t)(rg0 + r) * kGv + w];
                }
                fence_proxy_async_smem();
                __syncwarp();
            }
            if constexpr (kPaged) {
                constexpr int kNb = C::kTr / C::kBox;
                int ys[kNb];  // box b's physical row, from lane b (constant indices: registers)
#pragma unroll
                for (int b = 0; b < kNb; ++b) ys[b] = __shfl_sync(0xffffffffu, py, b);
                if (lane == 0) {
                    hdr[stage] = TcHeader{u, t, hnt, cur};
                    mbar_arrive_expect_tx(&full[stage],
                                          (uint32_t)nbox * C::kBox * (2u * C::kRb + C::kSbK + C::kSbV) + qb);
                    if (qb) copy_query();
                    int seg = 0;       // first box of the current run of physically contiguous boxes
                    int y0 = ys[0];    // and its physical row
#pragma unroll
                    for (int b = 0; b < kNb; ++b) {
                        if (b >= nbox) break;
                        if constexpr (!kFlatRows) {
                            tma_load_2d(sK + b * C::kBox * C::kRb, tmK, 0, ys[b], &full[stage], pol);
                            tma_load_2d(sV + b * C::kBox * C::kRb, tmV, 0, ys[b], &full[stage], pol);
                        }
                        // scales (and flat codes): one bulk copy per run of contiguous boxes
                        if (b + 1 == nbox || b + 1 == kNb || ys[b + 1 < kNb ? b + 1 : b] != ys[b] + C::kBox) {
                            const uint32_t rows = (uint32_t)(b + 1 - seg) * C::kBox;
                            if constexpr (kFlatRows) {
                                bulk_g2s(sK + seg * C::kBox * C::kRb, p.K + (size_t)y0 * C::kRb, rows * C::kRb,
                                         &full[stage], pol);
                                bulk_g2s(sV + seg * C::kBox * C::kRb, p.V + (size_t)y0 * C::kRb, rows * C::kRb,
                                         &full[stage], pol);
                            }
                            if constexpr (C::kSbK > 0)
                                bulk_g2s(sSK + seg * C::kBox * C::kSbK,
                                         reinterpret_cast<const uint8_t*>(p.scK) + (size_t)y0 * C::kSbK,
                                         rows * C::kSbK, &full[stage], pol);
                            bulk_g2s(sSV + seg * C::kBox * C::kSbV,
                                     reinterpret_cast<const uint8_t*>(p.scV) + (size_t)y0 * C::kSbV,
                                     rows * C::kSbV, &full[stage], pol);
                            seg = b + 1;
                            y0 = ys[b + 1 < kNb ? b + 1 : b];
                        }
                    }
                }
            } else if (lane == 0) {
                hdr[stage] = TcHeader{u, t, hnt, cur};
                // flat codes: the tile's rows inside the tensor, one bulk copy
                // per matrix (rows past the end stay stale; they are masked)
                constexpr int kBx = tc_box_rows<C>();
                const int nbx = (need + kBx - 1) / kBx;
                const uint32_t crows =
                    kFlatRows ? (uint32_t)max(0ll, min((long long)nbox * C::kBox, p.total_rows - t0))
                              : (uint32_t)nbx * kBx;
                const uint32_t bytes = crows * 2u * C::kRb + (uint32_t)brows * (C::kSbK + C::kSbV) + qb;
                mbar_arrive_expect_tx(&full[stage], bytes);
                if (qb) copy_query();
                if constexpr (kFlatRows) {
                    if (crows > 0) {
                        bulk_g2s(sK, p.K + (size_t)t0 * C::kRb, crows * C::kRb, &full[stage], pol);
                        bulk_g2s(sV, p.V + (size_t)t0 * C::kRb, crows * C::kRb, &full[stage], pol);
                    }
                } else {
                    for (int b = 0; b < nbx; ++b) {
                        const int y = (int)(t0 + (long long)b * kBx);
                        tma_load_2d(sK + b * kBx * C::kRb, tmK, 0, y, &full[stage], pol);
                        tma_load_2d(sV + b * kBx * C::kRb, tmV, 0, y, &full[stage], pol);
                    }
                }
                if (brows > 0) {
                    if constexpr (C::kSbK > 0)
                        bulk_g2s(sSK, reinterpret_cast<const uint8_t*>(p.scK) + (size_t)t0 * C::kSbK,
                                 (uint32_t)brows * C::kSbK, &full[stage], pol);
                    bulk_g2s(sSV, reinterpret_cast<const uint8_t*>(p.scV) + (size_t)t0 * C::kSbV,
                             (uint32_t)brows * C::kSbV, &full[stage], pol);
                }
            }
            __syncwarp();
            if (nxt < 0) {
                ++k;
                break;
            }
            cur = nxt;
        }
        u = __shfl_sync(0xffffffffu, unext, 0);
    }
    ensure_wait();
    // this CTA's last grab is done: count it; the last CTA resets the schedule
    // (fences: this CTA's grabs are performed before its count, and the reset
    // after every CTA's count)
    unsigned last = 0;
    if (lane == 0) {
        __threadfence();
        last = atomicAdd(&sched[1], 1u) == gridDim.x - 1 ? 1u : 0u;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (last) {
        __threadfence();
        if (lane == 0) {
            sched[0] = 0u;
            sched[1] = 0u;
            if (p.xR > 0 && p.xepoch_ptr) *p.xepoch_ptr = *shep;  // this step's epoch, for the next step
        }
    }
    if (ok && acquire(k)) {
        if (lane == 0) {
            hdr[k % C::kStages] = TcHeader{-1, 0, 0, 0};
            mbar_arrive(&full[k % C::kStages]);
        }
    }
    __syncwarp();
}

// ---- per-stream query state -------------------------------------------------------------

struct TcQ {
    uint32_t b[4][2];  // B fragments of the 4 score mmas (column g of this lane)
    int bias;          // q4: accumulator start of the low-nibble columns (lanes t < 2)
    float qs;          // 2^-e * log2(e)/sqrt(D) (q4: / 16)
};

// Per-warp query preparation from the query copy in shared memory (no CTA
// barrier): the head's exponent e (|q| * 2^e < 2^14, the scaling by 2^e is
// exact), then this lane's B-fragment bytes. q4 column n: n < 4 -> q of the
// even dims (low nibbles), n >= 4 -> odd dims; quant group (n >> 1) & 1;
// plane n & 1 (0: signed high byte, 1: low); only the lanes t' of that group's
// chunks carry nonzero values. The raw-byte mmas use columns 4..7 only (the
// same values as the low-nibble mmas there). q8 mma i covers chunk t' + 4 (i >> 1),
// half i & 1, in columns {0,1}, {4,5}, {2,3}, {6,7} for i = 0..3: a lane's
// column is active in exactly one of them.
__device__ __forceinline__ uint32_t tc_plane_byte(float x, float sc, int plane) {
    const int v = __float2int_rn(x * sc);
    const int hi = (v + 128) >> 8;  // balanced split: v = 256 hi + lo, lo in [-128, 127]
    return (uint32_t)((plane ? v - 256 * hi : hi) & 0xFF);
}

template <class C>
__device__ __forceinline__ void tc_load_q(TcQ& tq, const __half* qs, int g, int t, int lane) {
    constexpr int D = C::kD;
    static_assert(D == 128, "4 dims per lane");
    static_assert(!C::kChan || C::kKind == Kind::Q4, "per-channel K scales: q4 codes");
    const uint2 w4 = reinterpret_cast<const uint2*>(qs)[lane];  // dims 4 lane .. 4 lane + 3
    float2 fa = __half22float2(*reinterpret_cast<const __half2*>(&w4.x));
    float2 fb = __half22float2(*reinterpret_cast<const __half2*>(&w4.y));
    // per-channel K scales (stored after the query) fold into it: q'_d = q_d * s_d,
    // exact in fp32 (a product of two fp16 values)
    const __half* ks = qs + D;
    if constexpr (C::kChan) {
        const uint2 k4 = reinterpret_cast<const uint2*>(ks)[lane];
        const float2 ka = __half22float2(*reinterpret_cast<const __half2*>(&k4.x));
        const float2 kb = __half22float2(*reinterpret_cast<const __half2*>(&k4.y));
        fa.x *= ka.x;
        fa.y *= ka.y;
        fb.x *= kb.x;
        fb.y *= kb.y;
    }
    float amax = fmaxf(fmaxf(fabsf(fa.x), fabsf(fa.y)), fmaxf(fabsf(fb.x), fabsf(fb.y)));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    // amax = m 2^x with m in [0.5, 1): x = biased exponent - 126 (amax is a
    // normal float: fp16 values convert exactly)
    const int e = amax > 0.f ? 14 - (((__float_as_int(amax) >> 23) & 0xFF) - 126) : 0;
    const float sc = __int_as_float((127 + e) << 23);
    const int n = g, plane = g & 1;
    if constexpr (C::kNib) {
        const bool active = ((n >> 1) & 1) == (t >> 1);
        const int odd = n >= 4 ? 1 : 0;
        // dims 32 t .. 32 t + 31 of this lane's chunk: byte b holds dims 2b, 2b+1
        const uint4* src = reinterpret_cast<const uint4*>(qs + 32 * t);
        uint32_t wl[4] = {0u, 0u, 0u, 0u};
        if (active) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {  // 8 dims = 4 bytes per 16-byte load
                const uint4 h = src[c];
                const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
                uint32_t kw[4] = {0u, 0u, 0u, 0u};
                if constexpr (C::kChan) {
                    const uint4 hk = reinterpret_cast<const uint4*>(ks + 32 * t)[c];
                    kw[0] = hk.x;
                    kw[1] = hk.y;
                    kw[2] = hk.z;
                    kw[3] = hk.w;
                }
                uint32_t word = 0;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float2 f = __half22float2(*reinterpret_cast<const __half2*>(&hw[j]));
                    if constexpr (C::kChan) {
                        const float2 fk = __half22float2(*reinterpret_cast<const __half2*>(&kw[j]));
                        f.x *= fk.x;
                        f.y *= fk.y;
                    }
                    word |= tc_plane_byte(odd ? f.y : f.x, sc, plane) << (8 * j);
                }
                wl[c] = word;  // bytes 4c .. 4c+3 of the chunk
            }
        }
        // mma i (i & 1 = half), register r: bytes 8 (i & 1) + 4 r .. + 3
        tq.b[0][0] = wl[0];
        tq.b[0][1] = wl[1];
        tq.b[1][0] = wl[2];
        tq.b[1][1] = wl[3];
        tq.b[2][0] = odd ? wl[0] : 0u;
        tq.b[2][1] = odd ? wl[1] : 0u;
        tq.b[3][0] = odd ? wl[2] : 0u;
        tq.b[3][1] = odd ? wl[3] : 0u;
        // lane t < 2 starts the low-nibble columns of group t at -8 * sum(q over the group)
        int sq = __float2int_rn(fa.x * sc) + __float2int_rn(fa.y * sc) + __float2int_rn(fb.x * sc) +
                 __float2int_rn(fb.y * sc);
#pragma unroll
        for (int off = 1; off < 16; off <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);  // lanes of a group
        const int s0 = __shfl_sync(0xffffffffu, sq, 0), s1 = __shfl_sync(0xffffffffu, sq, 16);
        constexpr int kZero = C::kKind == Kind::Q3 ? 4 : 8;  // code of value 0
        tq.bias = t == 0 ? -kZero * s0 : t == 1 ? -kZero * s1 : 0;
    } else {
        const int ia = 2 * ((n >> 1) & 1) + (n >> 2);  // the mma whose column pair holds n
        const int chunk = t + 4 * (ia >> 1);
        const uint4 h = reinterpret_cast<const uint4*>(qs + 16 * chunk + 8 * (ia & 1))[0];
        const uint32_t hw[4] = {h.x, h.y, h.z, h.w};
        uint32_t wr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&hw[2 * r]));
            const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&hw[2 * r + 1]));
            wr[r] = tc_plane_byte(f0.x, sc, plane) | (tc_plane_byte(f0.y, sc, plane) << 8) |
                    (tc_plane_byte(f1.x, sc, plane) << 16) | (tc_plane_byte(f1.y, sc, plane) << 24);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            tq.b[i][0] = i == ia ? wr[0] : 0u;
            tq.b[i][1] = i == ia ? wr[1] : 0u;
        }
        tq.bias = 0;
    }
    const float base = rsqrtf((float)D) * kLog2e;
    // the two-field path scores 16 (q4) or 8 (q3) times the dot product
    tq.qs = base / sc * (C::kKind == Kind::Q4 ? 0.0625f : C::kKind == Kind::Q3 ? 0.125f : 1.f);
}

// ---- one tile of one warp ------------------------------------------------------------------

template <class C>
struct TcState {
    float m, l;
    float o[C::kPairs][C::kNib ? 4 : 2];
};

template <class C, bool kMasked>
__device__ __forceinline__ void tc_tile(uint32_t sK, uint32_t sV, const __half* sSK, const __half* sSV, uint8_t* sp,
                                        int wrow, int g, int t, long long t0, long long r0, long long r1,
                                        const TcQ& tq, const uint32_t* voff, uint32_t vbuf, TcState<C>& st) {
    constexpr bool kQ4 = C::kNib;  // q4 and (widened) q3: two fields per byte
    constexpr bool kQ3 = C::kKind == Kind::Q3;
    constexpr int kRb = C::kRb;
    // low field mask and the factor between the high field and raw - low
    constexpr uint32_t m4 = kQ3 ? 0x07070707u : 0x0F0F0F0Fu;
    constexpr int kHiMul = kQ3 ? 8 : 16;
    constexpr int kZero = kQ3 ? 4 : 8;  // code of value 0
    const int rowA = tc_row_a<C>(g), rowB = tc_row_b<C>(g);
    const uint32_t offA = (uint32_t)tc_swz<C>(rowA, t), offB = (uint32_t)tc_swz<C>(rowB, t);
    if constexpr (kQ3) {
        // widen this warp's 64 V rows into its buffer in the q4 chunk layout
        // (lane: granule lane % 4 of rows lane / 4 + 8 i), read back below by
        // ldmatrix; the previous tile's reads of the buffer are done (the
        // __syncwarp that ends tc_tile). All loads first: the shared-memory
        // accesses are volatile, so they issue in program order.
        const int r0_ = (threadIdx.x & 31) / 4, c = threadIdx.x & 3;
        uint32_t raw[8][3];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int k = 0; k < 3; ++k) raw[i][k] = lds32(sV + (uint32_t)((wrow + r0_ + 8 * i) * kRb + 12 * c + 4 * k));
#pragma unroll
        for (int i = 0; i < 8; ++i)
            sts128(vbuf + (uint32_t)tc_swz<C>(r0_ + 8 * i, c), tc_widen_q3(raw[i][0], raw[i][1], raw[i][2]));
    }
    // q3: granule t of rows A and B of every block, loaded ahead of the mmas
    uint32_t kraw[kQ3 ? 4 : 1][2][3];
    if constexpr (kQ3) {
#pragma unroll
        for (int blk = 0; blk < 4; ++blk)
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                const uint32_t rb = sK + (uint32_t)((wrow + 16 * blk) * kRb + 12 * t + 4 * k);
                kraw[blk][0][k] = lds32(rb + (uint32_t)(rowA * kRb));
                kraw[blk][1][k] = lds32(rb + (uint32_t)(rowB * kRb));
            }
    }

    // ---- scores: lane partials per block, rows A and B ------------------------------------
    int v[4][2];
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const uint32_t rb = sK + (uint32_t)((wrow + 16 * blk) * kRb);
        if constexpr (kQ4) {
            uint4 wa, wb;
            if constexpr (kQ3) {  // granule t of rows A and B, widened in registers
                wa = tc_widen_q3(kraw[blk][0][0], kraw[blk][0][1], kraw[blk][0][2]);
                wb = tc_widen_q3(kraw[blk][1][0], kraw[blk][1][1], kraw[blk][1][2]);
            } else {
                wa = lds128(rb + offA);
                wb = lds128(rb + offB);
            }
            int a1[4] = {0, tq.bias, 0, tq.bias}, a2[4] = {0, 0, 0, 0};
            mma_k32<false, true>(a1, wa.x & m4, wb.x & m4, wa.y & m4, wb.y & m4, tq.b[0][0], tq.b[0][1]);
            mma_k32<false, true>(a1, wa.z & m4, wb.z & m4, wa.w & m4, wb.w & m4, tq.b[1][0], tq.b[1][1]);
            mma_k32<false, true>(a2, wa.x, wb.x, wa.y, wb.y, tq.b[2][0], tq.b[2][1]);
            mma_k32<false, true>(a2, wa.z, wb.z, wa.w, wb.w, tq.b[3][0], tq.b[3][1]);
            // lanes t < 2: 16 (8) * (low fields . even q); t >= 2: raw . odd q - low . odd q
            const int alpha = t < 2 ? kHiMul : -1;
            v[blk][0] = alpha * (256 * a1[0] + a1[1]) + (256 * a2[0] + a2[1]);
            v[blk][1] = alpha * (256 * a1[2] + a1[3]) + (256 * a2[2] + a2[3]);
        } else {
            const uint32_t offA2 = (uint32_t)tc_swz<C>(rowA, t + 4), offB2 = (uint32_t)tc_swz<C>(rowB, t + 4);
            const uint4 wa = lds128(rb + offA), wb = lds128(rb + offB);
            const uint4 wc = lds128(rb + offA2), wd = lds128(rb + offB2);
            int a[4] = {0, 0, 0, 0};
            mma_k32<true, true>(a, wa.x, wb.x, wa.y, wb.y, tq.b[0][0], tq.b[0][1]);
            mma_k32<true, true>(a, wa.z, wb.z, wa.w, wb.w, tq.b[1][0], tq.b[1][1]);
            mma_k32<true, true>(a, wc.x, wd.x, wc.y, wd.y, tq.b[2][0], tq.b[2][1]);
            mma_k32<true, true>(a, wc.z, wd.z, wc.w, wd.w, tq.b[3][0], tq.b[3][1]);
            v[blk][0] = 256 * a[0] + a[1];
            v[blk][1] = 256 * a[2] + a[3];
        }
    }
    // reduce-scatter over the quad: lanes t, t^2 share a quant group (exact
    // integer adds), then t, t^1 join the two groups after their scales
    const bool hi = (t >> 1) != 0, odd = (t & 1) != 0;
    int u[2][2];
#pragma unroll
    for (int b = 0; b < 2; ++b)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int keep = hi ? v[2 + b][r] : v[b][r];
            const int send = hi ? v[b][r] : v[2 + b][r];
            u[b][r] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
        }
    const int grp = t & 1;
    float f[2][2];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
        const int rbase = wrow + 16 * (2 * (t >> 1) + b);
        if constexpr (C::kChan) {  // the K scales are in the query already
            f[b][0] = (float)u[b][0];
            f[b][1] = (float)u[b][1];
        } else {
            f[b][0] = (float)u[b][0] * __half2float(sSK[(rbase + rowA) * C::kNgrp + grp]);
            f[b][1] = (float)u[b][1] * __half2float(sSK[(rbase + rowB) * C::kNgrp + grp]);
        }
    }
    const int myrow0 = wrow + 16 * t + rowA, myrow1 = wrow + 16 * t + rowB;  // block t
    float s[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const float keep = odd ? f[1][r] : f[0][r];
        const float send = odd ? f[0][r] : f[1][r];
        s[r] = (keep + __shfl_xor_sync(0xffffffffu, send, 1)) * tq.qs;
    }
    bool valid[2] = {true, true};
    if constexpr (kMasked) {
        valid[0] = (t0 + myrow0 >= r0) && (t0 + myrow0 < r1);
        valid[1] = (t0 + myrow1 >= r0) && (t0 + myrow1 < r1);
        s[0] = valid[0] ? s[0] : -INFINITY;
        s[1] = valid[1] ? s[1] : -INFINITY;
    }

    // ---- online softmax over the warp's 64 rows -----------------------------------------------
    // warp max with one redux: float bits mapped to order-preserving ints
    float bm;
    {
        const int b = __float_as_int(fmaxf(s[0], s[1]));
        const int key = __reduce_max_sync(0xffffffffu, b < 0 ? b ^ 0x7FFFFFFF : b);
        bm = __int_as_float(key < 0 ? key ^ 0x7FFFFFFF : key);
    }
    const float mnew = fmaxf(st.m, bm);
    const float c = fast_exp2(st.m - mnew);
    st.m = mnew;
    const float e0 = fast_exp2(s[0] - mnew), e1 = fast_exp2(s[1] - mnew);
    st.l = st.l * c + e0 + e1;
    float2 vs0, vs1;
    if constexpr (C::kChan) {  // one V scale per row, for both quant groups
        const float a = __half2float(sSV[myrow0]), b = __half2float(sSV[myrow1]);
        vs0 = make_float2(a, a);
        vs1 = make_float2(b, b);
    } else {
        vs0 = __half22float2(*reinterpret_cast<const __half2*>(sSV + myrow0 * C::kNgrp));
        vs1 = __half22float2(*reinterpret_cast<const __half2*>(sSV + myrow1 * C::kNgrp));
    }
    float w[2][2] = {{e0 * vs0.x, e0 * vs0.y}, {e1 * vs1.x, e1 * vs1.y}};  // [row][group]
    if constexpr (kMasked) {
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            w[0][gi] = valid[0] ? w[0][gi] : 0.f;
            w[1][gi] = valid[1] ? w[1][gi] : 0.f;
        }
    }
    float wscale[2];
    int psum[2];
    uint32_t pk[2];
#pragma unroll
    for (int gi = 0; gi < 2; ++gi) {
        // weights are >= 0: their bit patterns order like the values
        const float wm = __uint_as_float(
            __reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(w[0][gi], w[1][gi]))));
        const float inv = wm > 0.f ? 32767.f / wm : 0.f;
        wscale[gi] = wm * (1.f / 32767.f);
        // p rides in the low bits of 1.5 * 2^23: byte 0 = low plane, byte 1 = high
        const uint32_t pa = __float_as_uint(fmaf(w[0][gi], inv, 12582912.0f));
        const uint32_t pb = __float_as_uint(fmaf(w[1][gi], inv, 12582912.0f));
        psum[gi] = (int)__reduce_add_sync(0xffffffffu, (pa - 0x4B400000u) + (pb - 0x4B400000u));
        pk[gi] = __byte_perm(pa, pb, 0x5140);  // [lo A, lo B, hi A, hi B]
    }
    // stage the weight planes as B fragments: block t, source quad g -> k = 4 t' + 2 sec + (0: A, 1: B)
    {
        const int tq_ = ((g & 1) << 1) | (g >> 2), sec = (g >> 1) & 1;
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            uint8_t* b = sp + ((t * 2 + gi) * 5) * 32 + tq_ * 8 + 2 * sec;
            const uint16_t hp = (uint16_t)(pk[gi] >> 16), lp = (uint16_t)(pk[gi] & 0xFFFFu);
            *reinterpret_cast<uint16_t*>(b + 0 * 32) = hp;      // column 0: high plane, first chunk
            *reinterpret_cast<uint16_t*>(b + 1 * 32) = lp;      // column 1: low plane
            *reinterpret_cast<uint16_t*>(b + 2 * 32 + 4) = hp;  // column 2: high plane, second chunk
            *reinterpret_cast<uint16_t*>(b + 3 * 32 + 4) = lp;  // column 3
        }
    }
    __syncwarp();

    // ---- output: O^T += V^T . P per chunk pair ---------------------------------------------------
    if (__any_sync(0xffffffffu, c != 1.f)) {
#pragma unroll
        for (int pi = 0; pi < C::kPairs; ++pi)
#pragma unroll
            for (int x = 0; x < (kQ4 ? 4 : 2); ++x) st.o[pi][x] *= c;
    }
    const int slot = min(g, 4);
    // V tile: the stage (q4, q8) or the warp's widened rows (q3)
    const uint32_t vrows = kQ3 ? vbuf : sV + (uint32_t)(wrow * C::kRbT);
    if constexpr (kQ3) __syncwarp();  // the widened rows are visible to the warp
    if constexpr (kQ4) {
        // two accumulator sets (blocks 0,1 and 2,3): shorter mma dependency chains
        int aR[2][2][4], aL[2][2][4];
#pragma unroll
        for (int pi = 0; pi < 2; ++pi)
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                aL[c][pi][0] = aL[c][pi][2] = 0;
                aL[c][pi][1] = aL[c][pi][3] = c == 0 ? -kZero * psum[pi] : 0;
                aR[c][pi][0] = aR[c][pi][2] = 0;
                aR[c][pi][1] = aR[c][pi][3] = c == 0 ? -(kZero + kHiMul * kZero) * psum[pi] : 0;
            }
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
#pragma unroll
            for (int pi = 0; pi < 2; ++pi) {
                const uint2 bf = *reinterpret_cast<const uint2*>(sp + ((blk * 2 + pi) * 5 + slot) * 32 + t * 8);
                const uint4 a = ldsm_x2_trans_b8(vrows + (uint32_t)(16 * blk * C::kRbT) + voff[pi]);
                mma_k32<false, false>(aR[blk >> 1][pi], a.x, a.y, a.z, a.w, bf.x, bf.y);
                mma_k32<false, false>(aL[blk >> 1][pi], a.x & m4, a.y & m4, a.z & m4, a.w & m4, bf.x, bf.y);
            }
        }
#pragma unroll
        for (int pi = 0; pi < 2; ++pi) {
            const auto sum = [&](int (&a)[2][2][4], int x) { return a[0][pi][x] + a[1][pi][x]; };
            const int xl0 = 256 * sum(aL, 0) + sum(aL, 1), xl1 = 256 * sum(aL, 2) + sum(aL, 3);
            const int xr0 = 256 * sum(aR, 0) + sum(aR, 1), xr1 = 256 * sum(aR, 2) + sum(aR, 3);
            const float ws = wscale[pi], ws16 = wscale[pi] * (1.f / kHiMul);
            st.o[pi][0] = fmaf((float)xl0, ws, st.o[pi][0]);
            st.o[pi][1] = fmaf((float)(xr0 - xl0), ws16, st.o[pi][1]);
            st.o[pi][2] = fmaf((float)xl1, ws, st.o[pi][2]);
            st.o[pi][3] = fmaf((float)(xr1 - xl1), ws16, st.o[pi][3]);
        }
    } else {
        int acc[C::kPairs][4];
#pragma unroll
        for (int pi = 0; pi < C::kPairs; ++pi)
#pragma unroll
            for (int x = 0; x < 4; ++x) acc[pi][x] = 0;
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) {
            uint2 bf[2];
#pragma unroll
            for (int gi = 0; gi < 2; ++gi)
                bf[gi] = *reinterpret_cast<const uint2*>(sp + ((blk * 2 + gi) * 5 + slot) * 32 + t * 8);
#pragma unroll
            for (int pi = 0; pi < C::kPairs; ++pi) {
                const uint4 a = ldsm_x2_trans_b8(vrows + (uint32_t)(16 * blk * C::kRbT) + voff[pi]);
                const uint2 b = bf[pi / (C::kPairs / 2)];
                mma_k32<true, false>(acc[pi], a.x, a.y, a.z, a.w, b.x, b.y);
            }
        }
#pragma unroll
        for (int pi = 0; pi < C::kPairs; ++pi) {
            const float ws = wscale[pi / (C::kPairs / 2)];
            st.o[pi][0] = fmaf((float)(256 * acc[pi][0] + acc[pi][1]), ws, st.o[pi][0]);
            st.o[pi][1] = fmaf((float)(256 * acc[pi][2] + acc[pi][3]), ws, st.o[pi][1]);
        }
    }
    __syncwarp();
}

// Output dim of o[pi][x] held by lane (g, t < 2).
template <class C>
__device__ __forceinline__ int tc_out_dim(int pi, int x, int g, int t) {
    const int chunk = 2 * pi + t;
    if constexpr (C::kNib) return 2 * (16 * chunk + g + 8 * (x >> 1)) + (x & 1);
    else return 16 * chunk + g + 8 * x;
}

// Single-pass log-sum-exp merge of a head's S slots (the reference's
// combine, src/voltattn.cu:651-672) for dims lane + 32 j, j < kJ, by one
// lane: the loads of a batch of kB slots are independent, so each batch
// costs one L2 round trip (one in all for S <= kB).
template <int kJ, int kB = 16>
__device__ __forceinline__ void tc_merge_slots(const float* hs, int S, int D, int lane, float& ms, float& ls,
                                               float* od) {
    ms = kNegMax;
    ls = 0.f;
#pragma unroll
    for (int j = 0; j < kJ; ++j) od[j] = 0.f;
    for (int i0 = 0; i0 < S; i0 += kB) {
        float m[kB], l[kB], o[kB][kJ];
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const bool in = i0 + i < S;
            const float* sp = hs + (size_t)(in ? i0 + i : 0) * (D + 2);
            m[i] = in ? __ldcg(sp) * kLog2e : kNegMax;  // slots hold natural-log m
            l[i] = in ? __ldcg(sp + 1) : 0.f;
#pragma unroll
            for (int j = 0; j < kJ; ++j) o[i][j] = in ? __ldcg(sp + 2 + lane + 32 * j) : 0.f;
        }
        float bm = ms;
#pragma unroll
        for (int i = 0; i < kB; ++i) bm = fmaxf(bm, m[i]);
        const float c = fast_exp2(ms - bm);
        ls *= c;
#pragma unroll
        for (int j = 0; j < kJ; ++j) od[j] *= c;
#pragma unroll
        for (int i = 0; i < kB; ++i) {
            const float a = fast_exp2(m[i] - bm);  // 0 for the padding (m = -FLT_MAX)
            ls = fmaf(l[i], a, ls);
#pragma unroll
            for (int j = 0; j < kJ; ++j) od[j] = fmaf(o[i][j], a, od[j]);
        }
        ms = bm;
    }
    ms *= kLn2;
}

// Ticket warp: takes the head ticket of each unit the consumers finished
// (handed over through a ring of kTRing entries, mbarriers `tdone` /
// `tfree`), so the ticket's release (which waits for the slot writes) and
// the round trip of the atomic stay off the consumers' path. The CTA that
// takes a head's last ticket merges its S slots here (4 dims per lane) and
// writes the output, then resets the ticket counter for the next call.
// Memory order: the consumers' slot writes precede their tdone arrivals
// (release, CTA scope); the wait on tdone acquires them; the gpu-scope
// acquire-release ticket is cumulative over them.
template <class C>
__device__ void tc_ticket_warp(const DecodeParams& p, const int* th, uint64_t* tdone, uint64_t* tfree,
                               volatile int* shok, const volatile unsigned* shep) {
    constexpr int D = C::kD;
    const int lane = threadIdx.x & 31;
    for (int n = 0;; ++n) {
        const int e = n % C::kTRing;
        if (!mbar_wait_bounded(&tdone[e], (uint32_t)(n / C::kTRing) & 1u)) {
            if (lane == 0) report_error(kErrFullWait);
            return;
        }
        const int h = th[e];
        if (h < 0) {
            if (lane == 0) VA_TL(4, global_timer_ns());  // timeline: 4 ticket warp done
            return;
        }
        unsigned ticket = 0;
        if (lane == 0) ticket = atomic_add_acq_rel_gpu(&p.counters[h], 1u);
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket == (unsigned)(p.S - 1)) {
            for (int kq = 0; kq < C::kG; ++kq) {  // the stream's query heads
                const size_t hq = (size_t)h * C::kG + kq;
                float ms, ls, od[D / 32];
                tc_merge_slots<D / 32>(p.ws + hq * p.S * (D + 2), p.S, D, lane, ms, ls, od);
                if (p.xR > 0) {  // split-L across GPUs: exchange, merge the ranks' partials, write out
                    if (lane == 0) VA_TL(14, global_timer_ns());  // timeline: 14 exchange entered
                    const bool xok =
                        peer_exchange_head<D / 32>(p.x, p.xR, p.xrank, *shep, p.xwait_ns, p.H * C::kG, D, (int)hq, ms,
                                                   ls, od, lane, 32, lane, [] { __syncwarp(); }, shok);
                    if (lane == 0) VA_TL(15, global_timer_ns());  // timeline: 15 exchange merged
                    if (xok) {
#pragma unroll
                        for (int j = 0; j < D / 32; ++j) p.out[hq * D + lane + 32 * j] = __float2half_rn(od[j]);
                    }
                    continue;
                }
#pragma unroll
                for (int j = 0; j < D / 32; ++j) {
                    const int d = lane + 32 * j;
                    if (p.out_mode == kOutHalf) {
                        p.out[hq * D + d] = __float2half_rn(od[j] / ls);
                    } else {
                        float* pp = p.partial + hq * (D + 2);
                        pp[2 + d] = od[j];
                        if (d == 0) {
                            pp[0] = ms;
                            pp[1] = ls;
                        }
                    }
                }
            }
            if (lane == 0) store_relaxed_gpu(&p.counters[h], 0u);
            if (lane == 0) VA_TL(5, global_timer_ns());  // timeline: 5 last head merge written
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfree[e]);
    }
}

template <class C, bool kPaged>
__global__ void __launch_bounds__(C::kThreads, 2)
    decode_tc_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    constexpr int D = C::kD;
    uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* vbufs = stages + C::kStages * C::kStageBytes;  // q3: per-warp widened V rows
    uint64_t* full = reinterpret_cast<uint64_t*>(vbufs + C::kVBuf);
    uint64_t* empty = full + C::kStages;
    TcHeader* hdr = reinterpret_cast<TcHeader*>(empty + C::kStages);
    uint8_t* qring = reinterpret_cast<uint8_t*>(hdr + C::kStages);
    float* shMerge = reinterpret_cast<float*>(qring + C::kStages * C::kQBytes);  // [warps][D] o, then m, l
    float* shM = shMerge + C::kWarps * D;
    float* shL = shM + C::kWarps;
    uint8_t* shP = reinterpret_cast<uint8_t*>(shMerge + C::kMergeFloats);
    uint64_t* tdone = reinterpret_cast<uint64_t*>(shP + C::kWarps * C::kPStage);
    uint64_t* tfree = tdone + C::kTRing;
    int* th = reinterpret_cast<int*>(tfree + C::kTRing);
    volatile int* shFail = th + C::kTRing;
    uint64_t* qbar = reinterpret_cast<uint64_t*>(th + C::kTRing + 4);  // first unit's query: own barrier
    uint8_t* qfirst = reinterpret_cast<uint8_t*>(qbar + 2);  // 16-byte aligned copy target

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // zero the weight staging once: only its nonzero halves are rewritten
    for (int i = threadIdx.x; i < C::kWarps * C::kPStage / 4; i += C::kThreads)
        reinterpret_cast<uint32_t*>(shP)[i] = 0u;
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
    // Programmatic dependent launch: every warp but the producer waits here for
    // the preceding grid (its ws, counters and out, and the query, which a
    // preceding kernel may have written). With kTcEarlyKv the producer streams
    // the first stages of K/V first, which no decode writes, and waits before
    // it reads the query or touches the schedule counters.
#ifdef VA_TC_TIMELINE
    // timeline: 13 the first stage landed (seen by the idle ticket warp, before its grid wait)
    if (kTcEarlyKv && warp == C::kWarps + 1 && lane == 0 && mbar_wait_bounded(&full[0], 0))
        VA_TL(13, global_timer_ns());
#endif
    if (warp != C::kWarps || !kTcEarlyKv) grid_dependency_wait();
    if (threadIdx.x == 0) grid_launch_dependents();
    if (threadIdx.x == 0) {  // timeline: 0 start, 1 SM
        VA_TL(0, global_timer_ns());
        unsigned smid;
        asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
        VA_TL(1, smid);
    }

    const int nunits = p.H * p.S;
    const int h0 = (int)blockIdx.x / p.S;  // head of the CTA's first unit (blockIdx.x < nunits)
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
    uint8_t* sp = shP + warp * C::kPStage;
    const int wrow = warp * C::kRpw;
    const uint32_t vbuf = smem_u32(vbufs) + (uint32_t)(warp * C::kRpw * C::kRbT);
    // ldmatrix row addresses of this lane (k = lane & 15 of chunk 2 pi + lane / 16)
    uint32_t voff[C::kPairs];
    {
        const int r = lane & 15, mat = lane >> 4;
        const int tp = r >> 2, j = r & 3;
        const int q = tc_q1(tp) + 2 * (j >> 1);
        const int row = (j & 1) ? tc_row_b<C>(q) : tc_row_a<C>(q);
#pragma unroll
        for (int pi = 0; pi < C::kPairs; ++pi) voff[pi] = (uint32_t)tc_swz<C>(row, 2 * pi + mat);
    }
    TcQ tq;
    TcState<C> st;
    TcUnit gm;
    int cur_h = -1;
    if (mbar_wait_bounded(qbar, 0)) {
        tc_load_q<C>(tq, reinterpret_cast<const __half*>(qfirst), g, t, lane);
        cur_h = h0;
    } else if (lane == 0) {
        report_error(kErrFullWait);
    }
    const bool tickets = p.out_mode != kOutSlots;
    int nu = 0;  // units finished by this CTA (ticket ring sequence)
    // hands entry nu to the ticket warp: h >= 0 a finished unit's head
    // (after this warp's slot writes), h = -1 the end
    const auto hand_over = [&](int h) {
        const int e = nu % C::kTRing;
        if (lane == 0) {
            if (tid == 0) th[e] = h;
            __threadfence_block();
        }
        named_barrier_sync(1, kConsumerThreads);  // th written, all slot writes issued
        __syncwarp();
        if (lane == 0) mbar_arrive(&tdone[e]);
        ++nu;
    };
    // waits until the ticket warp released ring entry nu (from 4 units ago)
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
        if (tid == 0 && k == 0) VA_TL(2, global_timer_ns());  // timeline: 2 first stage landed
        if (tid == 0 && k >= 1 && k < 4) VA_TL(7 + k, global_timer_ns());  // 8..10: stages 1..3 landed
        if (h.unit < 0) {
            if (tid == 0) {  // timeline: 3 last tile consumed, 6 stages consumed
                VA_TL(3, global_timer_ns());
                VA_TL(6, k);
            }
            break;
        }
        uint8_t* base = stages + (size_t)stage * C::kStageBytes;
        if (h.tile == 0) {
            gm = tc_unit_geom<C>(p, h.unit);
            if (gm.h != cur_h && h.ntiles > 0) {
                tc_load_q<C>(tq, reinterpret_cast<const __half*>(qring + stage * C::kQBytes), g, t, lane);
                cur_h = gm.h;
            }
            st.m = kNegMax;
            st.l = 0.f;
#pragma unroll
            for (int pi = 0; pi < C::kPairs; ++pi)
#pragma unroll
                for (int x = 0; x < (C::kNib ? 4 : 2); ++x) st.o[pi][x] = 0.f;
        }
        if (h.ntiles > 0) {
            const long long t0 = tc_tile_row<C>(gm, h.trow);
            const uint32_t sK = smem_u32(base), sV = sK + C::kTr * C::kRb;
            const __half* sSK = reinterpret_cast<const __half*>(base + 2 * C::kTr * C::kRb);
            const __half* sSV = reinterpret_cast<const __half*>(base + 2 * C::kTr * C::kRb + C::kTr * C::kSbK);
            const long long w0 = t0 + wrow;
            const bool interior = w0 >= gm.r0 && w0 + C::kRpw <= gm.r1;
            if (interior)
                tc_tile<C, false>(sK, sV, sSK, sSV, sp, wrow, g, t, t0, gm.r0, gm.r1, tq, voff, vbuf, st);
            else
                tc_tile<C, true>(sK, sV, sSK, sSV, sp, wrow, g, t, t0, gm.r0, gm.r1, tq, voff, vbuf, st);
        }
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (h.tile < h.ntiles - 1) continue;

        // ---- unit epilogue: warp partials -> CTA slot -> ticket warp ----------------------
        float l = st.l;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (t < 2) {
#pragma unroll
            for (int pi = 0; pi < C::kPairs; ++pi)
#pragma unroll
                for (int x = 0; x < (C::kNib ? 4 : 2); ++x)
                    shMerge[warp * D + tc_out_dim<C>(pi, x, g, t)] = st.o[pi][x];
        }
        if (lane == 0) {
            shM[warp] = st.m;
            shL[warp] = l;
        }
        named_barrier_sync(1, kConsumerThreads);
        {
            float ms = kNegMax;
#pragma unroll
            for (int w = 0; w < C::kWarps; ++w) ms = fmaxf(ms, shM[w]);
            float* slot = p.ws + ((size_t)gm.h * p.S + gm.s) * (D + 2);
            for (int d = tid; d < D; d += kConsumerThreads) {
                float ls = 0.f, od = 0.f;
#pragma unroll
                for (int w = 0; w < C::kWarps; ++w) {
                    const float a = fast_exp2(shM[w] - ms);
                    ls += shL[w] * a;
                    od += shMerge[w * D + d] * a;
                }
                slot[2 + d] = od;
                if (d == 0) {
                    slot[0] = ms * kLn2;  // natural-log units, as the reference's slots
                    slot[1] = ls;
                }
            }
        }
        if (tickets) {
            if (!ring_slot_free()) {
                if (lane == 0) {
                    report_error(kErrFullWait);
                    *shFail = 1;
                }
            }
            hand_over(gm.h);  // also the barrier that frees the merge area
        } else {
            named_barrier_sync(1, kConsumerThreads);
        }
    }
    if (tickets && ring_slot_free()) hand_over(-1);
    if (tid == 0) VA_TL(7, global_timer_ns());  // timeline: 7 consumers done
}

}  // namespace va
