// Prefill (multi-token) attention over the quantized KV cache on the
// Blackwell tensor cores: tcgen05.mma with shared-memory operands and
// accumulators in tensor memory (TMEM).
//
// The reference decodes one token at a time and has no prefill (its README
// lists batch-1 single-token decode as a limitation); the math per query row
// is the reference's (src/voltattn.cu:769-794): score_j = q.K_j / sqrt(D),
// softmax over the visible rows, o = sum_j p_j V_j, with K_j, V_j the
// dequantized cache rows (src/voltattn.cu:747-767: code * fp16 scale).
//
// Problem: Lq new tokens of one sequence whose K/V rows are already in the
// cache as its last Lq rows, Hq query heads over Hkv KV heads (head h reads
// KV head h / (Hq / Hkv)). Token i (0-based) sees cache rows
// [0, L - Lq + i] (causal). q, out: fp16 [Hq][Lq][D]; cache [Hkv][L] rows.
//
// One CTA per (query head, block of 128 tokens), 8 warps, 2 CTAs per SM (the
// two CTAs' phases interleave). Per block of 128 cache rows:
//   1. all warps dequantize the block's K and V rows to fp16 into shared
//      memory (all loads of a thread first, then code * scale, one rounding):
//      K while the previous block's PV runs, V while this block's S runs;
//   2. one thread issues S = Q K^T as 8 tcgen05.mma (M = 128 tokens,
//      N = 128 rows, K = 16 dims each) into TMEM columns [0, 128);
//   3. all 8 warps run the softmax: thread (warpgroup hf, TMEM lane r) takes
//      columns [64 hf, 64 hf + 64) of token row r. It reads S twice (row
//      maximum, exchanged with the other half through shared memory, then
//      the weights), masks only blocks on the diagonal, writes its half of P
//      (fp16 pairs) into S columns it has read, and rescales its half of the
//      running O in TMEM when the row maximum moved;
//   4. one thread issues O += P V as 8 tcgen05.mma with A = P read from TMEM
//      (N = 128 dims, K = 16 rows each) into TMEM columns [128, 256).
// The tiles use the canonical 128-byte-swizzled layout: two 64-element
// panels of 128 rows, row r of a panel at r * 128 bytes, 16-byte chunk c at
// (c ^ (r & 7)) * 16. The K tile is read K-major (rows = N), the V tile,
// with the same bytes layout, MN-major (dims contiguous), so V needs no
// transpose. Every wait on an mbarrier is bounded.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include <type_traits>

#include "common.cuh"
#include "formats.cuh"

namespace va {

struct PrefillParams {
    const uint8_t* K;
    const uint8_t* V;
    const __half* scK;
    const __half* scV;
    const __half* q;
    __half* out;
    int Hq, Hkv, L, Lq;
    // paged cache (page_rows > 0): row j of KV head k lives in page
    // block_table[j / page_rows] at physical row (page * Hkv + k) * page_rows +
    // j % page_rows of [num_pages][Hkv][page_rows]; entries outside the pool
    // read page 0
    const int* block_table;
    int page_rows, num_pages;
};

// kChanScales: the q4c+ layout, K codes with per-channel scales per KV head
// ([Hkv][D]) and V codes with one scale per row ([Hkv][L]).
template <Kind K, bool kChanScales = false>
struct PrefillCfg {
    static constexpr Kind kKind = K;
    static constexpr bool kChan = kChanScales;
    static constexpr int kD = 128;
    static constexpr int kBq = 128;  // tokens per CTA (MMA M)
    static constexpr int kBk = 128;  // cache rows per block (MMA N of S, K of O)
    static constexpr int kThreads = 256;
    static constexpr int kRb = kD * KindTraits<K>::kBits / 8;  // code bytes per cache row
    static constexpr int kTile = kBq * kD * 2;                 // one fp16 128 x 128 tile
    // Q, K, V + barriers and the row-max exchange: 100 KB, 2 CTAs per SM
    static constexpr int kSmemBytes = 1024 + 3 * kTile + 64 + 2 * kBq * 4;  // + row-max exchange
    static constexpr int kTmemCols = 256;  // S and O, 128 fp32 columns each (2 CTAs: all 512)
    static_assert(K == Kind::F16 || K == Kind::BF16 || K == Kind::F8 || K == Kind::Q8 || K == Kind::Q4 ||
                      K == Kind::Q3,
                  "16-bit rows, fp8 or integer codes");
    static_assert(!kChan || K == Kind::Q4, "per-channel / per-row scales: q4 codes");
    static_assert((kThreads / 16) % 8 == 0, "dequant rows of a thread share the swizzle phase");
};

// ---- tcgen05 / TMEM wrappers (PTX ISA 8.6+, sm_100a) ---------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* slot_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot_smem)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc05_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc05_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor: start, leading and stride byte offsets
// (16-byte units, 14 bits each), descriptor version 1 (bits 46..47), layout
// 128-byte swizzle (value 2 in bits 61..63).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp32 accumulator (bits 4..5 = 1), fp16
// A and B (formats 0), A K-major, B K-major or MN-major (bit 16), N >> 3 in
// bits 17..22, M >> 4 in bits 24..28.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int M, int N, bool b_mn_major) {
    return (1u << 4) | ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// The same with A (M x K, fp16) read from TMEM: lane m holds row m, 32-bit
// column c holds elements 2c (low half) and 2c + 1.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}
__device__ __forceinline__ void tmem_st32_u(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
        "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// Arrives on the mbarrier once all tcgen05.mma issued so far by this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp w of a
// warpgroup reads lanes 32 w .. 32 w + 31). The wait is in the same asm
// statement, so no use of the outputs can be scheduled before it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// The same load without the wait: two or more go out back to back, then one
// tmem_wait_ld_only, after which tmem_tie32 ties each group of 32 registers to
// the wait (an empty asm that redefines them), so no use is scheduled earlier.
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld_only() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_tie32(uint32_t* r) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
    uint32_t r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]),
        "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// sm_100 float forms that halve the softmax's instruction count: a
// three-input maximum, and paired fp32 FMA / add (two lanes in one 64-bit
// register pair).
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// Byte offset of (row, 16-byte chunk 0..15) in a swizzled 128 x 128 fp16 tile.
__host__ __device__ constexpr uint32_t pf_off(int row, int chunk) {
    return (uint32_t)((chunk >> 3) * 16384 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}

// fp16 pair {1024 + a, 1024 + b} from two bytes a, b < 256 placed by a byte
// permute next to the exponent byte 0x64 (1024 = 0x6400), then the code
// offset subtracted exactly (HSUB2) and the scale applied with one rounding
// (HMUL2): the same value as rounding code * scale from fp32.
__device__ __forceinline__ uint32_t pf_h2(uint32_t bytes, uint32_t sel, __half2 off, __half2 sc) {
    const uint32_t u = __byte_perm(bytes, 0x64646464u, sel);
    const __half2 h = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&u), off), sc);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Raw codes of dims 8 c .. 8 c + 7 of one cache row and the row's group
// scale. A thread loads all of its chunks first and converts them after, so
// the global-load latencies overlap instead of following one another (the
// shared-memory stores in between are through generic pointers, which the
// compiler will not move loads across).
template <Kind K>
struct PfRaw {
    uint32_t w[(K == Kind::F16 || K == Kind::BF16) ? 4 : (K == Kind::Q8 || K == Kind::F8) ? 2 : 1];
    __half sc;
};

// kScale: 0 = fp16 scales per 64-element group ([rows][2]), 1 = one scale per
// row ([rows]), 2 = none loaded (per-channel scales, applied by the caller).
template <Kind K, int kScale = 0>
__device__ __forceinline__ PfRaw<K> pf_load(const uint8_t* codes, const __half* scales, long long row, int c) {
    constexpr int kRb = PrefillCfg<K>::kRb;
    const uint8_t* src = codes + (size_t)row * kRb;
    PfRaw<K> r;
    if constexpr (K == Kind::F16 || K == Kind::BF16) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(src) + c);
        r.w[0] = v.x;
        r.w[1] = v.y;
        r.w[2] = v.z;
        r.w[3] = v.w;
        r.sc = __float2half(0.f);
    } else {
        if constexpr (kScale == 0) r.sc = __ldg(scales + (size_t)row * 2 + (c >> 3));
        else if constexpr (kScale == 1) r.sc = __ldg(scales + (size_t)row);
        else r.sc = __float2half(1.f);
        if constexpr (K == Kind::Q8 || K == Kind::F8) {
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(src) + c);
            r.w[0] = v.x;
            r.w[1] = v.y;
        } else if constexpr (K == Kind::Q4) {
            r.w[0] = __ldg(reinterpret_cast<const uint32_t*>(src) + c);
        } else {  // bits 24c .. 24c+23 of the row: two aligned words, funnel-shifted
            const uint32_t* w = reinterpret_cast<const uint32_t*>(src) + ((3 * c) >> 2);
            const uint32_t sh = 8u * ((3u * c) & 3u);
            const uint32_t lo = __ldg(w);
            const uint32_t hi = sh > 8u ? __ldg(w + 1) : 0u;  // word 1 only when the bytes straddle
            r.w[0] = __funnelshift_r(lo, hi, sh);
        }
    }
    return r;
}

// The chunk as 8 fp16 values.
template <Kind K>
__device__ __forceinline__ uint4 pf_convert(const PfRaw<K>& raw) {
    if constexpr (K == Kind::F16) {
        return make_uint4(raw.w[0], raw.w[1], raw.w[2], raw.w[3]);
    } else if constexpr (K == Kind::BF16) {
        // bf16 -> fp16: exact for values inside fp16's range (fp16 has the
        // longer mantissa); bf16 rows beyond it saturate to infinity
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&raw.w[i]));
            const __half2 h = __float22half2_rn(f);
            o[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
    } else if constexpr (K == Kind::F8) {
        // e4m3 pairs -> fp16 (exact), then the group scale with one rounding
        const __half2 sc = __half2half2(raw.sc);
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2_raw hr =
                __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(raw.w[i >> 1] >> (16 * (i & 1))), __NV_E4M3);
            const __half2 h = __hmul2(*reinterpret_cast<const __half2*>(&hr), sc);
            o[i] = *reinterpret_cast<const uint32_t*>(&h);
        }
        return make_uint4(o[0], o[1], o[2], o[3]);
    } else {
        const __half2 sc = __half2half2(raw.sc);
        uint4 r;
        if constexpr (K == Kind::Q8) {
            // signed byte + 128 = unsigned byte: 1024 + v + 128
            const __half2 off = __float2half2_rn(1152.f);
            const uint32_t a = raw.w[0] ^ 0x80808080u, b = raw.w[1] ^ 0x80808080u;
            r.x = pf_h2(a, 0x4140, off, sc);
            r.y = pf_h2(a, 0x4342, off, sc);
            r.z = pf_h2(b, 0x4140, off, sc);
            r.w = pf_h2(b, 0x4342, off, sc);
        } else if constexpr (K == Kind::Q4) {
            // byte b of the chunk holds dims 2b (low nibble) and 2b+1; nibble = code + 8
            const __half2 off = __float2half2_rn(1032.f);
            const uint32_t w = raw.w[0];
            const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
            const uint32_t p01 = __byte_perm(lo, hi, 0x5140), p23 = __byte_perm(lo, hi, 0x7362);
            r.x = pf_h2(p01, 0x4140, off, sc);
            r.y = pf_h2(p01, 0x4342, off, sc);
            r.z = pf_h2(p23, 0x4140, off, sc);
            r.w = pf_h2(p23, 0x4342, off, sc);
        } else {
            // field = code + 4; fields f0..f3 -> bytes of lo, f4..f7 -> bytes of hi
            const __half2 off = __float2half2_rn(1028.f);
            const uint32_t x = raw.w[0];
            const uint32_t lo = (x & 7u) | ((x << 5) & 0x700u) | ((x << 10) & 0x70000u) | ((x << 15) & 0x7000000u);
            const uint32_t y = x >> 12;
            const uint32_t hi = (y & 7u) | ((y << 5) & 0x700u) | ((y << 10) & 0x70000u) | ((y << 15) & 0x7000000u);
            r.x = pf_h2(lo, 0x4140, off, sc);
            r.y = pf_h2(lo, 0x4342, off, sc);
            r.z = pf_h2(hi, 0x4140, off, sc);
            r.w = pf_h2(hi, 0x4342, off, sc);
        }
        return r;
    }
}

// q4 chunk with a scale per dim pair (per-channel K scales of the chunk's 8 dims).
__device__ __forceinline__ uint4 pf_convert_q4_chan(uint32_t w, const __half2* sc4) {
    const __half2 off = __float2half2_rn(1032.f);
    const uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
    const uint32_t p01 = __byte_perm(lo, hi, 0x5140), p23 = __byte_perm(lo, hi, 0x7362);
    return make_uint4(pf_h2(p01, 0x4140, off, sc4[0]), pf_h2(p01, 0x4342, off, sc4[1]), pf_h2(p23, 0x4140, off, sc4[2]),
                      pf_h2(p23, 0x4342, off, sc4[3]));
}

__device__ __forceinline__ void sts128_generic(uint8_t* base, uint32_t off, uint4 v) {
    *reinterpret_cast<uint4*>(base + off) = v;
}

template <class C, bool kPaged>
__global__ void __launch_bounds__(C::kThreads, 2) prefill_tc_kernel(const PrefillParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* sQ = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sK = sQ + C::kTile;
    uint8_t* sV = sK + C::kTile;
    uint64_t* bar_s = reinterpret_cast<uint64_t*>(sV + C::kTile);
    uint64_t* bar_o = bar_s + 1;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(bar_o + 1);
    volatile int* fail = reinterpret_cast<volatile int*>(tslot + 1);
    float* xch = reinterpret_cast<float*>(bar_s + 8);  // [2][128]: the half-rows' maxima / sums

    constexpr int D = C::kD;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nqb = (int)gridDim.x;
    const int qb = nqb - 1 - (int)blockIdx.x;  // the longest (last) token blocks start first
    const int h = (int)blockIdx.y;
    const int hk = h / (p.Hq / p.Hkv);
    const int q0 = qb * C::kBq;
    const long long off0 = (long long)p.L - p.Lq;  // cache row of token 0

    if (warp == 0) tmem_alloc(tslot, C::kTmemCols);
    if (tid == 0) {
        mbar_init(bar_s, 1);
        mbar_init(bar_o, 1);
        *fail = 0;
        fence_mbar_init();
    }
    // this CTA's query tokens -> sQ (rows past Lq are zero)
    for (int i = tid; i < C::kBq * 16; i += C::kThreads) {
        const int r = i >> 4, c = i & 15;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (q0 + r < p.Lq)
            v = __ldg(reinterpret_cast<const uint4*>(p.q + ((size_t)h * p.Lq + q0 + r) * D) + c);
        sts128_generic(sQ, pf_off(r, c), v);
    }
    tc05_fence_before();
    __syncthreads();
    tc05_fence_after();
    const uint32_t tbase = *tslot;
    const uint32_t tS = tbase, tO = tbase + 128;
    const uint32_t sQa = smem_u32(sQ), sKa = smem_u32(sK), sVa = smem_u32(sV);
    constexpr uint32_t kIdescS = umma_idesc_f16(128, 128, false);
    constexpr uint32_t kIdescO = umma_idesc_f16(128, 128, true);

    // cache rows this CTA needs: [0, last], last = min(L - 1, off0 + q0 + 127)
    const long long last = min((long long)p.L - 1, off0 + q0 + C::kBq - 1);
    const int nkb = (int)(last / C::kBk) + 1;
    // softmax: every thread; warpgroup hf takes columns [64 hf, 64 hf + 64)
    // of its token row (TMEM lane = row) of S, P and O
    const int hf = warp >> 2;
    const int row = tid & 127;
    const long long vis = off0 + q0 + row;  // last visible cache row of this token
    const float qk_scale = rsqrtf((float)D) * kLog2e;
    float m = kNegMax, l = 0.f;
    const uint32_t lane_addr = ((uint32_t)((warp & 3) * 32) << 16) + 64 * hf;

    // one matrix (K or V) of cache block kb, dequantized into its tile. Thread
    // tid takes chunk c = tid % 16 of rows tid / 16 + 16 t: one base row per
    // block, the rest constant offsets (rows 16 apart keep the swizzle phase,
    // so the shared-memory offsets are constant too). All loads go out first.
    // q4c+: this thread's 8 dims (chunk tid % 16) of the KV head's channel scales
    __half2 kcs[4];
    if constexpr (C::kChan) {
        const __half* cs = p.scK + (size_t)hk * D + 8 * (tid & 15);
#pragma unroll
        for (int i = 0; i < 4; ++i) kcs[i] = __halves2half2(__ldg(cs + 2 * i), __ldg(cs + 2 * i + 1));
    }
    const auto dequant = [&](auto is_k, int kb, const uint8_t* codes, const __half* scales, uint8_t* dst) {
        // scale layout of this matrix: groups, or q4c+ channels (K) / rows (V)
        constexpr int kScale = !C::kChan ? 0 : decltype(is_k)::value ? 2 : 1;
        constexpr int kPer = C::kBk * 16 / C::kThreads;  // chunks per thread
        constexpr int kRowStep = C::kThreads / 16;
        const long long r0 = (long long)kb * C::kBk;
        const int c = tid & 15, rr = tid >> 4;
        PfRaw<C::kKind> raw[kPer];
        if constexpr (kPaged) {  // through the block table, row by row
#pragma unroll
            for (int t = 0; t < kPer; ++t) {
                const int gr = (int)min(r0 + rr + kRowStep * t, (long long)p.L - 1);  // L < 2^31: 32-bit division
                const int pi = gr / p.page_rows;
                int pg = __ldg(p.block_table + pi);
                pg = (pg >= 0 && pg < p.num_pages) ? pg : 0;
                const long long grow = ((long long)pg * p.Hkv + hk) * p.page_rows + (gr - pi * p.page_rows);
                raw[t] = pf_load<C::kKind, kScale>(codes, scales, grow, c);
            }
        } else if (r0 + C::kBk <= p.L) {
            const long long grow = (long long)hk * p.L + r0 + rr;
#pragma unroll
            for (int t = 0; t < kPer; ++t) raw[t] = pf_load<C::kKind, kScale>(codes, scales, grow + kRowStep * t, c);
        } else {  // the cache's last block: rows past L repeat row L - 1 (masked, weight 0)
#pragma unroll
            for (int t = 0; t < kPer; ++t) {
                const long long grow = (long long)hk * p.L + min(r0 + rr + kRowStep * t, (long long)p.L - 1);
                raw[t] = pf_load<C::kKind, kScale>(codes, scales, grow, c);
            }
        }
        const uint32_t so = pf_off(rr, c);
#pragma unroll
        for (int t = 0; t < kPer; ++t) {
            if constexpr (kScale == 2)
                sts128_generic(dst, so + kRowStep * 128 * t, pf_convert_q4_chan(raw[t].w[0], kcs));
            else
                sts128_generic(dst, so + kRowStep * 128 * t, pf_convert<C::kKind>(raw[t]));
        }
    };
    const auto issue_s = [&]() {  // S = Q K^T of the block in the K tile
        if (tid == 0) {
            tc05_fence_after();
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t o = (uint32_t)((kk >> 2) * 16384 + (kk & 3) * 32);
                umma_f16(tS, umma_desc_sw128(sQa + o, 16, 1024), umma_desc_sw128(sKa + o, 16, 1024), kIdescS,
                         kk > 0);
            }
            umma_commit(bar_s);
        }
    };
    // Schedule per block kb: wait S(kb); softmax; issue PV(kb); dequantize
    // K(kb+1) while PV(kb) runs (S(kb) has read K); wait PV(kb); issue
    // S(kb+1); dequantize V(kb+1) while S(kb+1) runs (PV(kb) has read V).
    using kIsK = std::integral_constant<bool, true>;
    using kIsV = std::integral_constant<bool, false>;
    dequant(kIsK{}, 0, p.K, p.scK, sK);
    dequant(kIsV{}, 0, p.V, p.scV, sV);
    fence_proxy_async_smem();
    tc05_fence_before();
    __syncthreads();
    issue_s();
    for (int kb = 0; kb < nkb; ++kb) {
        const long long r0 = (long long)kb * C::kBk;
        const bool ok_s = mbar_wait_bounded(bar_s, (uint32_t)kb & 1u);
        if (!ok_s && lane == 0) report_error(kErrFullWait);
        tc05_fence_after();
        // (a failed wait is agreed on at the row-max exchange below, the next
        // CTA barrier; until then the thread only reads TMEM)
        // 3. online softmax of this thread's half token row; P -> sP; rescale O
        {
            // two passes over S in TMEM (the row maximum, then the weights).
            // Columns j <= lim of this block are visible to the row: all of
            // them below the diagonal, none past the cache's end.
            const int lim = (int)max(-1ll, min(min(vis, (long long)p.L - 1) - r0, (long long)C::kBk - 1)) - 64 * hf;
            const bool full = lim >= 63;
            float bm0 = kNegMax, bm1 = kNegMax;
            {
                uint32_t s[2][32];
                tmem_ld32_nowait(tS + lane_addr, s[0]);
                tmem_ld32_nowait(tS + lane_addr + 32, s[1]);
                tmem_wait_ld_only();
                tmem_tie32(s[0]);
                tmem_tie32(s[1]);
#pragma unroll
                for (int j = 0; j < 64; j += 2) {
                    const float x0 = __uint_as_float(s[j >> 5][j & 31]), x1 = __uint_as_float(s[j >> 5][(j & 31) + 1]);
                    if (full) {
                        if (j & 2) bm1 = fmax3f(bm1, x0, x1);
                        else bm0 = fmax3f(bm0, x0, x1);
                    } else {
                        if (j <= lim) bm0 = fmaxf(bm0, x0);
                        if (j + 1 <= lim) bm1 = fmaxf(bm1, x1);
                    }
                }
            }
            // the row's maximum over both halves
            xch[hf * 128 + row] = fmaxf(bm0, bm1);
            if (__syncthreads_or(!ok_s)) {  // every thread leaves together
                if (tid == 0) *fail = 1;
                break;
            }
            const float bm = fmaxf(xch[row], xch[128 + row]);
            // the reference maximum moves only when the block's maximum exceeds
            // it by more than 8 (log2 units): weights stay <= 256, exact in
            // relative terms in fp16, and O is rarely rescaled. O and l share
            // the reference, so the result is the same. Both halves of a row
            // take the same decision (same m, same exchanged maximum).
            const float bms = bm * qk_scale;
            const float mnew = bms > m + 8.f ? bms : m;
            const float corr = fast_exp2(m - mnew);
            m = mnew;
            float2 sum2 = make_float2(0.f, 0.f);
            uint32_t pw[32];  // P of keys 64 hf .. 64 hf + 63 as fp16 pairs
            const float2 sc2 = make_float2(qk_scale, qk_scale), nm2 = make_float2(-mnew, -mnew);
#pragma unroll
            for (int cb = 0; cb < 2; ++cb) {
                float s[32];
                tmem_ld32(tS + lane_addr + 32 * cb, s);
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int j = 32 * cb + 8 * c4 + 2 * i;  // column 64 hf + j
                        const float2 x = ffma2(make_float2(s[j & 31], s[(j & 31) + 1]), sc2, nm2);
                        float a = fast_exp2(x.x);
                        float b = fast_exp2(x.y);
                        if (!full) {
                            a = j <= lim ? a : 0.f;
                            b = j + 1 <= lim ? b : 0.f;
                        }
                        sum2 = fadd2(sum2, make_float2(a, b));
                        const __half2 hp = __floats2half2_rn(a, b);
                        pw[j >> 1] = *reinterpret_cast<const uint32_t*>(&hp);
                    }
                }
            }
            // P into the first 32 of this half's S columns (all read above), the
            // A operand of O += P V
            tmem_st32_u(tS + lane_addr, pw);
            tmem_wait_st();
            l = l * corr + (sum2.x + sum2.y);  // this half's share of the row sum
            if (kb > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
#pragma unroll
                for (int cb = 0; cb < 2; ++cb) {
                    float o[32];
                    tmem_ld32(tO + lane_addr + 32 * cb, o);
#pragma unroll
                    for (int i = 0; i < 32; ++i) o[i] *= corr;
                    tmem_st32(tO + lane_addr + 32 * cb, o);
                }
                tmem_wait_st();
            }
        }
        tc05_fence_before();
        __syncthreads();
        // 4. O += P V
        if (tid == 0) {
            tc05_fence_after();
#pragma unroll
            for (int kk = 0; kk < C::kBk / 16; ++kk) {
                // keys 16 kk .. 16 kk + 15: TMEM columns 64 (kk / 4) + 8 (kk % 4)
                const uint32_t ta = tS + (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8);
                const uint32_t ob = (uint32_t)(kk * 16 * 128);  // 16 cache rows of 128 bytes per panel
                umma_f16_ts(tO, ta, umma_desc_sw128(sVa + ob, 16384, 1024), kIdescO, kb > 0 || kk > 0);
            }
            umma_commit(bar_o);
        }
        const bool more = kb + 1 < nkb;
        if (more) dequant(kIsK{}, kb + 1, p.K, p.scK, sK);
        const bool ok_o = mbar_wait_bounded(bar_o, (uint32_t)kb & 1u);
        if (!ok_o && lane == 0) report_error(kErrFullWait);
        tc05_fence_after();
        if (more) fence_proxy_async_smem();
        if (__syncthreads_or(!ok_o)) {
            if (tid == 0) *fail = 1;
            break;
        }
        if (more) {
            issue_s();
            dequant(kIsV{}, kb + 1, p.V, p.scV, sV);
            fence_proxy_async_smem();
        }
    }
    // epilogue: out = O / l for the CTA's valid tokens (l: both halves' sums)
    __syncthreads();
    xch[hf * 128 + row] = l;
    __syncthreads();
    if (!*fail) {
        const float inv = 1.f / (xch[row] + xch[128 + row]);
#pragma unroll
        for (int cb = 0; cb < 2; ++cb) {
            float o[32];
            tmem_ld32(tO + lane_addr + 32 * cb, o);
            if (q0 + row < p.Lq) {
                uint4* dst =
                    reinterpret_cast<uint4*>(p.out + ((size_t)h * p.Lq + q0 + row) * D + 64 * hf + 32 * cb);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint32_t w[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const __half2 hp = __floats2half2_rn(o[8 * c + 2 * i] * inv, o[8 * c + 2 * i + 1] * inv);
                        w[i] = *reinterpret_cast<const uint32_t*>(&hp);
                    }
                    dst[c] = make_uint4(w[0], w[1], w[2], w[3]);
                }
            }
        }
    }
    tc05_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc05_fence_after();
        tmem_dealloc(tbase, C::kTmemCols);
    }
}

// ---- staged prefill: the cache dequantized once, K/V tiles by TMA -----------------
//
// The kernel above dequantizes every K/V block in each CTA that reads it: with
// Hq / Hkv query heads per KV head the same block is converted Hq / Hkv times,
// and the conversion takes issue slots from the softmax. The staged variant
// converts the cache rows [0, L) of every KV head once into fp16 rows of a
// staging buffer [Hkv][Lpad][D] (Lpad = L rounded up to 128 rows, the pad rows
// zero), with the same arithmetic (pf_load / pf_convert, so the fp16 values
// are identical), and the attention kernel then moves K/V tiles into shared
// memory with 2-D tensor copies (cp.async.bulk.tensor, 128-byte swizzle, two
// 64-dim boxes per tile, no multicast): one thread issues them, no thread
// converts.

// One thread per 16-byte chunk (8 dims) of a staging row; blockIdx.y = 0: K,
// 1: V. Paged caches are gathered through the block table here.
template <class C, bool kPaged>
__global__ void __launch_bounds__(256) prefill_stage_kernel(const PrefillParams p, __half* __restrict__ stK,
                                                            __half* __restrict__ stV, int Lpad) {
    const bool is_k = blockIdx.y == 0;
    __half* dst = is_k ? stK : stV;
    const uint8_t* codes = is_k ? p.K : p.V;
    const __half* scales = is_k ? p.scK : p.scV;
    const long long n = (long long)p.Hkv * Lpad * 16;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int c = (int)(i & 15);
        const long long rr = i >> 4;  // staging row: (hk, j)
        const int hk = (int)(rr / Lpad);
        const int j = (int)(rr - (long long)hk * Lpad);
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (j < p.L) {
            long long grow;
            if constexpr (kPaged) {
                const int pi = j / p.page_rows;
                int pg = __ldg(p.block_table + pi);
                pg = (pg >= 0 && pg < p.num_pages) ? pg : 0;
                grow = ((long long)pg * p.Hkv + hk) * p.page_rows + (j - pi * p.page_rows);
            } else {
                grow = (long long)hk * p.L + j;
            }
            if constexpr (C::kChan) {
                if (is_k) {  // per-channel scales of the chunk's 8 dims
                    const __half* cs = p.scK + (size_t)hk * C::kD + 8 * c;
                    __half2 kcs[4];
#pragma unroll
                    for (int t = 0; t < 4; ++t) kcs[t] = __halves2half2(__ldg(cs + 2 * t), __ldg(cs + 2 * t + 1));
                    v = pf_convert_q4_chan(pf_load<C::kKind, 2>(codes, scales, grow, c).w[0], kcs);
                } else {
                    v = pf_convert<C::kKind>(pf_load<C::kKind, 1>(codes, scales, grow, c));
                }
            } else {
                v = pf_convert<C::kKind>(pf_load<C::kKind, 0>(codes, scales, grow, c));
            }
        }
        reinterpret_cast<uint4*>(dst)[i] = v;
    }
}

// 2-D tensor copy of a box of the fp16 staging rows into shared memory.
__device__ __forceinline__ void pf_tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

}  // namespace va
