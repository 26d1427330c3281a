// KV group quantizer / packer as a GPU kernel, bit-exact with the reference's
// host quantize() (src/voltattn.cu:705-745):
//   amax = max_i |x_i| over a 64-element group (nan elements ignored, as
//          std::max(amax, fabs(nan)) keeps amax);
//   s    = amax > 0 ? amax / lim : 1   (IEEE fp32 division), stored as fp16 (RNE);
//   v    = (int)lrint(x / stored_scale) (IEEE division, round-half-even), then
//          clamped to [-lim, lim]. lrint of nan / |y| >= 2^63 yields the x86-64
//          "integer indefinite" LONG_MIN whose low 32 bits are 0; finite values
//          narrow to int by keeping the low 32 bits — both reproduced here;
//   packing: q8 int8; q4 nibble (v+8), even element low; q3 field (v+4) at bits
//          3*(e%8) of the little-endian 3-byte granule e/8.
// Eight threads own one group (eight consecutive elements each, two 16-byte
// loads), reduce amax with three shuffles and write one packed word each.
#pragma once

#include "common.cuh"

namespace va {

__device__ __forceinline__ int lrint_narrow(float y) {
    if (!(fabsf(y) < 9.2233720368547758e18f)) return 0;  // nan, +-inf, |y| >= 2^63
    const long long t = __float2ll_rn(y);                 // round half to even
    return (int)(unsigned int)(unsigned long long)t;
}

// BITS value of the fp8 format (f8+, no reference counterpart): e4m3 codes
// with the same group rule, lim = 448 (the largest finite e4m3 value):
// s = amax > 0 ? amax / 448 : 1 stored as fp16, code = e4m3(x / stored s)
// rounded to nearest even with saturation to +-448 (nan stays nan).
constexpr int kBitsF8 = -8;

// One 64-element group, eight consecutive elements per thread (8 lanes per
// group, lane-aligned): loads, reduces amax over the 8 lanes, quantizes and
// packs. `src` points at this thread's 8 inputs; element `e0` (a multiple of
// 8) and scale index `sidx` place the result. All 32 lanes must call it.
template <int BITS>
__device__ __forceinline__ void quantize_group_part(const float* src, bool active, int part, long long e0,
                                                    long long sidx, uint8_t* __restrict__ codes,
                                                    __half* __restrict__ scales) {
    constexpr int lim = BITS == 8 ? 127 : BITS == 4 ? 7 : BITS == kBitsF8 ? 448 : 3;
    float v[8];
    if (active) {
        const float4* p = reinterpret_cast<const float4*>(src);
        const float4 a = __ldg(p), b = __ldg(p + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));  // fmaxf drops nan operands
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (!active) return;

    const float s = amax > 0.f ? __fdiv_rn(amax, (float)lim) : 1.f;
    const __half hs = __float2half_rn(s);
    const float sh = __half2float(hs);
    if constexpr (BITS == kBitsF8) {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0 |= (uint32_t)__nv_cvt_float_to_fp8(__fdiv_rn(v[i], sh), __NV_SATFINITE, __NV_E4M3) << (8 * i);
            w1 |= (uint32_t)__nv_cvt_float_to_fp8(__fdiv_rn(v[4 + i], sh), __NV_SATFINITE, __NV_E4M3) << (8 * i);
        }
        *reinterpret_cast<uint2*>(codes + e0) = make_uint2(w0, w1);
        if (part == 0) scales[sidx] = hs;
        return;
    }
    int c[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = max(-lim, min(lim, lrint_narrow(__fdiv_rn(v[i], sh))));

    if constexpr (BITS == 8) {
        uint32_t w0 = 0, w1 = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0 |= (uint32_t)(uint8_t)(int8_t)c[i] << (8 * i);
            w1 |= (uint32_t)(uint8_t)(int8_t)c[4 + i] << (8 * i);
        }
        *reinterpret_cast<uint2*>(codes + e0) = make_uint2(w0, w1);
    } else if constexpr (BITS == 4) {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) w |= (uint32_t)(c[i] + 8) << (4 * i);
        *reinterpret_cast<uint32_t*>(codes + e0 / 2) = w;
    } else {
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) w |= (uint32_t)(c[i] + 4) << (3 * i);
        uint8_t* dst = codes + (e0 / 8) * 3;
        dst[0] = (uint8_t)w;
        dst[1] = (uint8_t)(w >> 8);
        dst[2] = (uint8_t)(w >> 16);
    }
    if (part == 0) scales[sidx] = hs;
}

template <int BITS>
__global__ void __launch_bounds__(256) quantize_kernel(const float* __restrict__ x, uint8_t* __restrict__ codes,
                                                       __half* __restrict__ scales, long long ngroups) {
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long grp = tid >> 3;
    const int part = (int)(tid & 7);
    const bool active = grp < ngroups;
    quantize_group_part<BITS>(x + (active ? grp * kGroup + part * 8 : 0), active, part, grp * kGroup + part * 8,
                              grp, codes, scales);
}

// q4c+ (no reference counterpart, the layout of KIVI-style caches): K with a
// static scale per (head, channel) over all positions, V with one scale per
// row. Both follow the group rule above with the group being a channel's L
// values (K) or a row's D values (V): s = amax > 0 ? amax / lim : 1 stored as
// fp16, code = lrint(x / stored s) narrowed and clamped, packed as q8 / q4.

// Per-channel K: CTA (head, 32-channel block), 256 threads = 32 channels x 8
// row phases. Pass 1: channel amax over the head's L rows; pass 2: codes.
template <int BITS>
__global__ void __launch_bounds__(256) quantize_kchan_kernel(const float* __restrict__ x, uint8_t* __restrict__ codes,
                                                             __half* __restrict__ scales, int L, int D) {
    constexpr int lim = BITS == 8 ? 127 : 7;
    const int h = blockIdx.y, d = blockIdx.x * 32 + (threadIdx.x & 31), ph = threadIdx.x >> 5;
    const float* xh = x + (size_t)h * L * D;
    float amax = 0.f;
    for (int j = ph; j < L; j += 8) amax = fmaxf(amax, fabsf(__ldg(xh + (size_t)j * D + d)));  // drops nan
    __shared__ float red[8][32];
    __shared__ float shs[32];
    red[ph][threadIdx.x & 31] = amax;
    __syncthreads();
    if (ph == 0) {
        for (int k = 1; k < 8; ++k) amax = fmaxf(amax, red[k][threadIdx.x & 31]);
        const float sv = amax > 0.f ? __fdiv_rn(amax, (float)lim) : 1.f;
        const __half hs = __float2half_rn(sv);
        scales[(size_t)h * D + d] = hs;
        shs[threadIdx.x & 31] = __half2float(hs);
    }
    __syncthreads();
    const float sh = shs[threadIdx.x & 31];
    for (int j = ph; j < L; j += 8) {
        const int c = max(-lim, min(lim, lrint_narrow(__fdiv_rn(__ldg(xh + (size_t)j * D + d), sh))));
        const size_t e = ((size_t)h * L + j) * D + d;
        if constexpr (BITS == 8) {
            codes[e] = (uint8_t)(int8_t)c;
        } else {
            // dims 2k (low nibble) and 2k+1 (high) of a byte: the even lane writes
            const int hi = __shfl_down_sync(0xffffffffu, c, 1);
            if ((d & 1) == 0) codes[e / 2] = (uint8_t)((c + 8) | ((hi + 8) << 4));
        }
    }
}

// Per-token V: one warp per row, D / 32 consecutive dims per lane.
template <int BITS>
__global__ void __launch_bounds__(256) quantize_vtok_kernel(const float* __restrict__ x, uint8_t* __restrict__ codes,
                                                            __half* __restrict__ scales, long long rows, int D) {
    constexpr int lim = BITS == 8 ? 127 : 7;
    const long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    const int per = D / 32;  // 4 (D = 128) or 2 (D = 64)
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (r < rows)
        for (int i = 0; i < per; ++i) v[i] = __ldg(x + r * D + lane * per + i);
    float amax = 0.f;
    for (int i = 0; i < per; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if (r >= rows) return;
    const float sv = amax > 0.f ? __fdiv_rn(amax, (float)lim) : 1.f;
    const __half hs = __float2half_rn(sv);
    const float sh = __half2float(hs);
    if (lane == 0) scales[r] = hs;
    uint32_t w = 0;
    for (int i = 0; i < per; ++i) {
        const int c = max(-lim, min(lim, lrint_narrow(__fdiv_rn(v[i], sh))));
        w |= BITS == 8 ? (uint32_t)(uint8_t)(int8_t)c << (8 * i) : (uint32_t)(c + 8) << (4 * i);
    }
    uint8_t* dst = codes + (size_t)r * D * BITS / 8 + (size_t)lane * per * BITS / 8;
    for (int i = 0; i < per * BITS / 8; ++i) dst[i] = (uint8_t)(w >> (8 * i));
}

// KV append: new rows x [B*Hkv][D] (one token per sequence) quantized into a
// cache [B][Hkv][Lcap][D] at row pos[b] of every KV head of sequence b, with
// the same arithmetic as quantize_kernel (the rows come out exactly as if the
// whole cache had been quantized at once). BITS = 16 stores fp16 rows.
// Page map of a paged cache for append_kernel (table == nullptr: the
// capacity-padded [B][Hkv][Lcap] layout).
struct PageMap {
    const int* table;
    int max_pages, rows, num_pages;
};

template <int BITS>
__global__ void __launch_bounds__(256) append_kernel(const float* __restrict__ x, uint8_t* __restrict__ codes,
                                                     __half* __restrict__ scales, int Hkv, int Lcap, int D,
                                                     const int* __restrict__ pos, long long nrows, PageMap pm) {
    const int G = D / kGroup;
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long grp = tid >> 3;  // source group: row grp / G, group grp % G
    const int part = (int)(tid & 7);
    const long long rs = grp / G;
    const int gi = (int)(grp - rs * G);
    const bool active = rs < nrows;
    long long rd = 0;
    bool inb = false;
    if (active) {
        const int b = (int)(rs / Hkv);
        const int p = __ldg(pos + b);
        if (pm.table) {
            // paged: row p of the sequence lives in page table[b][p / rows]
            const int kvh = (int)(rs - (long long)b * Hkv);
            const int pg = p >= 0 ? p / pm.rows : -1;
            const int pp = (pg >= 0 && pg < pm.max_pages) ? __ldg(pm.table + (size_t)b * pm.max_pages + pg) : -1;
            inb = pp >= 0 && pp < pm.num_pages;
            rd = inb ? ((long long)pp * Hkv + kvh) * pm.rows + p % pm.rows : 0;
        } else {
            inb = p >= 0 && p < Lcap;
            rd = rs * (long long)Lcap + (inb ? p : 0);  // (b*Hkv + kvh)*Lcap + pos[b]
        }
    }
    const float* src = x + (active ? rs * D + gi * kGroup + part * 8 : 0);
    if constexpr (BITS == 16) {
        if (active && inb) {
            const float4* p4 = reinterpret_cast<const float4*>(src);
            const float4 a = __ldg(p4), c = __ldg(p4 + 1);
            __half2 h[4] = {__floats2half2_rn(a.x, a.y), __floats2half2_rn(a.z, a.w), __floats2half2_rn(c.x, c.y),
                            __floats2half2_rn(c.z, c.w)};
            *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(codes) + rd * D + gi * kGroup + part * 8) =
                *reinterpret_cast<uint4*>(h);
        }
    } else {
        quantize_group_part<BITS>(src, active && inb, part, rd * D + gi * kGroup + part * 8, rd * G + gi, codes,
                                  scales);
    }
}

}  // namespace va
