// KV formats: geometry and in-register dequantization of one lane's slice of
// a row. Layouts follow the reference exactly (src/voltattn.cu:189-190 q8,
// :254-256 q4 nibble order, :563-600 q3 granules, :694-745 scales).
//
// Conversions avoid the integer->float converter: a code is placed in the low
// mantissa bits of 2^23 (bit pattern 0x4B000000 | u) and the bias subtracted
// with one FADD, which is exact for |u| < 2^23.
#pragma once

#include "common.cuh"

namespace va {

enum class Kind : int { F16 = 0, Q8 = 1, Q4 = 2, Q3 = 3, BF16 = 4, F8 = 5 };

// Kinds decoded in floating point by the streaming kernel: fp16 and bf16 rows
// (no scales) and fp8 e4m3 codes with per-group fp16 scales.
__host__ __device__ constexpr bool is_float_kind(Kind k) {
    return k == Kind::F16 || k == Kind::BF16 || k == Kind::F8;
}

template <Kind K>
struct KindTraits;

template <>
struct KindTraits<Kind::F16> {
    static constexpr int kBits = 16;
    static constexpr int kDpl = 16;  // dims per lane in the staged kernel
};
template <>
struct KindTraits<Kind::Q8> {
    static constexpr int kBits = 8;
    static constexpr int kDpl = 16;
};
template <>
struct KindTraits<Kind::Q4> {
    static constexpr int kBits = 4;
    static constexpr int kDpl = 32;
};
template <>
struct KindTraits<Kind::Q3> {
    static constexpr int kBits = 3;
    static constexpr int kDpl = 32;
};
template <>
struct KindTraits<Kind::BF16> {
    static constexpr int kBits = 16;
    static constexpr int kDpl = 16;
};
template <>
struct KindTraits<Kind::F8> {
    static constexpr int kBits = 8;
    static constexpr int kDpl = 16;
};

// Raw bytes of one lane's DPL dims: 32 B (f16), 16 B (q8, q4), 12 B (q3).
template <Kind K>
struct LaneRaw {
    static constexpr int kWords = KindTraits<K>::kDpl * KindTraits<K>::kBits / 32;
    uint32_t w[kWords];
};

// Loads a lane slice from shared memory (16-byte aligned for f16/q8/q4,
// 4-byte aligned for q3).
template <Kind K>
__device__ __forceinline__ void load_lane(LaneRaw<K>& r, const uint8_t* p) {
    if constexpr (K == Kind::Q3) {
        const uint32_t* p32 = reinterpret_cast<const uint32_t*>(p);
#pragma unroll
        for (int i = 0; i < 3; ++i) r.w[i] = p32[i];
    } else {
        const uint4* p128 = reinterpret_cast<const uint4*>(p);
#pragma unroll
        for (int i = 0; i < LaneRaw<K>::kWords / 4; ++i) {
            const uint4 v = p128[i];
            r.w[4 * i + 0] = v.x;
            r.w[4 * i + 1] = v.y;
            r.w[4 * i + 2] = v.z;
            r.w[4 * i + 3] = v.w;
        }
    }
}

template <Kind K>
__device__ __forceinline__ void zero_lane(LaneRaw<K>& r) {
#pragma unroll
    for (int i = 0; i < LaneRaw<K>::kWords; ++i) r.w[i] = 0u;
}

// Value of dim i (0 <= i < DPL) of a lane slice, as the exact integer code
// (quantized kinds) or the fp16 value (f16), in fp32.
template <Kind K, int I>
__device__ __forceinline__ float lane_value(const LaneRaw<K>& r) {
    if constexpr (K == Kind::F16) {
        const uint32_t w = r.w[I / 2];
        const __half2 h2 = *reinterpret_cast<const __half2*>(&w);
        return (I & 1) ? __high2float(h2) : __low2float(h2);
    } else if constexpr (K == Kind::Q8) {
        // byte I%4 of word I/4, biased to unsigned (v + 128), into 2^23's mantissa
        const uint32_t u = r.w[I / 4] ^ 0x80808080u;
        const uint32_t bits = __byte_perm(u, 0x4B000000u, 0x7540u + (I & 3));
        return __uint_as_float(bits) - 8388736.0f;  // 2^23 + 128
    } else if constexpr (K == Kind::Q4) {
        // dims 2k / 2k+1 are the low / high nibble of byte k: nibble I of the
        // little-endian word stream, nibble = v + 8
        const uint32_t w = r.w[I / 8];
        constexpr int sh = 4 * (I % 8);
        const uint32_t bits = ((w >> sh) & 0xFu) | 0x4B000000u;
        return __uint_as_float(bits) - 8388616.0f;  // 2^23 + 8
    } else {
        // element I at bit 3*I of the lane's 96-bit little-endian stream
        // (the lane slice starts on a granule boundary), field = v + 4
        constexpr int bit = 3 * I;
        constexpr int wi = bit / 32;
        constexpr int off = bit % 32;
        uint32_t x;
        if constexpr (off <= 29) {
            x = r.w[wi] >> off;
        } else {
            x = __funnelshift_r(r.w[wi], r.w[wi + 1], off);
        }
        const uint32_t bits = (x & 7u) | 0x4B000000u;
        return __uint_as_float(bits) - 8388612.0f;  // 2^23 + 4
    }
}

template <Kind K, int I = 0>
__device__ __forceinline__ float lane_dot(const LaneRaw<K>& r, const float* qf, float acc) {
    if constexpr (I < KindTraits<K>::kDpl) {
        acc = fmaf(qf[I], lane_value<K, I>(r), acc);
        return lane_dot<K, I + 1>(r, qf, acc);
    } else {
        return acc;
    }
}

template <Kind K, int I = 0>
__device__ __forceinline__ void lane_axpy(const LaneRaw<K>& r, float w, float* o) {
    if constexpr (I < KindTraits<K>::kDpl) {
        o[I] = fmaf(w, lane_value<K, I>(r), o[I]);
        lane_axpy<K, I + 1>(r, w, o);
    }
}

}  // namespace va
