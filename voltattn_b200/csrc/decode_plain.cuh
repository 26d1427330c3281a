// Plain decode kernels: the f16 / q8 / q4 members of the reference's kernel
// family (src/voltattn.cu:122-320), kept as attribution baselines next to the
// staged "+" kernels. One warp per KV position with the 32 lanes across D
// (D/32 dims per lane), plain global loads, one online-softmax chain per
// warp, WARPS warps per block merged in shared memory into one workspace slot
// per (head, split); the separate combine kernel then merges the S slots
// (two launches, as the reference does).
#pragma once

#include "common.cuh"
#include "lse_merge.cuh"

namespace va {

constexpr int kPlainWarps = 4;

template <int BITS, int P>
struct PlainLane;

// f16: P halves
template <int P>
struct PlainLane<16, P> {
    __device__ static void load(const uint8_t* base, size_t row, int lane, float* v, float scale) {
        (void)scale;
        const __half* p = reinterpret_cast<const __half*>(base) + row * (32 * P) + lane * P;
        if constexpr (P == 4) {
            const uint2 w = *reinterpret_cast<const uint2*>(p);
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
            v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
        } else {
            const uint32_t w = *reinterpret_cast<const uint32_t*>(p);
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w));
            v[0] = a.x; v[1] = a.y;
        }
    }
};

// q8: P int8 codes
template <int P>
struct PlainLane<8, P> {
    __device__ static void load(const uint8_t* base, size_t row, int lane, float* v, float scale) {
        const int8_t* p = reinterpret_cast<const int8_t*>(base) + row * (32 * P) + lane * P;
        if constexpr (P == 4) {
            const char4 c = *reinterpret_cast<const char4*>(p);
            v[0] = c.x * scale; v[1] = c.y * scale; v[2] = c.z * scale; v[3] = c.w * scale;
        } else {
            const char2 c = *reinterpret_cast<const char2*>(p);
            v[0] = c.x * scale; v[1] = c.y * scale;
        }
    }
};

// q4: P nibbles (P/2 bytes), low nibble = even dim, value = nibble - 8
template <int P>
struct PlainLane<4, P> {
    __device__ static void load(const uint8_t* base, size_t row, int lane, float* v, float scale) {
        const uint8_t* p = base + row * (16 * P) + lane * (P / 2);
        uint32_t w;
        if constexpr (P == 4) w = *reinterpret_cast<const uint16_t*>(p);
        else w = *p;
#pragma unroll
        for (int i = 0; i < P; ++i) v[i] = (float)((int)((w >> (4 * i)) & 0xFu) - 8) * scale;
    }
};

template <int BITS, int D>
__global__ void __launch_bounds__(32 * kPlainWarps) decode_plain_kernel(const uint8_t* __restrict__ K,
                                                                        const uint8_t* __restrict__ V,
                                                                        const __half* __restrict__ scK,
                                                                        const __half* __restrict__ scV,
                                                                        const __half* __restrict__ q,
                                                                        float* __restrict__ ws, int L, int S,
                                                                        int chunk) {
    constexpr int P = D / 32;
    constexpr int G = D / kGroup;
    const int h = blockIdx.x, s = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = (lane * P) / kGroup;
    const int j0 = s * chunk;
    const int j1 = min(L, j0 + chunk);
    const float qscale = rsqrtf((float)D) * kLog2e;
    float qf[P];
#pragma unroll
    for (int i = 0; i < P; ++i) qf[i] = __half2float(q[(size_t)h * D + lane * P + i]) * qscale;

    float m = kNegMax, l = 0.f, o[P];
#pragma unroll
    for (int i = 0; i < P; ++i) o[i] = 0.f;
    for (int j = j0 + warp; j < j1; j += kPlainWarps) {
        const size_t row = (size_t)h * L + j;
        float ks = 1.f, vs = 1.f;
        if constexpr (BITS != 16) {
            ks = __half2float(scK[row * G + g]);
            vs = __half2float(scV[row * G + g]);
        }
        float kv[P], vv[P];
        PlainLane<BITS, P>::load(K, row, lane, kv, ks);
        PlainLane<BITS, P>::load(V, row, lane, vv, vs);
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < P; ++i) acc = fmaf(qf[i], kv[i], acc);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
        const float mn = fmaxf(m, acc);
        const float c = fast_exp2(m - mn), e = fast_exp2(acc - mn);
        l = l * c + e;
        m = mn;
#pragma unroll
        for (int i = 0; i < P; ++i) o[i] = fmaf(o[i], c, e * vv[i]);
    }

    __shared__ float shM[kPlainWarps], shL[kPlainWarps], shO[kPlainWarps][D];
    if (lane == 0) {
        shM[warp] = m;
        shL[warp] = l;
    }
#pragma unroll
    for (int i = 0; i < P; ++i) shO[warp][lane * P + i] = o[i];
    __syncthreads();
    const int t = threadIdx.x;
    if (t < D) {
        float ms = kNegMax;
#pragma unroll
        for (int w = 0; w < kPlainWarps; ++w) ms = fmaxf(ms, shM[w]);
        float ls = 0.f, od = 0.f;
#pragma unroll
        for (int w = 0; w < kPlainWarps; ++w) {
            const float a = fast_exp2(shM[w] - ms);
            ls += shL[w] * a;
            od += shO[w][t] * a;
        }
        float* slot = ws + ((size_t)h * S + s) * (D + 2);
        slot[2 + t] = od;
        if (t == 0) {
            slot[0] = ms * kLn2;
            slot[1] = ls;
        }
    }
}

// Log-sum-exp merge of R*S slots per head (combine, src/voltattn.cu:651-672):
// slots [R][H][S][D+2] with m in natural-log units. mode 0: fp16 out[H][D];
// mode 1: fp32 partial[H][D+2] (merged m, l, o). One 256-thread block per head.
constexpr int kCombineThreads = 256;

__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const float* __restrict__ slots, int R, int H,
                                                                  int S, int D, __half* __restrict__ out,
                                                                  float* __restrict__ partial, int mode) {
    __shared__ float sh_a[kCombineThreads], sh_red[64];
    const int h = blockIdx.x, tid = threadIdx.x;
    auto slot = [&](int i) {
        const int r = i / S, s = i - r * S;
        return slots + (((size_t)r * H + h) * S + s) * (D + 2);
    };
    float ms, ls, od;
    lse_merge(slot, R * S, D, tid, kCombineThreads, LseScratch{sh_a, sh_red}, [] { __syncthreads(); }, ms, ls, od);
    if (tid < D) {
        if (mode == 0) {
            out[(size_t)h * D + tid] = __float2half_rn(od / ls);
        } else {
            float* pp = partial + (size_t)h * (D + 2);
            pp[2 + tid] = od;
            if (tid == 0) {
                pp[0] = ms;
                pp[1] = ls;
            }
        }
    }
}

}  // namespace va
