// voltattn oracle — TEST INFRASTRUCTURE ONLY.
//
// A plain C++ (host, no CUDA) restatement of the reference's CPU path for the
// fused dequant + online-softmax attention decode:
//   * the seeded selftest data generator      (reference src/voltattn.cu:839-846)
//   * the bench data fill `fill_fast`         (src/voltattn.cu:959-965)
//   * the symmetric per-group KV quantizer    (src/voltattn.cu:705-745)
//   * the exact dequantizer `dq`              (src/voltattn.cu:747-767)
//   * the double-precision reference          (src/voltattn.cu:769-794)
//   * the split-L log-sum-exp combine         (src/voltattn.cu:651-672)
//   * a grouped-query / variable-length extension of `reference` (no counterpart
//     in the reference: query head h reads KV head h / group, per sequence).
//   * the f8+ / bf16+ formats (no counterpart in the reference): an e4m3 fp8
//     encoder / decoder written from the format's definition (1 sign, 4
//     exponent bits with bias 7, 3 mantissa bits, no infinities, the all-ones
//     pattern is nan, largest finite 448) with round-to-nearest-even and
//     saturation, the f8 group quantizer, and bf16 round-to-nearest-even.
//
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may load
// this library, and only as the checker. The product (voltattn_b200/) never
// links or calls it; there is no CPU fallback anywhere in the product.
//
// Pinning: tests/test_oracle_golden.py checks every function here against
// golden vectors produced by the reference's own host functions
// (tests/golden/make_golden.py, which loads oracle/_ref/libvoltattn_ref.so built
// from the reference source by oracle/Makefile).
//
// fp16 conversions are this file's own round-to-nearest-even bit manipulation
// (IEEE 754 binary16), checked exhaustively against the reference's host
// conversion in the golden tests.

#include <cmath>
#include <cstdint>
#include <cstring>
#include <algorithm>
#include <random>
#include <thread>
#include <vector>

namespace {

constexpr int kGroup = 64;  // quant group along D (src/voltattn.cu:60)

// ---- IEEE binary16 <-> binary32 -------------------------------------------

float half_bits_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    uint32_t mant = h & 0x3FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {  // subnormal: renormalise
            int e = -1;
            do { mant <<= 1; ++e; } while ((mant & 0x400u) == 0);
            mant &= 0x3FFu;
            bits = sign | (uint32_t)(127 - 15 - e) << 23 | (mant << 13);
        }
    } else if (exp == 0x1F) {
        // inf keeps its sign; every nan becomes the canonical 0x7FFFFFFF, as
        // the reference's host conversion (cuda_fp16 host path) produces.
        bits = mant ? 0x7FFFFFFFu : (sign | 0x7F800000u);
    } else {
        bits = sign | (exp + (127 - 15)) << 23 | (mant << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

uint16_t float_to_half_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) {  // inf or nan
        if (ax == 0x7F800000u) return sign | 0x7C00u;
        return 0x7FFFu;  // canonical nan, whatever the sign and payload
    }
    // Largest float that still rounds below 2^16 is 65519.99...; 65520 -> inf.
    if (ax >= 0x477FF000u) return sign | 0x7C00u;
    if (ax >= 0x38800000u) {  // normal half range (>= 2^-14)
        const uint32_t mant = ax & 0x7FFFFFu;
        const uint32_t exp = (ax >> 23) - (127 - 15);
        uint32_t h = (exp << 10) | (mant >> 13);
        const uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // RNE, may carry into exp
        return sign | (uint16_t)h;
    }
    if (ax < 0x33000000u) return sign;  // below half of the smallest subnormal (2^-25)
    // subnormal half: value = m * 2^-24, m in [0, 1024]
    const uint32_t e = ax >> 23;                     // biased float exponent
    const uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;  // 24-bit significand
    // value = mant * 2^(e-150); in units of 2^-24 that is mant * 2^(e-126), so
    // drop (126 - e) low bits, which is 14..24 on this branch.
    const int drop = 126 - (int)e;
    uint32_t q = mant >> drop;
    const uint32_t rem = mant & ((1u << drop) - 1u);
    const uint32_t halfway = 1u << (drop - 1);
    if (rem > halfway || (rem == halfway && (q & 1u))) ++q;
    return sign | (uint16_t)q;
}

// ---- quantizer (src/voltattn.cu:705-745) -----------------------------------

int limit_for_bits(int bits) { return bits == 8 ? 127 : bits == 4 ? 7 : 3; }

size_t payload_bytes(int bits, size_t n) {  // qbytes, src/voltattn.cu:692
    return bits == 8 ? n : bits == 4 ? n / 2 : n * 3 / 8;
}

// Reads the signed code of element `idx` from a packed payload
// (layout of src/voltattn.cu:736-741 and :751-763).
int code_at(const uint8_t* codes, int bits, size_t idx) {
    if (bits == 8) return (int)(int8_t)codes[idx];
    if (bits == 4) {
        const uint8_t b = codes[idx / 2];
        return (int)((idx % 2 == 0) ? (b & 0xF) : (b >> 4)) - 8;
    }
    const size_t byte0 = (idx / 8) * 3;
    const int bo = (int)(idx % 8) * 3;
    uint32_t w = codes[byte0 + (bo >> 3)];
    if ((bo & 7) + 3 > 8) w |= (uint32_t)codes[byte0 + (bo >> 3) + 1] << 8;
    return (int)((w >> (bo & 7)) & 7) - 4;
}

}  // namespace

extern "C" {

float or_half_to_float(uint16_t h) { return half_bits_to_float(h); }
uint16_t or_float_to_half(float f) { return float_to_half_bits(f); }

void or_half_to_float_vec(const uint16_t* h, size_t n, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = half_bits_to_float(h[i]);
}
void or_float_to_half_vec(const float* f, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = float_to_half_bits(f[i]);
}

size_t or_payload_bytes(int bits, size_t n) { return payload_bytes(bits, n); }

// Selftest data for one case: K then V (n = H*L*D floats each) then q (H*D
// fp16), drawn from std::mt19937(seed) and std::normal_distribution<float>(0,1)
// in that order (src/voltattn.cu:839-846).
void or_gen_case(unsigned seed, int H, int L, int D, float* kx, float* vx, uint16_t* q) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(0.f, 1.f);
    const size_t n = (size_t)H * L * D;
    for (size_t i = 0; i < n; ++i) kx[i] = nd(rng);
    for (size_t i = 0; i < n; ++i) vx[i] = nd(rng);
    for (size_t i = 0; i < (size_t)H * D; ++i) q[i] = float_to_half_bits(nd(rng));
}

// The selftest seed rule (src/voltattn.cu:922).
unsigned or_selftest_seed(int H, int L, int D, int S) {
    return 0xC0FFEEu ^ (unsigned)(H * 131 + L * 7 + D + S);
}

// Bench fill: 64-bit LCG, top bits as a signed fraction in [-1, 1)
// (src/voltattn.cu:959-965).
void or_fill_fast(float* v, size_t n, uint64_t s) {
    for (size_t i = 0; i < n; ++i) {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        v[i] = (float)((int32_t)(s >> 33)) * (1.f / 2147483648.f);
    }
}

// Bench query pattern ((i % 7) - 3) / 4 as fp16 (src/voltattn.cu:985).
void or_bench_query(int H, int D, uint16_t* q) {
    for (size_t i = 0; i < (size_t)H * D; ++i)
        q[i] = float_to_half_bits((float)((int)(i % 7) - 3) * 0.25f);
}

// Symmetric per-group quantizer (src/voltattn.cu:709-745). x is fp32 [H][L][D];
// `codes` receives the packed payload (or_payload_bytes(bits, H*L*D) bytes) and
// `scales` the fp16 bit patterns [H][L][D/64]. Each group's scale is amax/lim
// rounded to fp16; codes are round-half-even(x / stored scale), clamped.
void or_quantize(const float* x, int H, int L, int D, int bits, uint8_t* codes, uint16_t* scales) {
    const int G = D / kGroup;
    const int lim = limit_for_bits(bits);
    const size_t n = (size_t)H * L * D;
    if (bits != 8) std::memset(codes, 0, payload_bytes(bits, n));
    for (size_t rowg = 0; rowg < (size_t)H * L * G; ++rowg) {
        const size_t base = (rowg / G) * D + (rowg % G) * kGroup;
        float amax = 0.f;
        for (int i = 0; i < kGroup; ++i) amax = std::max(amax, std::fabs(x[base + i]));
        const float s = amax > 0.f ? amax / (float)lim : 1.f;
        scales[rowg] = float_to_half_bits(s);
        const float sh = half_bits_to_float(scales[rowg]);
        for (int i = 0; i < kGroup; ++i) {
            // lrint then narrowing to int, exactly as the reference's
            // `(int)std::lrint(x / sh)` behaves on x86-64 / glibc.
            int v = (int)std::lrint(x[base + i] / sh);
            v = std::max(-lim, std::min(lim, v));
            const size_t e = base + i;
            if (bits == 8) {
                codes[e] = (uint8_t)(int8_t)v;
            } else if (bits == 4) {
                const uint8_t nib = (uint8_t)(v + 8);
                uint8_t& b = codes[e / 2];
                b = (e % 2 == 0) ? (uint8_t)((b & 0xF0) | nib) : (uint8_t)((b & 0x0F) | (nib << 4));
            } else {
                const size_t byte0 = (e / 8) * 3;
                const int bo = (int)(e % 8) * 3;
                const uint32_t enc = (uint32_t)(v + 4) << (bo & 7);
                codes[byte0 + (bo >> 3)] |= (uint8_t)enc;
                if ((bo & 7) + 3 > 8) codes[byte0 + (bo >> 3) + 1] |= (uint8_t)(enc >> 8);
            }
        }
    }
}

// q4c+ quantizers (no reference counterpart): the group rule of or_quantize
// with the group = one channel's L values of a head (K, scales [H][D]) or one
// row's D values (V, scales [H][L]); codes packed as q8 / q4. bits = 8 or 4.
static void put_code(uint8_t* codes, int bits, size_t e, int v) {
    if (bits == 8) {
        codes[e] = (uint8_t)(int8_t)v;
    } else {
        const uint8_t nib = (uint8_t)(v + 8);
        uint8_t& b = codes[e / 2];
        b = (e % 2 == 0) ? (uint8_t)((b & 0xF0) | nib) : (uint8_t)((b & 0x0F) | (nib << 4));
    }
}

void or_quantize_kchan(const float* x, int H, int L, int D, int bits, uint8_t* codes, uint16_t* scales) {
    const int lim = limit_for_bits(bits);
    for (int h = 0; h < H; ++h)
        for (int d = 0; d < D; ++d) {
            float amax = 0.f;
            for (int j = 0; j < L; ++j) amax = std::max(amax, std::fabs(x[((size_t)h * L + j) * D + d]));
            const float s = amax > 0.f ? amax / (float)lim : 1.f;
            scales[(size_t)h * D + d] = float_to_half_bits(s);
            const float sh = half_bits_to_float(scales[(size_t)h * D + d]);
            for (int j = 0; j < L; ++j) {
                const size_t e = ((size_t)h * L + j) * D + d;
                int v = (int)std::lrint(x[e] / sh);
                put_code(codes, bits, e, std::max(-lim, std::min(lim, v)));
            }
        }
}

void or_quantize_vtok(const float* x, int H, int L, int D, int bits, uint8_t* codes, uint16_t* scales) {
    const int lim = limit_for_bits(bits);
    for (size_t r = 0; r < (size_t)H * L; ++r) {
        float amax = 0.f;
        for (int d = 0; d < D; ++d) amax = std::max(amax, std::fabs(x[r * D + d]));
        const float s = amax > 0.f ? amax / (float)lim : 1.f;
        scales[r] = float_to_half_bits(s);
        const float sh = half_bits_to_float(scales[r]);
        for (int d = 0; d < D; ++d) {
            int v = (int)std::lrint(x[r * D + d] / sh);
            put_code(codes, bits, r * D + d, std::max(-lim, std::min(lim, v)));
        }
    }
}

// Exact values float(double(scale) * code) of the two layouts.
void or_dequant_kchan(const uint8_t* codes, const uint16_t* scales, int H, int L, int D, int bits, float* out) {
    for (size_t idx = 0; idx < (size_t)H * L * D; ++idx) {
        const size_t h = idx / ((size_t)L * D), d = idx % D;
        out[idx] = (float)((double)half_bits_to_float(scales[h * D + d]) * code_at(codes, bits, idx));
    }
}

void or_dequant_vtok(const uint8_t* codes, const uint16_t* scales, int H, int L, int D, int bits, float* out) {
    for (size_t idx = 0; idx < (size_t)H * L * D; ++idx)
        out[idx] = (float)((double)half_bits_to_float(scales[idx / D]) * code_at(codes, bits, idx));
}

// e4m3: round to nearest even, saturating to +-448; nan -> 0x7F.
static uint8_t e4m3_encode(float x) {
    if (std::isnan(x)) return 0x7F;
    const uint8_t sign = std::signbit(x) ? 0x80 : 0x00;
    const float a = std::fabs(x);
    if (a >= 448.f) return sign | 0x7E;  // the largest finite value (inf included)
    if (a < 0.015625f) {                 // below 2^-6: subnormals, step 2^-9
        // m in [0, 8]; m == 8 is the smallest normal 2^-6 whose code is also 8
        return sign | (uint8_t)std::nearbyint(a * 512.f);
    }
    int e;
    std::frexp(a, &e);  // a = f 2^e, f in [0.5, 1): a's exponent is e - 1
    int E = e - 1 + 7;
    float r = std::nearbyint(std::ldexp(a, -(e - 1)) * 8.f);  // 8..16
    if (r == 16.f) {
        r = 8.f;
        ++E;
    }
    return sign | (uint8_t)((E << 3) | ((int)r - 8));
}

static float e4m3_decode(uint8_t c) {
    const int E = (c >> 3) & 15, M = c & 7;
    if (E == 15 && M == 7) return NAN;
    const float v = E == 0 ? std::ldexp((float)M, -9) : std::ldexp(1.f + (float)M / 8.f, E - 7);
    return (c & 0x80) ? -v : v;
}

// f8+ group quantizer: the rule of or_quantize with lim = 448 and e4m3 codes.
void or_quantize_f8(const float* x, int H, int L, int D, uint8_t* codes, uint16_t* scales) {
    const int G = D / kGroup;
    for (size_t rowg = 0; rowg < (size_t)H * L * G; ++rowg) {
        const size_t base = (rowg / G) * D + (rowg % G) * kGroup;
        float amax = 0.f;
        for (int i = 0; i < kGroup; ++i) amax = std::max(amax, std::fabs(x[base + i]));
        const float s = amax > 0.f ? amax / 448.f : 1.f;
        scales[rowg] = float_to_half_bits(s);
        const float sh = half_bits_to_float(scales[rowg]);
        for (int i = 0; i < kGroup; ++i) codes[base + i] = e4m3_encode(x[base + i] / sh);
    }
}

void or_dequant_f8(const uint8_t* codes, const uint16_t* scales, int H, int L, int D, float* out) {
    const int G = D / kGroup;
    const size_t n = (size_t)H * L * D;
    for (size_t idx = 0; idx < n; ++idx) {
        const size_t rowg = (idx / D) * G + (idx % D) / kGroup;
        out[idx] = (float)((double)half_bits_to_float(scales[rowg]) * (double)e4m3_decode(codes[idx]));
    }
}

void or_e4m3_encode_vec(const float* x, size_t n, uint8_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = e4m3_encode(x[i]);
}

void or_e4m3_decode_vec(const uint8_t* c, size_t n, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = e4m3_decode(c[i]);
}

// bf16 round-to-nearest-even (nan stays a quiet nan): bit patterns and values.
void or_float_to_bf16_vec(const float* x, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) {
        uint32_t u;
        std::memcpy(&u, &x[i], 4);
        if ((u & 0x7FFFFFFFu) > 0x7F800000u) {
            out[i] = (uint16_t)((u >> 16) | 0x40u);
        } else {
            u += 0x7FFFu + ((u >> 16) & 1u);
            out[i] = (uint16_t)(u >> 16);
        }
    }
}

// Exact dequantization of every element: float(double(scale) * code)
// (src/voltattn.cu:747-767 and the float narrowing at :858-859).
void or_dequant(const uint8_t* codes, const uint16_t* scales, int H, int L, int D, int bits, float* out) {
    const int G = D / kGroup;
    const size_t n = (size_t)H * L * D;
    for (size_t idx = 0; idx < n; ++idx) {
        const size_t rowg = (idx / D) * G + (idx % D) / kGroup;
        const double s = (double)half_bits_to_float(scales[rowg]);
        out[idx] = (float)(s * code_at(codes, bits, idx));
    }
}

// fp16 -> fp32 copy of an fp16 cache (the f16 formats' "exact" values,
// src/voltattn.cu:851-853).
void or_round_to_half(const float* x, size_t n, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = half_bits_to_float(float_to_half_bits(x[i]));
}

// Double-precision two-pass softmax attention for heads [h0, h1)
// (src/voltattn.cu:769-794). kd/vd are [H][L][D] floats, q fp16 [H][D].
static void reference_heads(const float* kd, const float* vd, const uint16_t* q, int L, int D,
                            int h0, int h1, float* out) {
    std::vector<double> sc(L), od(D);
    for (int h = h0; h < h1; ++h) {
        double mx = -1e300;
        for (int j = 0; j < L; ++j) {
            double acc = 0.0;
            const float* krow = kd + ((size_t)h * L + j) * D;
            for (int d = 0; d < D; ++d) acc += (double)half_bits_to_float(q[(size_t)h * D + d]) * krow[d];
            sc[j] = acc / std::sqrt((double)D);
            mx = std::max(mx, sc[j]);
        }
        double Z = 0.0;
        std::fill(od.begin(), od.end(), 0.0);
        for (int j = 0; j < L; ++j) {
            const double p = std::exp(sc[j] - mx);
            Z += p;
            const float* vrow = vd + ((size_t)h * L + j) * D;
            for (int d = 0; d < D; ++d) od[d] += p * vrow[d];
        }
        for (int d = 0; d < D; ++d) out[(size_t)h * D + d] = (float)(od[d] / Z);
    }
}

void or_reference(const float* kd, const float* vd, const uint16_t* q, int H, int L, int D, float* out) {
    reference_heads(kd, vd, q, L, D, 0, H, out);
}

// Same math with heads spread over `threads` host threads.
void or_reference_mt(const float* kd, const float* vd, const uint16_t* q, int H, int L, int D,
                     float* out, int threads) {
    if (threads < 1) threads = 1;
    threads = std::min(threads, H);
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        const int h0 = (int)((long)H * t / threads), h1 = (int)((long)H * (t + 1) / threads);
        pool.emplace_back(reference_heads, kd, vd, q, L, D, h0, h1, out);
    }
    for (auto& th : pool) th.join();
}

// Log-sum-exp merge of S partial slots per head, slot = (m, l, o[D]) fp32,
// ws[(h*S + s)*(D+2) + ...]; out fp16 [H][D] (src/voltattn.cu:651-672),
// computed in double.
void or_combine(const float* ws, int H, int S, int D, uint16_t* out) {
    for (int h = 0; h < H; ++h) {
        double mStar = -1e300;
        for (int s = 0; s < S; ++s) mStar = std::max(mStar, (double)ws[(size_t)(h * S + s) * (D + 2)]);
        double lStar = 0.0;
        for (int s = 0; s < S; ++s) {
            const float* slot = ws + (size_t)(h * S + s) * (D + 2);
            lStar += slot[1] * std::exp(slot[0] - mStar);
        }
        for (int d = 0; d < D; ++d) {
            double od = 0.0;
            for (int s = 0; s < S; ++s) {
                const float* slot = ws + (size_t)(h * S + s) * (D + 2);
                od += slot[2 + d] * std::exp(slot[0] - mStar);
            }
            out[(size_t)h * D + d] = float_to_half_bits((float)(od / lStar));
        }
    }
}

// Partial (m, l, o[D]) of one head over positions [j0, j1), in double, in
// the same slot layout as or_combine reads. m is the max scaled score, l the
// sum of exp(score - m), o the exp-weighted sum of V rows. An empty range gives
// (-FLT_MAX, 0, 0) like an empty split of the reference kernels.
void or_partial(const float* kd, const float* vd, const uint16_t* q, int H, int L, int D, int h,
                int j0, int j1, float* slot) {
    (void)H;
    if (j1 <= j0) {
        slot[0] = -3.402823466e38f;
        slot[1] = 0.f;
        for (int d = 0; d < D; ++d) slot[2 + d] = 0.f;
        return;
    }
    std::vector<double> sc(j1 - j0), od(D, 0.0);
    double mx = -1e300;
    for (int j = j0; j < j1; ++j) {
        double acc = 0.0;
        const float* krow = kd + ((size_t)h * L + j) * D;
        for (int d = 0; d < D; ++d) acc += (double)half_bits_to_float(q[(size_t)h * D + d]) * krow[d];
        sc[j - j0] = acc / std::sqrt((double)D);
        mx = std::max(mx, sc[j - j0]);
    }
    double Z = 0.0;
    for (int j = j0; j < j1; ++j) {
        const double p = std::exp(sc[j - j0] - mx);
        Z += p;
        const float* vrow = vd + ((size_t)h * L + j) * D;
        for (int d = 0; d < D; ++d) od[d] += p * vrow[d];
    }
    slot[0] = (float)mx;
    slot[1] = (float)Z;
    for (int d = 0; d < D; ++d) slot[2 + d] = (float)od[d];
}

// Grouped-query, variable-length decode reference (extension; the reference
// is batch 1 with one KV head per query head). Sequence b has lens[b]
// positions; its KV heads live at kv + (b*Hkv + g) * Lmax * D (row-major
// [B][Hkv][Lmax][D], rows >= lens[b] ignored); query head hq of sequence b
// (q at [B][Hq][D]) reads KV head hq / (Hq/Hkv). out fp32 [B][Hq][D].
void or_reference_gqa(const float* kd, const float* vd, const uint16_t* q, const int* lens, int B,
                      int Hq, int Hkv, int Lmax, int D, float* out) {
    const int group = Hq / Hkv;
    for (int b = 0; b < B; ++b) {
        for (int hq = 0; hq < Hq; ++hq) {
            const int g = hq / group;
            const size_t kvoff = ((size_t)b * Hkv + g) * Lmax * D;
            reference_heads(kd + kvoff, vd + kvoff, q + ((size_t)b * Hq + hq) * D, lens[b], D, 0, 1,
                            out + ((size_t)b * Hq + hq) * D);
        }
    }
}

}  // extern "C"
