// Reference shim — TEST INFRASTRUCTURE ONLY (builds oracle/_ref/libvoltattn_ref.so).
//
// Compiles the UNMODIFIED reference translation unit (its path is given on the
// command line as VOLTATTN_REF_SRC by oracle/Makefile; no reference source is
// stored in this repository) with its `main` renamed, and exports plain C
// entry points around the reference's own host functions and kernels:
//   quantize()      src/voltattn.cu:709     dq()        :748
//   reference()     :770                    fill_fast() :960
//   launch()        :803                    probe_ceiling() :935
//   selftest()      :911                    bench()     :967
// Used to generate golden vectors (tests/golden/make_golden.py), to time the
// reference's CPU path (bench.py --impl reference, cpu_baseline) and, on a GPU
// box, to run the reference kernels rebuilt for sm_100a as a speed bar.
// Note: the reference's CUDA_CHECK exits the process on any CUDA error.

#define main voltattn_ref_main
#include VOLTATTN_REF_SRC
#undef main

#include <thread>

namespace {
Fmt fmt_from_int(int f) {
    switch (f) {
        case 0: return Fmt::F16;
        case 1: return Fmt::F16M;
        case 2: return Fmt::Q8;
        case 3: return Fmt::Q8M;
        case 4: return Fmt::Q4;
        case 5: return Fmt::Q4M;
        default: return Fmt::Q3M;
    }
}
}  // namespace

extern "C" {

int ref_group() { return GROUP; }

uint16_t ref_float2half(float f) {
    const __half h = __float2half(f);
    uint16_t b;
    std::memcpy(&b, &h, 2);
    return b;
}

float ref_half2float(uint16_t b) {
    __half h;
    std::memcpy(&h, &b, 2);
    return __half2float(h);
}

void ref_float2half_vec(const float* f, size_t n, uint16_t* out) {
    for (size_t i = 0; i < n; ++i) out[i] = ref_float2half(f[i]);
}

void ref_half2float_vec(const uint16_t* h, size_t n, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = ref_half2float(h[i]);
}

// quantize(): payload bytes to `codes`, fp16 scale bits to `scales`.
void ref_quantize(const float* x, int H, int L, int D, int bits, void* codes, uint16_t* scales) {
    const size_t n = (size_t)H * L * D;
    std::vector<float> xv(x, x + n);
    const Quantized z = quantize(xv, H, L, D, bits);
    std::memcpy(codes, z.data(bits), qbytes(bits, n));
    std::memcpy(scales, z.scale.data(), z.scale.size() * 2);
}

// dq() of every element, narrowed to float as run_case does.
void ref_dequant(const void* codes, const uint16_t* scales, int H, int L, int D, int bits, float* out) {
    const size_t n = (size_t)H * L * D;
    Quantized z;
    const size_t pb = qbytes(bits, n);
    if (bits == 8) { z.q8.resize(n); std::memcpy(z.q8.data(), codes, pb); }
    else if (bits == 4) { z.q4.resize(pb); std::memcpy(z.q4.data(), codes, pb); }
    else { z.q3.resize(pb); std::memcpy(z.q3.data(), codes, pb); }
    z.scale.resize((size_t)H * L * (D / GROUP));
    std::memcpy(z.scale.data(), scales, z.scale.size() * 2);
    for (size_t i = 0; i < n; ++i) out[i] = (float)dq(z, H, L, D, bits, i);
}

void ref_reference(const float* kd, const float* vd, const uint16_t* q, int H, int L, int D, float* out) {
    const size_t n = (size_t)H * L * D;
    std::vector<float> k(kd, kd + n), v(vd, vd + n);
    std::vector<__half> qh((size_t)H * D);
    std::memcpy(qh.data(), q, qh.size() * 2);
    const std::vector<float> r = reference(k, v, qh, H, L, D);
    std::memcpy(out, r.data(), r.size() * 4);
}

// The reference's per-head math, unchanged, with heads spread over `threads`
// host threads (each thread calls reference() on one-head slices).
void ref_reference_mt(const float* kd, const float* vd, const uint16_t* q, int H, int L, int D,
                      float* out, int threads) {
    if (threads < 1) threads = 1;
    if (threads > H) threads = H;
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) {
        pool.emplace_back([=]() {
            const size_t hn = (size_t)L * D;
            for (int h = t; h < H; h += threads) {
                std::vector<float> k(kd + h * hn, kd + (h + 1) * hn), v(vd + h * hn, vd + (h + 1) * hn);
                std::vector<__half> qh(D);
                std::memcpy(qh.data(), q + (size_t)h * D, (size_t)D * 2);
                const std::vector<float> r = reference(k, v, qh, 1, L, D);
                std::memcpy(out + (size_t)h * D, r.data(), (size_t)D * 4);
            }
        });
    }
    for (auto& th : pool) th.join();
}

void ref_fill_fast(float* v, size_t n, uint64_t s) {
    std::vector<float> x(n);
    fill_fast(x, s);
    std::memcpy(v, x.data(), n * 4);
}

// ---- GPU side (needs a device; run on the GPU box only) ----

// launch(): fmt index in reference order f16,f16+,q8,q8+,q4,q4+,q3+.
int ref_launch(int fmt, void* K, void* V, void* scK, void* scV, void* q, void* out, float* ws, int H,
               int L, int D, int S, int sync) {
    DeviceBufs b;
    b.K = K; b.V = V; b.scK = scK; b.scV = scV;
    b.q = (__half*)q; b.out = (__half*)out; b.ws = ws;
    launch(fmt_from_int(fmt), b, H, L, D, S);
    if (sync) {
        if (cudaGetLastError() != cudaSuccess) return 1;
        if (cudaDeviceSynchronize() != cudaSuccess) return 2;
    }
    return 0;
}

// Speed bar: n back-to-back launch() calls of the reference (its decode kernel
// and its combine, on the legacy default stream), rotating over `copies` caches
// (K[i], V[i], scK[i], scV[i]), timed with CUDA events around all of them.
// Returns the average ms per launch() in *ms; 0 on success.
int ref_time_launches(int fmt, void* const* K, void* const* V, void* const* scK, void* const* scV, int copies,
                      void* q, void* out, float* ws, int H, int L, int D, int S, int n, float* ms) {
    cudaEvent_t e0, e1;
    if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) return 1;
    const auto bufs = [&](int i) {
        DeviceBufs b;
        b.K = K[i % copies]; b.V = V[i % copies];
        b.scK = scK ? scK[i % copies] : nullptr; b.scV = scV ? scV[i % copies] : nullptr;
        b.q = (__half*)q; b.out = (__half*)out; b.ws = ws;
        return b;
    };
    for (int i = 0; i < 3; ++i) launch(fmt_from_int(fmt), bufs(i), H, L, D, S);
    if (cudaDeviceSynchronize() != cudaSuccess) return 2;
    cudaEventRecord(e0);
    for (int i = 0; i < n; ++i) launch(fmt_from_int(fmt), bufs(i), H, L, D, S);
    cudaEventRecord(e1);
    if (cudaEventSynchronize(e1) != cudaSuccess) return 3;
    float t = 0.f;
    cudaEventElapsedTime(&t, e0, e1);
    *ms = t / (float)n;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    return cudaGetLastError() == cudaSuccess ? 0 : 4;
}

double ref_probe_ceiling() { return probe_ceiling(); }
int ref_selftest() { return selftest(); }
void ref_bench() { bench(); }

}  // extern "C"
