// voltattn — command-line harness over the C ABI, same contract as the
// reference binary (src/voltattn.cu:1072-1086):
//   voltattn            selftest (42 cases), exit code 0 / 1
//   voltattn --bench    selftest, then the benchmark table
//   voltattn --probe    one line: the measured HBM read ceiling
// Extra options: --L <n> (bench length, repeatable), --fmt <name> (bench
// format, repeatable), --json (bench rows as JSON lines).
//
// The selftest follows run_case()/selftest() (src/voltattn.cu:837-931): the
// same shapes, seeds and std::mt19937 + std::normal_distribution<float> data
// order, the same pass gate (|g - r| <= 3e-3 + 2e-2 |r|). Differences: K/V are
// packed by the GPU quantizer (va_quantize), and the checker is an fp64 GPU
// kernel in this file that evaluates softmax attention over the exactly
// dequantized cache (scale * code in double), so this binary needs no CPU
// attention code.

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "../../../include/voltattn.h"

namespace {

#define CK(call)                                                                                   \
    do {                                                                                           \
        cudaError_t e__ = (call);                                                                  \
        if (e__ != cudaSuccess) {                                                                  \
            std::fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e__), __FILE__, __LINE__); \
            std::exit(1);                                                                          \
        }                                                                                          \
    } while (0)

#define VA(call)                                                                                   \
    do {                                                                                           \
        int s__ = (call);                                                                          \
        if (s__ != VA_OK) {                                                                        \
            std::fprintf(stderr, "voltattn error %s at %s:%d\n", va_status_string(s__), __FILE__, __LINE__); \
            std::exit(1);                                                                          \
        }                                                                                          \
    } while (0)

// ---- fp64 checker ------------------------------------------------------------

__device__ double dq_elem(const uint8_t* codes, const __half* scales, int bits, size_t idx, int D) {
    if (bits == 16) return (double)__half2float(reinterpret_cast<const __half*>(codes)[idx]);
    const size_t rowg = (idx / D) * (D / 64) + (idx % D) / 64;
    const double s = (double)__half2float(scales[rowg]);
    int v;
    if (bits == 8) {
        v = (int)(int8_t)codes[idx];
    } else if (bits == 4) {
        const uint8_t b = codes[idx / 2];
        v = (int)((idx & 1) ? (b >> 4) : (b & 0xF)) - 8;
    } else {
        const size_t byte0 = (idx / 8) * 3;
        const int bo = (int)(idx % 8) * 3;
        uint32_t w = codes[byte0 + (bo >> 3)];
        if ((bo & 7) + 3 > 8) w |= (uint32_t)codes[byte0 + (bo >> 3) + 1] << 8;
        v = (int)((w >> (bo & 7)) & 7) - 4;
    }
    return s * v;
}

__global__ void check_scores(const uint8_t* K, const __half* sK, const __half* q, int bits, int H, int L, int D,
                             double* sc) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long long)H * L) return;
    const int h = (int)(i / L);
    double acc = 0.0;
    for (int d = 0; d < D; ++d) acc += (double)__half2float(q[(size_t)h * D + d]) * dq_elem(K, sK, bits, (size_t)i * D + d, D);
    sc[i] = acc / sqrt((double)D);
}

__global__ void check_output(const uint8_t* V, const __half* sV, const double* sc, int bits, int L, int D,
                             float* out) {
    const int h = blockIdx.x, d = threadIdx.x;
    __shared__ double red[128];
    double mx = -1e300;
    for (int j = threadIdx.x; j < L; j += blockDim.x) mx = fmax(mx, sc[(size_t)h * L + j]);
    red[threadIdx.x] = mx;
    __syncthreads();
    for (int s = 64; s > 0; s >>= 1) {
        if (threadIdx.x < s) red[threadIdx.x] = fmax(red[threadIdx.x], red[threadIdx.x + s]);
        __syncthreads();
    }
    mx = red[0];
    if (d >= D) return;
    double Z = 0.0, od = 0.0;
    for (int j = 0; j < L; ++j) {
        const double p = exp(sc[(size_t)h * L + j] - mx);
        Z += p;
        od += p * dq_elem(V, sV, bits, ((size_t)h * L + j) * D + d, D);
    }
    out[(size_t)h * D + d] = (float)(od / Z);
}

int fmt_bits(int f) { return va_fmt_bits(f); }

// ---- selftest (src/voltattn.cu:837-931) ------------------------------------------

bool run_case(int fmt, int H, int L, int D, int S, unsigned seed, double* maxerr) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(0.f, 1.f);
    const size_t n = (size_t)H * L * D;
    std::vector<float> kx(n), vx(n);
    for (auto& v : kx) v = nd(rng);
    for (auto& v : vx) v = nd(rng);
    std::vector<__half> q((size_t)H * D);
    for (auto& v : q) v = __float2half(nd(rng));

    const int bits = fmt_bits(fmt);
    const size_t pb = va_payload_bytes(fmt, n);
    const size_t sb = (size_t)H * L * (D / 64) * 2;
    uint8_t *K, *V, *sK = nullptr, *sV = nullptr;
    __half *qd, *out;
    float *ref, *xk, *xv;
    double* sc;
    CK(cudaMalloc(&K, pb));
    CK(cudaMalloc(&V, pb));
    CK(cudaMalloc(&qd, (size_t)H * D * 2));
    CK(cudaMalloc(&out, (size_t)H * D * 2));
    CK(cudaMalloc(&ref, (size_t)H * D * 4));
    CK(cudaMalloc(&sc, (size_t)H * L * 8));
    CK(cudaMemcpy(qd, q.data(), (size_t)H * D * 2, cudaMemcpyHostToDevice));
    if (bits == 16) {
        std::vector<__half> kh(n), vh(n);
        for (size_t i = 0; i < n; ++i) kh[i] = __float2half(kx[i]);
        for (size_t i = 0; i < n; ++i) vh[i] = __float2half(vx[i]);
        CK(cudaMemcpy(K, kh.data(), pb, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(V, vh.data(), pb, cudaMemcpyHostToDevice));
    } else {
        CK(cudaMalloc(&sK, sb));
        CK(cudaMalloc(&sV, sb));
        CK(cudaMalloc(&xk, n * 4));
        CK(cudaMalloc(&xv, n * 4));
        CK(cudaMemcpy(xk, kx.data(), n * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(xv, vx.data(), n * 4, cudaMemcpyHostToDevice));
        VA(va_quantize(bits, xk, K, sK, H, L, D, nullptr));
        VA(va_quantize(bits, xv, V, sV, H, L, D, nullptr));
        CK(cudaFree(xk));
        CK(cudaFree(xv));
    }
    const size_t wsb = va_workspace_bytes(H, D, S);
    void* ws;
    CK(cudaMalloc(&ws, wsb));
    VA(va_workspace_init(ws, wsb, nullptr));
    const va_bufs b{K, V, sK, sV, qd, out};
    VA(va_decode(fmt, &b, H, L, D, S, ws, wsb, nullptr));
    const long long rows = (long long)H * L;
    check_scores<<<(unsigned)((rows + 127) / 128), 128>>>(K, (const __half*)sK, qd, bits, H, L, D, sc);
    check_output<<<H, 128>>>(V, (const __half*)sV, sc, bits, L, D, ref);
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    std::vector<__half> got((size_t)H * D);
    std::vector<float> r((size_t)H * D);
    CK(cudaMemcpy(got.data(), out, got.size() * 2, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(r.data(), ref, r.size() * 4, cudaMemcpyDeviceToHost));
    double me = 0.0;
    bool ok = true;
    for (size_t i = 0; i < got.size(); ++i) {
        const double g = (double)__half2float(got[i]), rr = (double)r[i];
        const double err = std::fabs(g - rr);
        me = std::max(me, err);
        if (!(err <= 3e-3 + 2e-2 * std::fabs(rr))) ok = false;
    }
    *maxerr = me;
    for (void* p : {(void*)K, (void*)V, (void*)sK, (void*)sV, (void*)qd, (void*)out, (void*)ref, (void*)sc, ws})
        if (p) CK(cudaFree(p));
    int derr = 0;
    VA(va_device_error(&derr));
    return ok && derr == 0;
}

int selftest() {
    struct Case { int H, L, D, S; };
    const Case cases[] = {{8, 257, 128, 1}, {8, 257, 128, 3}, {2, 4096, 128, 5},
                          {40, 1000, 128, 2}, {8, 129, 64, 1}, {8, 513, 64, 4}};
    int fails = 0;
    for (int f = VA_F16; f <= VA_Q3P; ++f) {
        for (const Case& c : cases) {
            double me = 0.0;
            const bool ok = run_case(f, c.H, c.L, c.D, c.S,
                                     0xC0FFEEu ^ (unsigned)(c.H * 131 + c.L * 7 + c.D + c.S), &me);
            std::printf("%-4s  H=%-3d L=%-5d D=%-3d S=%-2d  maxerr=%.2e  %s\n", va_fmt_name(f), c.H, c.L, c.D, c.S,
                        me, ok ? "PASS" : "FAIL");
            if (!ok) ++fails;
        }
    }
    if (fails) {
        std::printf("%d case(s) FAILED\n", fails);
        return 1;
    }
    std::printf("all cases passed\n");
    return 0;
}

// ---- bench (src/voltattn.cu:959-1070) ----------------------------------------------

void fill_fast(std::vector<float>& v, uint64_t s) {  // the reference's LCG fill, :960-965
    for (auto& x : v) {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        x = (float)((int32_t)(s >> 33)) * (1.f / 2147483648.f);
    }
}

void bench(const std::vector<int>& Ls, const std::vector<int>& fmts, bool json) {
    cudaDeviceProp prop{};
    CK(cudaGetDeviceProperties(&prop, 0));
    double ceil_gbs = 0.0;
    VA(va_probe_ceiling(0, 0, 0, &ceil_gbs));
    if (!json) {
        std::printf("device: %s (sm_%d%d, %d SMs, L2 %d MB)\n", prop.name, prop.major, prop.minor,
                    prop.multiProcessorCount, prop.l2CacheSize >> 20);
        std::printf("measured read ceiling: %.1f GB/s\n\n", ceil_gbs);
        std::printf("| fmt  | L      | KV bytes | S   | best ms | avg ms  | GB/s   | MBU   | tok/s  | vs f16 | vs f16+ |\n");
        std::printf("|------|--------|----------|-----|---------|---------|--------|-------|--------|--------|---------|\n");
    }
    const int H = 32, D = 128;
    for (const int L : Ls) {
        const size_t n = (size_t)H * L * D;
        std::vector<float> kx(n), vx(n);
        fill_fast(kx, 0x1234u + (unsigned)L);
        fill_fast(vx, 0x5678u + (unsigned)L);
        std::vector<__half> q((size_t)H * D);
        for (size_t i = 0; i < q.size(); ++i) q[i] = __float2half((float)((int)(i % 7) - 3) * 0.25f);
        float *xk, *xv;
        CK(cudaMalloc(&xk, n * 4));
        CK(cudaMalloc(&xv, n * 4));
        CK(cudaMemcpy(xk, kx.data(), n * 4, cudaMemcpyHostToDevice));
        CK(cudaMemcpy(xv, vx.data(), n * 4, cudaMemcpyHostToDevice));
        double f16_ms = 0.0, f16p_ms = 0.0;
        for (const int f : fmts) {
            const int bits = fmt_bits(f);
            const size_t pb = va_payload_bytes(f, n), sb = bits == 16 ? 0 : (size_t)H * L * (D / 64) * 2;
            const size_t copy_bytes = 2 * (pb + sb);
            const size_t want = 4ull * (size_t)prop.l2CacheSize;
            const int copies = (int)std::min<size_t>(64, std::max<size_t>(2, (want + copy_bytes - 1) / copy_bytes));
            std::vector<va_bufs> bufs(copies);
            __half *qd, *out;
            CK(cudaMalloc(&qd, (size_t)H * D * 2));
            CK(cudaMalloc(&out, (size_t)H * D * 2));
            CK(cudaMemcpy(qd, q.data(), (size_t)H * D * 2, cudaMemcpyHostToDevice));
            std::vector<void*> owned;
            for (int r = 0; r < copies; ++r) {
                void *K, *V, *sK = nullptr, *sV = nullptr;
                CK(cudaMalloc(&K, pb));
                CK(cudaMalloc(&V, pb));
                owned.push_back(K);
                owned.push_back(V);
                if (bits == 16) {
                    std::vector<__half> kh(n), vh(n);
                    if (r == 0) {
                        for (size_t i = 0; i < n; ++i) kh[i] = __float2half(kx[i]);
                        for (size_t i = 0; i < n; ++i) vh[i] = __float2half(vx[i]);
                        CK(cudaMemcpy(K, kh.data(), pb, cudaMemcpyHostToDevice));
                        CK(cudaMemcpy(V, vh.data(), pb, cudaMemcpyHostToDevice));
                    } else {
                        CK(cudaMemcpy(K, bufs[0].K, pb, cudaMemcpyDeviceToDevice));
                        CK(cudaMemcpy(V, bufs[0].V, pb, cudaMemcpyDeviceToDevice));
                    }
                } else {
                    CK(cudaMalloc(&sK, sb));
                    CK(cudaMalloc(&sV, sb));
                    owned.push_back(sK);
                    owned.push_back(sV);
                    VA(va_quantize(bits, xk, K, sK, H, L, D, nullptr));
                    VA(va_quantize(bits, xv, V, sV, H, L, D, nullptr));
                }
                bufs[r] = va_bufs{K, V, sK, sV, qd, out};
            }
            int S = 1;
            VA(va_suggest_splits(f, H, L, D, &S));
            const size_t wsb = va_workspace_bytes(H, D, S);
            void* ws;
            CK(cudaMalloc(&ws, wsb));
            VA(va_workspace_init(ws, wsb, nullptr));
            cudaStream_t st;
            CK(cudaStreamCreate(&st));
            for (int w = 0; w < 3; ++w) VA(va_decode(f, &bufs[w % copies], H, L, D, S, ws, wsb, st));
            CK(cudaStreamSynchronize(st));
            cudaEvent_t e0, e1;
            CK(cudaEventCreate(&e0));
            CK(cudaEventCreate(&e1));
            double best_ms = 1e30;
            for (int rep = 0; rep < 20; ++rep) {  // single launches, best of 20 (as the reference)
                CK(cudaEventRecord(e0, st));
                VA(va_decode(f, &bufs[rep % copies], H, L, D, S, ws, wsb, st));
                CK(cudaEventRecord(e1, st));
                CK(cudaEventSynchronize(e1));
                float ms = 0.f;
                CK(cudaEventElapsedTime(&ms, e0, e1));
                best_ms = std::min(best_ms, (double)ms);
            }
            // back-to-back launches captured in a CUDA graph: the steady-state average
            const int per = copies * std::max(1, 64 / copies);
            cudaGraph_t g;
            cudaGraphExec_t ge;
            CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
            for (int i = 0; i < per; ++i) VA(va_decode(f, &bufs[i % copies], H, L, D, S, ws, wsb, st));
            CK(cudaStreamEndCapture(st, &g));
            CK(cudaGraphInstantiate(&ge, g, 0));
            CK(cudaGraphLaunch(ge, st));
            CK(cudaStreamSynchronize(st));
            const int reps = 10;
            CK(cudaEventRecord(e0, st));
            for (int r = 0; r < reps; ++r) CK(cudaGraphLaunch(ge, st));
            CK(cudaEventRecord(e1, st));
            CK(cudaEventSynchronize(e1));
            float tot = 0.f;
            CK(cudaEventElapsedTime(&tot, e0, e1));
            const double avg_ms = tot / (reps * per);
            const double gbs = (double)copy_bytes / (avg_ms * 1e6);
            if (f == VA_F16) f16_ms = avg_ms;
            if (f == VA_F16P) f16p_ms = avg_ms;
            if (json) {
                std::printf("{\"fmt\": \"%s\", \"L\": %d, \"bytes\": %zu, \"splits\": %d, \"best_ms\": %.5f, "
                            "\"avg_ms\": %.5f, \"gbs\": %.1f, \"mbu\": %.4f, \"tok_s\": %.1f}\n",
                            va_fmt_name(f), L, copy_bytes, S, best_ms, avg_ms, gbs, gbs / ceil_gbs, 1e3 / avg_ms);
            } else {
                std::printf("| %-4s | %-6d | %7.1fMB | %-3d | %7.4f | %7.4f | %6.1f | %4.1f%% | %6.0f | %5.2fx | %6.2fx |\n",
                            va_fmt_name(f), L, copy_bytes / 1e6, S, best_ms, avg_ms, gbs, 100.0 * gbs / ceil_gbs,
                            1e3 / avg_ms, f16_ms > 0 ? f16_ms / avg_ms : 0.0, f16p_ms > 0 ? f16p_ms / avg_ms : 0.0);
            }
            std::fflush(stdout);
            CK(cudaGraphExecDestroy(ge));
            CK(cudaGraphDestroy(g));
            CK(cudaEventDestroy(e0));
            CK(cudaEventDestroy(e1));
            CK(cudaStreamDestroy(st));
            for (void* p : owned) CK(cudaFree(p));
            CK(cudaFree(ws));
            CK(cudaFree(qd));
            CK(cudaFree(out));
        }
        CK(cudaFree(xk));
        CK(cudaFree(xv));
    }
    if (!json) {
        std::printf("\nbytes = compressed K+V payload + fp16 group scales; q/out/workspace excluded.\n");
        std::printf("avg ms: CUDA graph of back-to-back decodes over rotating copies (> 4x L2);\n");
        std::printf("best ms: best single launch of 20, as the reference reports.\n");
    }
}

}  // namespace

int main(int argc, char** argv) {
    std::vector<int> Ls, fmts;
    bool do_bench = false, do_probe = false, json = false;
    for (int i = 1; i < argc; ++i) {
        const std::string a = argv[i];
        if (a == "--bench") do_bench = true;
        else if (a == "--probe") do_probe = true;
        else if (a == "--json") json = true;
        else if (a == "--L" && i + 1 < argc) Ls.push_back(std::atoi(argv[++i]));
        else if (a == "--fmt" && i + 1 < argc) {
            const int f = va_fmt_from_name(argv[++i]);
            if (f < 0) {
                std::fprintf(stderr, "unknown format %s\n", argv[i]);
                return 2;
            }
            fmts.push_back(f);
        } else {
            std::fprintf(stderr, "usage: voltattn [--bench [--L n]... [--fmt f]... [--json]] | --probe\n");
            return 2;
        }
    }
    if (do_probe) {
        double g = 0.0;
        VA(va_probe_ceiling(0, 0, 0, &g));
        std::printf("measured read ceiling: %.1f GB/s\n", g);
        return 0;
    }
    if (do_bench) {
        const int rc = selftest();
        if (rc) return rc;
        std::printf("\n");
        if (Ls.empty()) Ls = {4096, 16384, 65536};
        if (fmts.empty()) fmts = {VA_F16, VA_F16P, VA_Q8, VA_Q8P, VA_Q4, VA_Q4P, VA_Q3P};
        bench(Ls, fmts, json);
        return 0;
    }
    return selftest();
}
