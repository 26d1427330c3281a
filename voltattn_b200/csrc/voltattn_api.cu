// C ABI of voltattn_b200 (declared in include/voltattn.h): argument checks,
// workspace layout, kernel selection and launch. No CPU compute path: every
// entry point either launches its kernels or returns an error status.

#include <algorithm>
#include <atomic>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/voltattn.h"
#include "common.cuh"
#include "decode_plain.cuh"
#include "decode_mma.cuh"
#include "decode_stream.cuh"
#include "decode_tc.cuh"
#include "decode_tcg.cuh"
#include "exchange.cuh"
#include "prefill_tc.cuh"
#include "launch.cuh"
#include "probe.cuh"
#include "quantize.cuh"

using namespace va;
using namespace va::host;

namespace {

bool is_valid_fmt(int f) { return f >= VA_F16 && f <= VA_Q4CP; }
bool is_f16(int f) { return f == VA_F16 || f == VA_F16P || f == VA_BF16P; }  // 16-bit rows, no scales
bool is_plain(int f) { return f == VA_F16 || f == VA_Q8 || f == VA_Q4; }
int fmt_bits(int f) {
    return is_f16(f) ? 16 : (f == VA_Q8 || f == VA_Q8P || f == VA_F8P) ? 8 : (f == VA_Q3P) ? 3 : 4;  // q4c+: 4
}

size_t slots_bytes(int H, int D, int S) { return (size_t)H * S * (D + 2) * sizeof(float); }
size_t counters_offset(int H, int D, int S) { return (slots_bytes(H, D, S) + 255) & ~(size_t)255; }

size_t gqa_ws_bytes(int B, int Hq, int Hkv, int D, int S) {
    const size_t slots = (size_t)B * Hq * S * (D + 2) * sizeof(float);
    return ((slots + 255) & ~(size_t)255) + (((size_t)(B * Hkv + 2) * sizeof(unsigned) + 255) & ~(size_t)255);
}

template <int BITS>
void launch_plain_bits(const va_bufs* b, float* ws, int H, int L, int D, int S, cudaStream_t st) {
    const int chunk = (L + S - 1) / S;  // the reference's split rule, src/voltattn.cu:804
    const dim3 grid((unsigned)H, (unsigned)S);
    const auto* K = static_cast<const uint8_t*>(b->K);
    const auto* V = static_cast<const uint8_t*>(b->V);
    const auto* sK = static_cast<const __half*>(b->scK);
    const auto* sV = static_cast<const __half*>(b->scV);
    const auto* q = static_cast<const __half*>(b->q);
    if (D == 128)
        decode_plain_kernel<BITS, 128><<<grid, 32 * kPlainWarps, 0, st>>>(K, V, sK, sV, q, ws, L, S, chunk);
    else
        decode_plain_kernel<BITS, 64><<<grid, 32 * kPlainWarps, 0, st>>>(K, V, sK, sV, q, ws, L, S, chunk);
}

int check_decode_args(int fmt, const va_bufs* b, int H, int L, int D, int S) {
    if (!is_valid_fmt(fmt) || !b) return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    if (H < 1 || L < 1 || S < 1 || S > 65535) return VA_ERR_INVALID;
    if ((long long)H * S > INT_MAX / 2) return VA_ERR_INVALID;
    if (!b->K || !b->V || !b->q || !b->out) return VA_ERR_INVALID;
    if (!is_f16(fmt) && (!b->scK || !b->scV)) return VA_ERR_INVALID;
    if (!aligned16(b->K) || !aligned16(b->V)) return VA_ERR_ALIGN;
    if (!is_f16(fmt) && (!aligned16(b->scK) || !aligned16(b->scV))) return VA_ERR_ALIGN;
    if ((reinterpret_cast<uintptr_t>(b->q) & 1u) || (reinterpret_cast<uintptr_t>(b->out) & 1u)) return VA_ERR_ALIGN;
    return VA_OK;
}

DecodeParams make_params(const va_bufs* b, int H, int L, int S, float* ws, unsigned* counters, int mode,
                         float* partial) {
    DecodeParams p;
    p.K = static_cast<const uint8_t*>(b->K);
    p.V = static_cast<const uint8_t*>(b->V);
    p.scK = static_cast<const __half*>(b->scK);
    p.scV = static_cast<const __half*>(b->scV);
    p.q = static_cast<const __half*>(b->q);
    p.out = static_cast<__half*>(b->out);
    p.partial = partial;
    p.ws = ws;
    p.counters = counters;
    p.H = H;
    p.L = L;
    p.S = S;
    const int per = (L + S - 1) / S;
    p.chunk = (per + 7) & ~7;  // whole 8-row blocks per split
    p.total_rows = (long long)H * L;
    p.out_mode = mode;
    p.Hkv = H;
    p.lens = nullptr;
    p.block_table = nullptr;
    p.max_pages = 0;
    p.page_rows = 0;
    p.num_pages = 0;
    p.mq = 1;
    std::memset(&p.x, 0, sizeof(p.x));
    p.xR = 0;
    p.xrank = 0;
    p.xepoch = 0;
    p.xepoch_ptr = nullptr;
    p.xwait_ns = 0;
    return p;
}

int decode_impl(int fmt, const va_bufs* b, int H, int L, int D, int S, void* ws, size_t ws_bytes, float* partial,
                void* stream) {
    int rc = check_decode_args(fmt, b, H, L, D, S);
    if (rc) return rc;
    if (!ws || !aligned16(ws) || ws_bytes < slots_bytes(H, D, S)) return VA_ERR_WORKSPACE;
    const bool fused_ok = ws_bytes >= va_workspace_bytes(H, D, S);
    if (partial && !fused_ok) return VA_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* slots = static_cast<float*>(ws);
    if (fmt == VA_Q4CP) {  // tile kernel only: D = 128, fused workspace, bulk-copied query
        if (D != 128) return VA_ERR_UNSUPPORTED;
        if (!fused_ok) return VA_ERR_WORKSPACE;
        if ((reinterpret_cast<uintptr_t>(b->q) & 15u) != 0) return VA_ERR_ALIGN;
        if ((long long)H * L >= (1ll << 31)) return VA_ERR_TOO_LARGE;
        unsigned* counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + counters_offset(H, D, S));
        const DecodeParams p =
            make_params(b, H, L, S, slots, counters, partial ? kOutPartial : kOutHalf, partial);
        return launch_tc<TcCfg<Kind::Q4, 128, true>>(p, st);
    }
    if (is_plain(fmt) || !fused_ok) {
        if (is_plain(fmt)) {
            if (partial) return VA_ERR_UNSUPPORTED;
            const int bits = fmt_bits(fmt);
            if (bits == 16) launch_plain_bits<16>(b, slots, H, L, D, S, st);
            else if (bits == 8) launch_plain_bits<8>(b, slots, H, L, D, S, st);
            else launch_plain_bits<4>(b, slots, H, L, D, S, st);
            VA_CUDA(cudaGetLastError());
        } else {
            const DecodeParams p = make_params(b, H, L, S, slots, nullptr, kOutSlots, nullptr);
            rc = launch_stream_fmt_g<1>(fmt, p, D, st);
            if (rc) return rc;
        }
        combine_kernel<<<H, kCombineThreads, 0, st>>>(slots, 1, H, S, D, static_cast<__half*>(b->out), nullptr, 0);
        VA_CUDA(cudaGetLastError());
        return VA_OK;
    }
    unsigned* counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + counters_offset(H, D, S));
    const DecodeParams p =
        make_params(b, H, L, S, slots, counters, partial ? kOutPartial : kOutHalf, partial);
    return launch_stream_fmt_g<1>(fmt, p, D, st);
}

// Fixed workspace of va_decode_noalloc (see include/voltattn.h). In host
// code the symbol is only a handle: its device address comes from
// cudaGetSymbolAddress, once per device, with that device current.
constexpr size_t kNoAllocScratchBytes = 4u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

int noalloc_scratch(int dev, void** out) {
    static void* addr[kMaxDevices] = {nullptr};
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void* p = nullptr;
        VA_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        addr[dev] = p;
    }
    *out = addr[dev];
    return VA_OK;
}

}  // namespace

// ---- decode with host-side q / out: one cached CUDA graph per argument set ----
struct HostStepKey {
    int dev, fmt, H, L, D, S;
    va_bufs b;
    const void* q_host;
    void* out_host;
    void* ws;
    size_t ws_bytes;
    cudaStream_t st;
    bool operator==(const HostStepKey& o) const { return std::memcmp(this, &o, sizeof(*this)) == 0; }
};
// The cached executable graph is shared: a launch holds a reference until it
// has synchronised, so evicting the entry meanwhile cannot destroy it.
using GraphExecRef = std::shared_ptr<CUgraphExec_st>;
struct HostStepGraph {
    HostStepKey key;
    GraphExecRef exec;
};
constexpr size_t kHostStepGraphs = 16;  // cached graphs (oldest evicted)
std::mutex g_host_step_mu;
// Wall-clock bound of the split-L peer waits (va_set_peer_wait_limit).
std::atomic<unsigned long long> g_peer_wait_ns{kWaitLimitNs};
std::vector<HostStepGraph> g_host_steps;

extern "C" {

int va_version(void) { return 100; }

const char* va_fmt_name(int fmt) {
    static const char* names[] = {"f16", "f16+", "q8", "q8+", "q4", "q4+", "q3+", "bf16+", "f8+", "q4c+"};
    return is_valid_fmt(fmt) ? names[fmt] : nullptr;
}

int va_fmt_from_name(const char* name) {
    if (!name) return -1;
    for (int f = VA_F16; f <= VA_Q4CP; ++f)
        if (std::strcmp(name, va_fmt_name(f)) == 0) return f;
    return -1;
}

int va_fmt_bits(int fmt) { return is_valid_fmt(fmt) ? fmt_bits(fmt) : -1; }

size_t va_payload_bytes(int fmt, size_t n) {
    if (!is_valid_fmt(fmt)) return 0;
    const int bits = fmt_bits(fmt);
    return bits == 16 ? 2 * n : bits == 8 ? n : bits == 4 ? n / 2 : n * 3 / 8;
}

const char* va_status_string(int status) {
    switch (status) {
        case VA_OK: return "ok";
        case VA_ERR_INVALID: return "invalid argument (format, shape or null pointer)";
        case VA_ERR_ALIGN: return "misaligned pointer (K/V/scales must be 16-byte aligned)";
        case VA_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
        case VA_ERR_CUDA: return "CUDA runtime error (see va_last_cuda_error)";
        case VA_ERR_UNSUPPORTED: return "unsupported configuration (D must be 64 or 128)";
        case VA_ERR_DEVICE: return "a kernel reported a device-side error";
        case VA_ERR_TOO_LARGE: return "size beyond the stated maximum";
        default: return "unknown status";
    }
}

int va_last_cuda_error(void) { return last_cuda_error(); }

size_t va_workspace_bytes(int H, int D, int S) {
    if (H < 1 || S < 1 || D < 1) return 0;
    // per-head tickets plus the two words of the dynamic unit schedule
    return counters_offset(H, D, S) + (((size_t)(H + 2) * sizeof(unsigned) + 255) & ~(size_t)255);
}

int va_workspace_init(void* ws, size_t bytes, void* stream) {
    if (!ws) return VA_ERR_WORKSPACE;
    VA_CUDA(cudaMemsetAsync(ws, 0, bytes, static_cast<cudaStream_t>(stream)));
    return VA_OK;
}

int va_suggest_splits(int fmt, int H, int L, int D, int* S) {
    if (!S || !is_valid_fmt(fmt) || H < 1 || L < 1) return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    const int nsm = sm_count(dev);
    if (is_plain(fmt)) {
        // one CTA per (head, split): aim for ~4 waves of 4-warp blocks
        const int want = std::max(1, (nsm * 16) / H);
        *S = std::max(1, std::min({want, (L + 63) / 64, 65535}));
        return VA_OK;
    }
    int occ = 1;
    int tr;
    double unit_rows;  // fixed cost of a unit in rows of streaming
    const Kind kk = fmt == VA_Q4P ? Kind::Q4 : fmt == VA_Q8P ? Kind::Q8 : Kind::Q3;
    const bool tc = D == 128 && (fmt == VA_Q4P || fmt == VA_Q8P || fmt == VA_Q3P) &&
                    pick_consumer(kk, D, 1) == Consumer::kTc;
    if (fmt == VA_Q4CP) {
        rc = tc_ctas_per_sm<TcCfg<Kind::Q4, 128, true>>(dev, &occ);
        tr = TcCfg<Kind::Q4, 128, true>::kTr;
        unit_rows = 512.0;
    } else if (tc) {
        // tile kernel: per-unit query setup, slot and ticket hand-over
        rc = fmt == VA_Q4P   ? tc_ctas_per_sm<TcCfg<Kind::Q4, 128>>(dev, &occ)
             : fmt == VA_Q8P ? tc_ctas_per_sm<TcCfg<Kind::Q8, 128>>(dev, &occ)
                             : tc_ctas_per_sm<TcCfg<Kind::Q3, 128>>(dev, &occ);
        tr = TcCfg<Kind::Q4, 128>::kTr;  // 256 rows for every format
        unit_rows = 512.0;
    } else {
        rc = stream_cfg_occupancy(fmt, D, dev, &occ);
        tr = stream_cfg_tile_rows(fmt, D);
        unit_rows = 256.0;
    }
    if (rc) return rc;
    const long long cap = (long long)nsm * occ;
    // cost ~ (units per CTA) * (rows per unit + a fixed per-unit overhead:
    // the merge and ticket); keep units at least one 8-row block long
    double best = 1e300;
    int bestS = 1;
    const int smax = std::min(65535, std::max(1, (L + 7) / 8));
    for (int s = 1; s <= smax; ++s) {
        const long long units = (long long)H * s;
        const long long per_cta = (units + cap - 1) / cap;
        const int rows = (((L + s - 1) / s) + 7) & ~7;
        const double cost = (double)per_cta * (rows + unit_rows + 0.5 * tr);
        if (cost < best - 1e-9) {
            best = cost;
            bestS = s;
        }
    }
    *S = bestS;
    return VA_OK;
}

int va_decode(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* ws, size_t ws_bytes, void* stream) {
    return decode_impl(fmt, bufs, H, L, D, S, ws, ws_bytes, nullptr, stream);
}

int va_decode_partial(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* ws, size_t ws_bytes,
                      float* partial, void* stream) {
    if (!partial) return VA_ERR_INVALID;
    if (is_plain(fmt)) return VA_ERR_UNSUPPORTED;
    return decode_impl(fmt, bufs, H, L, D, S, ws, ws_bytes, partial, stream);
}

int va_combine_partials(const float* slots, int R, int H, int S, int D, void* out, void* stream) {
    if (!slots || !out || R < 1 || H < 1 || S < 1 || D < 1 || D > 128) return VA_ERR_INVALID;
    combine_kernel<<<H, kCombineThreads, 0, static_cast<cudaStream_t>(stream)>>>(slots, R, H, S, D,
                                                                      static_cast<__half*>(out), nullptr, 0);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

namespace {
// Bytes of a rank's epoch-tagged gather words [2][R][H][D+2] (peer.cuh),
// rounded to 256.
size_t gather_bytes(int R, int H, int D) {
    return ((size_t)2 * R * H * (D + 2) * sizeof(unsigned long long) + 255) & ~(size_t)255;
}
}  // namespace

int va_set_peer_wait_limit(double seconds) {
    if (!(seconds > 0.0) || seconds > 60.0) return VA_ERR_INVALID;
    g_peer_wait_ns.store((unsigned long long)(seconds * 1e9));
    return VA_OK;
}

size_t va_exchange_buffer_bytes(int R, int H, int D) {
    if (R < 1 || R > kMaxRanks || H < 1 || D < 1) return 0;
    // epoch-tagged gather words, and a 256-byte block whose first word counts
    // this rank's steps (va_decode_splitl with epoch 0)
    return gather_bytes(R, H, D) + 256;
}

int va_exchange_combine(const float* partial, int H, int D, int R, int rank, void* const* peer_buffers,
                        unsigned epoch, void* out, void* stream) {
    if (!partial || !peer_buffers || !out || R < 1 || R > kMaxRanks || rank < 0 || rank >= R || H < 1 || D < 1 ||
        D > 128 || epoch == 0)
        return VA_ERR_INVALID;
    PeerBuffers pb = {};
    for (int r = 0; r < R; ++r) {
        if (!peer_buffers[r] || !aligned16(peer_buffers[r])) return VA_ERR_INVALID;
        pb.gather[r] = static_cast<unsigned long long*>(peer_buffers[r]);
    }
    exchange_combine_kernel<<<H, 128, 0, static_cast<cudaStream_t>(stream)>>>(
        partial, H, D, R, rank, pb, epoch, g_peer_wait_ns.load(), static_cast<__half*>(out));
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int va_decode_splitl(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* ws, size_t ws_bytes, int R,
                     int rank, void* const* peer_buffers, unsigned epoch, void* stream) {
    if (!peer_buffers || R < 1 || R > kMaxRanks || rank < 0 || rank >= R) return VA_ERR_INVALID;
    int rc = check_decode_args(fmt, bufs, H, L, D, S);
    if (rc) return rc;
    const Kind kind = fmt == VA_Q4P ? Kind::Q4 : fmt == VA_Q8P ? Kind::Q8 : Kind::Q3;
    if ((fmt != VA_Q4P && fmt != VA_Q8P && fmt != VA_Q3P) || D != 128 || pick_consumer(kind, D, 1) != Consumer::kTc)
        return VA_ERR_UNSUPPORTED;
    if ((long long)H * L >= (1ll << 31)) return VA_ERR_TOO_LARGE;
    if ((reinterpret_cast<uintptr_t>(bufs->q) & 15u) != 0) return VA_ERR_ALIGN;  // the query is bulk-copied
    if (!ws || !aligned16(ws) || ws_bytes < va_workspace_bytes(H, D, S)) return VA_ERR_WORKSPACE;
    unsigned* counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + counters_offset(H, D, S));
    DecodeParams p = make_params(bufs, H, L, S, static_cast<float*>(ws), counters, kOutHalf, nullptr);
    for (int r = 0; r < R; ++r) {
        if (!peer_buffers[r] || !aligned16(peer_buffers[r])) return VA_ERR_INVALID;
        p.x.gather[r] = static_cast<unsigned long long*>(peer_buffers[r]);
    }
    p.xR = R;
    p.xrank = rank;
    p.xepoch = epoch;
    if (epoch == 0)  // the step count lives in this rank's buffer, after the gather words
        p.xepoch_ptr = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(peer_buffers[rank]) + gather_bytes(R, H, D));
    p.xwait_ns = g_peer_wait_ns.load();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (fmt == VA_Q4P) return launch_tc<TcCfg<Kind::Q4, 128>>(p, st);
    if (fmt == VA_Q8P) return launch_tc<TcCfg<Kind::Q8, 128>>(p, st);
    return launch_tc<TcCfg<Kind::Q3, 128>>(p, st);
}

int va_quantize(int bits, const float* x, void* codes, void* scales, int H, int L, int D, void* stream) {
    if (bits != 8 && bits != 4 && bits != 3) return VA_ERR_INVALID;
    if (!x || !codes || !scales || H < 1 || L < 1) return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    if (!aligned16(x) || !aligned16(codes) || (reinterpret_cast<uintptr_t>(scales) & 1u)) return VA_ERR_ALIGN;
    const long long ngroups = (long long)H * L * (D / kGroup);
    const long long threads = ngroups * 8;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* c = static_cast<uint8_t*>(codes);
    auto* s = static_cast<__half*>(scales);
    if (bits == 8) quantize_kernel<8><<<blocks, 256, 0, st>>>(x, c, s, ngroups);
    else if (bits == 4) quantize_kernel<4><<<blocks, 256, 0, st>>>(x, c, s, ngroups);
    else quantize_kernel<3><<<blocks, 256, 0, st>>>(x, c, s, ngroups);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

namespace {
// Small transfers by loads and stores (16-byte words, grid-stride). Either side
// may be pinned host memory, which unified addressing maps into the device's
// address space: a few KB then cost a kernel instead of a copy-engine transfer.
__global__ void __launch_bounds__(256) copy_small_kernel(uint4* __restrict__ dst, const uint4* __restrict__ src,
                                                         size_t n16) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = src[i];
}
}  // namespace

namespace {
// The address a kernel uses for p: device (or managed) memory as is, pinned
// host memory through its device mapping. Ordinary pageable host memory, which
// a kernel cannot reach, and unknown pointers give VA_ERR_INVALID, so no kernel
// is ever launched on them.
int device_view(const void* p, void** out) {
    cudaPointerAttributes a;
    const cudaError_t e = cudaPointerGetAttributes(&a, p);
    if (e != cudaSuccess) {
        (void)cudaGetLastError();  // the failed query leaves no error behind
        return VA_ERR_INVALID;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
        *out = const_cast<void*>(p);
        return VA_OK;
    }
    if (a.type == cudaMemoryTypeHost && a.devicePointer) {
        *out = a.devicePointer;
        return VA_OK;
    }
    return VA_ERR_INVALID;
}
}  // namespace

int va_copy_small(void* dst, const void* src, size_t bytes, void* stream) {
    if (!dst || !src) return VA_ERR_INVALID;
    if (!aligned16(dst) || !aligned16(src) || (bytes & 15u)) return VA_ERR_ALIGN;
    if (bytes == 0) return VA_OK;
    void *d = nullptr, *s = nullptr;
    int rc = device_view(dst, &d);
    if (!rc) rc = device_view(src, &s);
    if (rc) return rc;
    const size_t n16 = bytes / 16;
    const unsigned blocks = (unsigned)std::min<size_t>((n16 + 255) / 256, 1184);
    copy_small_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint4*>(d),
                                                                            static_cast<const uint4*>(s), n16);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int va_quantize_f8(const float* x, void* codes, void* scales, int H, int L, int D, void* stream) {
    if (!x || !codes || !scales || H < 1 || L < 1) return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(codes) & 7u) || (reinterpret_cast<uintptr_t>(scales) & 1u))
        return VA_ERR_ALIGN;
    const long long ngroups = (long long)H * L * (D / kGroup);
    const unsigned blocks = (unsigned)((ngroups * 8 + 255) / 256);
    quantize_kernel<kBitsF8><<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, static_cast<uint8_t*>(codes), static_cast<__half*>(scales), ngroups);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int va_quantize_kchan(int bits, const float* x, void* codes, void* scales, int H, int L, int D, void* stream) {
    if ((bits != 8 && bits != 4) || !x || !codes || !scales || H < 1 || L < 1) return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(scales) & 1u)) return VA_ERR_ALIGN;
    const dim3 grid((unsigned)(D / 32), (unsigned)H);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* c = static_cast<uint8_t*>(codes);
    auto* sc = static_cast<__half*>(scales);
    if (bits == 8) quantize_kchan_kernel<8><<<grid, 256, 0, st>>>(x, c, sc, L, D);
    else quantize_kchan_kernel<4><<<grid, 256, 0, st>>>(x, c, sc, L, D);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int va_quantize_vtok(int bits, const float* x, void* codes, void* scales, int H, int L, int D, void* stream) {
    if ((bits != 8 && bits != 4) || !x || !codes || !scales || H < 1 || L < 1) return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(scales) & 1u)) return VA_ERR_ALIGN;
    const long long rows = (long long)H * L;
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* c = static_cast<uint8_t*>(codes);
    auto* sc = static_cast<__half*>(scales);
    if (bits == 8) quantize_vtok_kernel<8><<<blocks, 256, 0, st>>>(x, c, sc, rows, D);
    else quantize_vtok_kernel<4><<<blocks, 256, 0, st>>>(x, c, sc, rows, D);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int va_append_kv(int bits, const float* x, void* codes, void* scales, int B, int Hkv, int Lcap, int D,
                 const int* pos, void* stream) {
    if (bits != 16 && bits != 8 && bits != 4 && bits != 3) return VA_ERR_INVALID;
    if (!x || !codes || !pos || (bits != 16 && !scales) || B < 1 || Hkv < 1 || Lcap < 1) return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    if (!aligned16(x) || !aligned16(codes) || (scales && (reinterpret_cast<uintptr_t>(scales) & 1u)))
        return VA_ERR_ALIGN;
    const long long nrows = (long long)B * Hkv;
    const long long threads = nrows * (D / kGroup) * 8;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* c = static_cast<uint8_t*>(codes);
    auto* sc = static_cast<__half*>(scales);
    switch (bits) {
        case 16: append_kernel<16><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, Lcap, D, pos, nrows, PageMap{}); break;
        case 8: append_kernel<8><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, Lcap, D, pos, nrows, PageMap{}); break;
        case 4: append_kernel<4><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, Lcap, D, pos, nrows, PageMap{}); break;
        default: append_kernel<3><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, Lcap, D, pos, nrows, PageMap{}); break;
    }
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int va_probe_ceiling_method(int device, int method, size_t bytes, int reps, double* gbs) {
    if (!gbs || (method != 0 && method != 1)) return VA_ERR_INVALID;
    if (bytes == 0) bytes = 4ull << 30;
    if (reps <= 0) reps = 20;
    bytes &= ~(size_t)(kProbeChunk - 1);
    if (bytes < (size_t)kProbeChunk) return VA_ERR_INVALID;
    int prev = 0;
    VA_CUDA(cudaGetDevice(&prev));
    VA_CUDA(cudaSetDevice(device));
    if (device < 0 || device >= kMaxDevices) return VA_ERR_UNSUPPORTED;
    void* buf = nullptr;
    unsigned* sink = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = VA_OK;
    do {
        cudaError_t e = cudaMalloc(&buf, bytes);
        if (e != cudaSuccess) { rc = cuda_fail(e); break; }
        if ((e = cudaMalloc(&sink, 16)) != cudaSuccess) { rc = cuda_fail(e); break; }
        if ((e = cudaMemset(buf, 0, bytes)) != cudaSuccess) { rc = cuda_fail(e); break; }
        if ((e = cudaMemset(sink, 0, 16)) != cudaSuccess) { rc = cuda_fail(e); break; }
        if ((e = cudaEventCreate(&e0)) != cudaSuccess || (e = cudaEventCreate(&e1)) != cudaSuccess) {
            rc = cuda_fail(e);
            break;
        }
        const int nsm = sm_count(device);
        const int bulk_smem = kProbeStages * kProbeChunk + kProbeStages * 8;
        if (method == 1) {
            e = cudaFuncSetAttribute(probe_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bulk_smem);
            if (e != cudaSuccess) { rc = cuda_fail(e); break; }
        }
        auto run = [&]() {
            if (method == 0)
                probe_vec_kernel<<<nsm * 4, 512>>>(static_cast<const uint4*>(buf), bytes / 16, sink);
            else
                probe_bulk_kernel<<<nsm, 32, bulk_smem>>>(static_cast<const uint8_t*>(buf), bytes / kProbeChunk,
                                                          sink);
        };
        for (int w = 0; w < 3; ++w) run();
        if ((e = cudaDeviceSynchronize()) != cudaSuccess) { rc = cuda_fail(e); break; }
        double best = 0.0;
        for (int r = 0; r < reps; ++r) {
            cudaEventRecord(e0);
            run();
            cudaEventRecord(e1);
            if ((e = cudaEventSynchronize(e1)) != cudaSuccess) { rc = cuda_fail(e); break; }
            float ms = 0.f;
            cudaEventElapsedTime(&ms, e0, e1);
            if (ms > 0.f) best = std::max(best, (double)bytes / (ms * 1e6));
        }
        if (rc) break;
        if ((e = cudaGetLastError()) != cudaSuccess) { rc = cuda_fail(e); break; }
        *gbs = best;
    } while (false);
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (sink) cudaFree(sink);
    if (buf) cudaFree(buf);
    cudaSetDevice(prev);
    return rc;
}

int va_probe_ceiling(int device, size_t bytes, int reps, double* gbs) {
    if (!gbs) return VA_ERR_INVALID;
    double a = 0.0, b = 0.0;
    int rc = va_probe_ceiling_method(device, 0, bytes, reps, &a);
    if (rc) return rc;
    rc = va_probe_ceiling_method(device, 1, bytes, reps, &b);
    if (rc) return rc;
    *gbs = std::max(a, b);
    return VA_OK;
}

size_t va_gqa_workspace_bytes(int B, int Hq, int D, int S) {
    if (B < 1 || Hq < 1 || D < 1 || S < 1) return 0;
    return gqa_ws_bytes(B, Hq, Hq, D, S);  // counters sized for the largest Hkv (= Hq)
}

int va_decode_gqa(int fmt, const va_bufs* b, const int* lens, int B, int Hq, int Hkv, int Lmax, int D, int S,
                  void* ws, size_t ws_bytes, void* stream) {
    if (!is_valid_fmt(fmt) || !b || !lens) return VA_ERR_INVALID;
    if (is_plain(fmt)) return VA_ERR_UNSUPPORTED;
    if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv) return VA_ERR_INVALID;
    const int G = Hq / Hkv;
    if (G != 1 && G != 2 && G != 4 && G != 8) return VA_ERR_UNSUPPORTED;
    const long long streams = (long long)B * Hkv;
    if (streams > INT_MAX / 2) return VA_ERR_INVALID;
    int rc = check_decode_args(fmt, b, (int)streams, Lmax, D, S);
    if (rc) return rc;
    if (!ws || !aligned16(ws) || ws_bytes < gqa_ws_bytes(B, Hq, Hkv, D, S)) return VA_ERR_WORKSPACE;
    const size_t slots = (size_t)B * Hq * S * (D + 2) * sizeof(float);
    unsigned* counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + ((slots + 255) & ~(size_t)255));
    DecodeParams p = make_params(b, (int)streams, Lmax, S, static_cast<float*>(ws), counters, kOutHalf, nullptr);
    p.Hkv = Hkv;
    p.lens = lens;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (fmt == VA_Q4CP) {  // the tile kernel with channel scales per stream ([B*Hkv][D]), one query head each
        if (G != 1 || D != 128) return VA_ERR_UNSUPPORTED;
        if ((reinterpret_cast<uintptr_t>(b->q) & 15u) != 0) return VA_ERR_ALIGN;
        if (p.total_rows >= (1ll << 31)) return VA_ERR_TOO_LARGE;
        return launch_tc<TcCfg<Kind::Q4, 128, true>>(p, st);
    }
    switch (G) {
        case 1: return launch_stream_fmt_g<1>(fmt, p, D, st);
        case 2: return launch_stream_fmt_g<2>(fmt, p, D, st);
        case 4: return launch_stream_fmt_g<4>(fmt, p, D, st);
        default: return launch_stream_fmt_g<8>(fmt, p, D, st);
    }
}

int va_decode_multiquery(int fmt, const va_bufs* b, const int* lens, int B, int Hq, int Hkv, int Q, int Lmax,
                         int D, int S, void* ws, size_t ws_bytes, void* stream) {
    if (!is_valid_fmt(fmt) || !b || !lens) return VA_ERR_INVALID;
    if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv || Q < 1 || Lmax < 1 || S < 1) return VA_ERR_INVALID;
    const int slots = (Hq / Hkv) * Q;  // query slots per KV stream: (query head, token)
    if (fmt != VA_Q4P || D != 128 || (slots != 2 && slots != 4 && slots != 8) ||
        pick_consumer(Kind::Q4, D, slots) != Consumer::kTc)
        return VA_ERR_UNSUPPORTED;
    const long long streams = (long long)B * Hkv;
    if (streams > INT_MAX / 2) return VA_ERR_INVALID;
    int rc = check_decode_args(fmt, b, (int)streams, Lmax, D, S);
    if (rc) return rc;
    if ((reinterpret_cast<uintptr_t>(b->q) & 15u) != 0) return VA_ERR_ALIGN;  // the query is bulk-copied
    if (!ws || !aligned16(ws) || ws_bytes < gqa_ws_bytes(B, Hq * Q, Hkv, D, S)) return VA_ERR_WORKSPACE;
    const size_t slot_bytes = (size_t)B * Hq * Q * S * (D + 2) * sizeof(float);
    unsigned* counters =
        reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + ((slot_bytes + 255) & ~(size_t)255));
    DecodeParams p = make_params(b, (int)streams, Lmax, S, static_cast<float*>(ws), counters, kOutHalf, nullptr);
    p.Hkv = Hkv;
    p.lens = lens;
    p.mq = Q;
    if (p.total_rows >= (1ll << 31)) return VA_ERR_TOO_LARGE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (slots == 2) return launch_tcg<TcgCfg<Kind::Q4, 128, 2>>(p, st);
    if (slots == 4) return launch_tcg<TcgCfg<Kind::Q4, 128, 4>>(p, st);
    return launch_tcg<TcgCfg<Kind::Q4, 128, 8>>(p, st);
}

int va_decode_paged(int fmt, const va_bufs* b, const int* block_table, int max_pages, const int* lens, int B,
                    int Hq, int Hkv, int page_rows, int num_pages, int D, int S, void* ws, size_t ws_bytes,
                    void* stream) {
    if (!is_valid_fmt(fmt) || !b || !block_table || !lens) return VA_ERR_INVALID;
    if (B < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv || max_pages < 1 || page_rows < 1 || num_pages < 1 || S < 1)
        return VA_ERR_INVALID;
    const int G = Hq / Hkv;
    // the tile kernels: q3+ / q4+ / q8+ with one query head per KV head, q4+
    // with 2, 4 or 8; copy boxes of 32 rows stay inside a page
    const Kind kind = fmt == VA_Q8P ? Kind::Q8 : fmt == VA_Q3P ? Kind::Q3 : Kind::Q4;
    const bool tc = D == 128 && page_rows % 32 == 0 &&
                    ((G == 1 && (fmt == VA_Q3P || fmt == VA_Q4P || fmt == VA_Q8P || fmt == VA_Q4CP)) ||
                     ((G == 2 || G == 4 || G == 8) && fmt == VA_Q4P)) &&
                    pick_consumer(kind, D, G) == Consumer::kTc;
    // every other "+" format and shape: the streaming / mma kernels, whose
    // producer copies each run of rows inside a page (whole 8-row blocks)
    const bool streamed = !tc && (D == 64 || D == 128) && page_rows % 8 == 0 && !is_plain(fmt) &&
                          fmt != VA_Q4CP && (G == 1 || G == 2 || G == 4 || G == 8);
    if (!tc && !streamed) return VA_ERR_UNSUPPORTED;
    const long long streams = (long long)B * Hkv;
    const long long rows = (long long)num_pages * Hkv * page_rows;
    const long long lmax = (long long)max_pages * page_rows;
    if (streams * S > INT_MAX / 2 || rows >= (1ll << 31) || lmax > INT_MAX) return VA_ERR_TOO_LARGE;
    int rc = check_decode_args(fmt, b, (int)streams, (int)std::min<long long>(lmax, INT_MAX), D, S);
    if (rc) return rc;
    if ((reinterpret_cast<uintptr_t>(b->q) & 15u) != 0) return VA_ERR_ALIGN;  // the query is bulk-copied
    if (!ws || !aligned16(ws) || ws_bytes < gqa_ws_bytes(B, Hq, Hkv, D, S)) return VA_ERR_WORKSPACE;
    const size_t slots = (size_t)B * Hq * S * (D + 2) * sizeof(float);
    unsigned* counters = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(ws) + ((slots + 255) & ~(size_t)255));
    DecodeParams p = make_params(b, (int)streams, (int)lmax, S, static_cast<float*>(ws), counters, kOutHalf, nullptr);
    p.total_rows = rows;
    p.Hkv = Hkv;
    p.lens = lens;
    p.block_table = block_table;
    p.max_pages = max_pages;
    p.page_rows = page_rows;
    p.num_pages = num_pages;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (streamed) {
        switch (G) {
            case 1: return launch_stream_fmt_g<1>(fmt, p, D, st);
            case 2: return launch_stream_fmt_g<2>(fmt, p, D, st);
            case 4: return launch_stream_fmt_g<4>(fmt, p, D, st);
            default: return launch_stream_fmt_g<8>(fmt, p, D, st);
        }
    }
    if (G == 2) return launch_tcg<TcgCfg<Kind::Q4, 128, 2>>(p, st);
    if (G == 4) return launch_tcg<TcgCfg<Kind::Q4, 128, 4>>(p, st);
    if (G == 8) return launch_tcg<TcgCfg<Kind::Q4, 128, 8>>(p, st);
    if (fmt == VA_Q3P) return launch_tc<TcCfg<Kind::Q3, 128>>(p, st);
    if (fmt == VA_Q4CP) return launch_tc<TcCfg<Kind::Q4, 128, true>>(p, st);  // V row scales paged, K per stream
    return fmt == VA_Q4P ? launch_tc<TcCfg<Kind::Q4, 128>>(p, st) : launch_tc<TcCfg<Kind::Q8, 128>>(p, st);
}

int va_append_kv_paged(int bits, const float* x, void* codes, void* scales, const int* block_table, int max_pages,
                       int B, int Hkv, int page_rows, int num_pages, int D, const int* pos, void* stream) {
    if (bits != 16 && bits != 8 && bits != 4 && bits != 3) return VA_ERR_INVALID;
    if (!x || !codes || !pos || !block_table || (bits != 16 && !scales) || B < 1 || Hkv < 1 || max_pages < 1 ||
        page_rows < 1 || num_pages < 1)
        return VA_ERR_INVALID;
    if (D != 64 && D != 128) return VA_ERR_UNSUPPORTED;
    if (!aligned16(x) || !aligned16(codes) || (scales && (reinterpret_cast<uintptr_t>(scales) & 1u)))
        return VA_ERR_ALIGN;
    const long long nrows = (long long)B * Hkv;
    const long long threads = nrows * (D / kGroup) * 8;
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    auto* c = static_cast<uint8_t*>(codes);
    auto* sc = static_cast<__half*>(scales);
    const PageMap pm{block_table, max_pages, page_rows, num_pages};
    switch (bits) {
        case 16: append_kernel<16><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, 0, D, pos, nrows, pm); break;
        case 8: append_kernel<8><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, 0, D, pos, nrows, pm); break;
        case 4: append_kernel<4><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, 0, D, pos, nrows, pm); break;
        default: append_kernel<3><<<blocks, 256, 0, st>>>(x, c, sc, Hkv, 0, D, pos, nrows, pm); break;
    }
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int va_decode_noalloc(int fmt, const va_bufs* bufs, int H, int L, int D, int S, void* stream) {
    const int rc = check_decode_args(fmt, bufs, H, L, D, S);
    if (rc) return rc;
    const size_t need = va_workspace_bytes(H, D, S);
    if (need > kNoAllocScratchBytes) return VA_ERR_TOO_LARGE;
    int dev;
    int r = current_device(&dev);
    if (r) return r;
    void* ws = nullptr;
    r = noalloc_scratch(dev, &ws);
    if (r) return r;
    // the array keeps the previous call's contents: zero the counters the
    // fused combine expects, in stream order before the decode. This stays
    // unconditional: a previous call with another geometry left slot floats
    // where these counters sit, and one whose kernel stopped early (a bounded
    // wait that gave up) left counters set, which the host cannot see without
    // a synchronising read. The cost is one small memset per call.
    unsigned char* base = static_cast<unsigned char*>(ws);
    VA_CUDA(cudaMemsetAsync(base + counters_offset(H, D, S), 0, need - counters_offset(H, D, S),
                            static_cast<cudaStream_t>(stream)));
    return decode_impl(fmt, bufs, H, L, D, S, ws, need, nullptr, stream);
}

static int prefill_impl(int fmt, const va_bufs* b, int Hq, int Hkv, int L, int Lq, int D, const int* block_table,
                        int page_rows, int num_pages, void* stream, void* ws = nullptr, size_t ws_bytes = 0) {
    if (!is_valid_fmt(fmt) || !b) return VA_ERR_INVALID;
    if (Hq < 1 || Hkv < 1 || Hq % Hkv || Lq < 1 || L < Lq) return VA_ERR_INVALID;
    if (D != 128) return VA_ERR_UNSUPPORTED;
    if (Hq > 65535 || (long long)Hkv * L >= (1ll << 40)) return VA_ERR_TOO_LARGE;
    if (!b->K || !b->V || !b->q || !b->out) return VA_ERR_INVALID;
    if (!is_f16(fmt) && (!b->scK || !b->scV)) return VA_ERR_INVALID;
    if (!aligned16(b->K) || !aligned16(b->V) || !aligned16(b->q) || !aligned16(b->out)) return VA_ERR_ALIGN;
    if (!is_f16(fmt) && ((reinterpret_cast<uintptr_t>(b->scK) & 3u) || (reinterpret_cast<uintptr_t>(b->scV) & 3u)))
        return VA_ERR_ALIGN;
    PrefillParams p;
    p.K = static_cast<const uint8_t*>(b->K);
    p.V = static_cast<const uint8_t*>(b->V);
    p.scK = static_cast<const __half*>(b->scK);
    p.scV = static_cast<const __half*>(b->scV);
    p.q = static_cast<const __half*>(b->q);
    p.out = static_cast<__half*>(b->out);
    p.Hq = Hq;
    p.Hkv = Hkv;
    p.L = L;
    p.Lq = Lq;
    p.block_table = block_table;
    p.page_rows = page_rows;
    p.num_pages = num_pages;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (ws) {  // staged: the cache converted once, tiles by tensor copies
        if (!aligned16(ws) || ws_bytes < prefill_stage_bytes(Hkv, L, D)) return VA_ERR_WORKSPACE;
        if ((long long)Hkv * prefill_stage_rows(L) >= (1ll << 31)) return VA_ERR_TOO_LARGE;
        return launch_prefill_staged_fmt(fmt, p, ws, st);
    }
    return launch_prefill_fmt(fmt, p, st);
}

size_t va_prefill_workspace_bytes(int Hkv, int L, int D) {
    if (Hkv < 1 || L < 1 || D != 128) return 0;
    return prefill_stage_bytes(Hkv, L, D);
}

int va_prefill_ws(int fmt, const va_bufs* b, int Hq, int Hkv, int L, int Lq, int D, void* ws, size_t ws_bytes,
                  void* stream) {
    if (!ws) return VA_ERR_WORKSPACE;
    return prefill_impl(fmt, b, Hq, Hkv, L, Lq, D, nullptr, 0, 0, stream, ws, ws_bytes);
}

int va_prefill_paged_ws(int fmt, const va_bufs* b, const int* block_table, int max_pages, int page_rows,
                        int num_pages, int Hq, int Hkv, int L, int Lq, int D, void* ws, size_t ws_bytes,
                        void* stream) {
    if (!ws) return VA_ERR_WORKSPACE;
    if (!block_table || page_rows < 1 || num_pages < 1 || max_pages < 1) return VA_ERR_INVALID;
    if (fmt == VA_Q4CP) return VA_ERR_UNSUPPORTED;  // its V scales are per sequence row, not paged
    if ((long long)max_pages * page_rows < L) return VA_ERR_INVALID;
    if ((long long)num_pages * Hkv * page_rows >= (1ll << 40)) return VA_ERR_TOO_LARGE;
    return prefill_impl(fmt, b, Hq, Hkv, L, Lq, D, block_table, page_rows, num_pages, stream, ws, ws_bytes);
}

int va_prefill(int fmt, const va_bufs* b, int Hq, int Hkv, int L, int Lq, int D, void* stream) {
    return prefill_impl(fmt, b, Hq, Hkv, L, Lq, D, nullptr, 0, 0, stream);
}

int va_prefill_paged(int fmt, const va_bufs* b, const int* block_table, int max_pages, int page_rows, int num_pages,
                     int Hq, int Hkv, int L, int Lq, int D, void* stream) {
    if (!block_table || page_rows < 1 || num_pages < 1 || max_pages < 1) return VA_ERR_INVALID;
    if (fmt == VA_Q4CP) return VA_ERR_UNSUPPORTED;  // its V scales are per sequence row, not paged
    if ((long long)max_pages * page_rows < L) return VA_ERR_INVALID;
    if ((long long)num_pages * Hkv * page_rows >= (1ll << 40)) return VA_ERR_TOO_LARGE;
    return prefill_impl(fmt, b, Hq, Hkv, L, Lq, D, block_table, page_rows, num_pages, stream);
}

int va_decode_host(int fmt, const va_bufs* bufs, const void* q_host, void* out_host, int H, int L, int D, int S,
                   void* ws, size_t ws_bytes, void* stream) {
    if (!bufs || !q_host || !out_host) return VA_ERR_INVALID;
    if (!aligned16(q_host) || !aligned16(out_host) || !aligned16(bufs->q)) return VA_ERR_ALIGN;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // A created stream replays the graph cached for this argument set; it was
    // built from pointers validated below on the first call with them.
    HostStepKey key;
    std::memset(&key, 0, sizeof(key));
    if (st) {
        int rc = current_device(&key.dev);
        if (rc) return rc;
        key.fmt = fmt;
        key.H = H;
        key.L = L;
        key.D = D;
        key.S = S;
        key.b = *bufs;
        key.q_host = q_host;
        key.out_host = out_host;
        key.ws = ws;
        key.ws_bytes = ws_bytes;
        key.st = st;
        GraphExecRef cached;
        {
            std::lock_guard<std::mutex> lock(g_host_step_mu);
            for (const auto& g : g_host_steps)
                if (g.key == key) cached = g.exec;
        }
        if (cached) {
            VA_CUDA(cudaGraphLaunch(cached.get(), st));
            VA_CUDA(cudaStreamSynchronize(st));
            return VA_OK;
        }
    }
    // Pageable host memory is rejected here, before any launch: a kernel cannot
    // reach it. The decode stores its output straight into out_host (mapped
    // pinned memory takes plain global stores; the synchronize below makes
    // them visible to the host).
    void *q_dev = nullptr, *out_dev = nullptr;
    int rc = device_view(q_host, &q_dev);
    if (!rc) rc = device_view(out_host, &out_dev);
    if (rc) return rc;
    va_bufs b2 = *bufs;
    b2.out = out_dev;
    rc = check_decode_args(fmt, &b2, H, L, D, S);
    if (rc) return rc;
    const size_t bytes = (size_t)H * D * sizeof(__half);
    // q_host is copied into bufs->q by one small kernel (the decode kernels
    // bulk-copy the query from device memory; 288 CTAs loading it from host
    // memory themselves measured 51 against 34 us per step)
    const auto step = [&]() -> int {
        int r = va_copy_small(const_cast<void*>(bufs->q), q_dev, bytes, st);
        if (!r) r = decode_impl(fmt, &b2, H, L, D, S, ws, ws_bytes, nullptr, st);
        return r;
    };
    if (!st) {  // the legacy default stream cannot be captured: direct launches
        rc = step();
        if (rc) return rc;
        VA_CUDA(cudaStreamSynchronize(st));
        return VA_OK;
    }
    cudaGraphExec_t exec = nullptr;
    // first call with these arguments: run directly (also the warm-up of the
    // decode's one-time set-up), then capture the same launches
    rc = step();
    if (rc) return rc;
    VA_CUDA(cudaStreamSynchronize(st));
    cudaGraph_t graph = nullptr;
    VA_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    const int rc_cap = step();
    const cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (rc_cap || e != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return rc_cap ? rc_cap : VA_ERR_CUDA;
    }
    const cudaError_t ei = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ei != cudaSuccess) return VA_ERR_CUDA;
    GraphExecRef ref(exec, [](cudaGraphExec_t x) { cudaGraphExecDestroy(x); });
    std::lock_guard<std::mutex> lock(g_host_step_mu);
    if (g_host_steps.size() >= kHostStepGraphs) g_host_steps.erase(g_host_steps.begin());
    g_host_steps.push_back(HostStepGraph{key, std::move(ref)});
    return VA_OK;
}

int va_device_error(int* code) {
    if (!code) return VA_ERR_INVALID;
    int v = 0;
    VA_CUDA(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
    const int zero = 0;
    VA_CUDA(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
    *code = v;
    return VA_OK;
}

}  // extern "C"
