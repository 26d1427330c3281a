// Launchers of the tcgen05 prefill kernel (prefill_tc.cuh).
#include <algorithm>
#include <mutex>

#include "launch.cuh"
#include "prefill_pp.cuh"
#include "prefill_tc.cuh"

namespace va {
#ifdef PF_TIMELINE
__device__ unsigned long long g_pf_tl[4096 * 8];
#endif
namespace host {

template <class C>
static int launch_prefill(const PrefillParams& p, cudaStream_t st) {
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    static bool attr_set[kMaxDevices] = {false};
    static std::mutex mu;
    if (!attr_set[dev]) {
        std::lock_guard<std::mutex> lock(mu);
        if (!attr_set[dev]) {
            VA_CUDA(cudaFuncSetAttribute(prefill_tc_kernel<C, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            VA_CUDA(cudaFuncSetAttribute(prefill_tc_kernel<C, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            attr_set[dev] = true;
        }
    }
    const dim3 grid((unsigned)((p.Lq + C::kBq - 1) / C::kBq), (unsigned)p.Hq);
    if (p.page_rows > 0)
        prefill_tc_kernel<C, true><<<grid, C::kThreads, C::kSmemBytes, st>>>(p);
    else
        prefill_tc_kernel<C, false><<<grid, C::kThreads, C::kSmemBytes, st>>>(p);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int prefill_stage_rows(int L) { return (L + 127) / 128 * 128; }

size_t prefill_stage_bytes(int Hkv, int L, int D) {
    return (size_t)2 * Hkv * prefill_stage_rows(L) * D * sizeof(__half);
}

template <class C>
static int launch_prefill_staged(const PrefillParams& p, void* ws, cudaStream_t st) {
    int dev;
    int rc = current_device(&dev);
    if (rc) return rc;
    static bool attr_set[kMaxDevices] = {false};
    static std::mutex mu;
    if (!attr_set[dev]) {
        std::lock_guard<std::mutex> lock(mu);
        if (!attr_set[dev]) {
            VA_CUDA(cudaFuncSetAttribute(prefill_pp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PpCfg::kSmemBytes));
            attr_set[dev] = true;
        }
    }
    const int Lpad = prefill_stage_rows(p.L);
    __half* stK = static_cast<__half*>(ws);
    __half* stV = stK + (size_t)p.Hkv * Lpad * C::kD;
    const long long chunks = (long long)p.Hkv * Lpad * 16;
    const unsigned blocks = (unsigned)std::min<long long>((chunks + 255) / 256, (long long)sm_count(dev) * 8);
    const dim3 sgrid(blocks, 2);
    if (p.page_rows > 0)
        prefill_stage_kernel<C, true><<<sgrid, 256, 0, st>>>(p, stK, stV, Lpad);
    else
        prefill_stage_kernel<C, false><<<sgrid, 256, 0, st>>>(p, stK, stV, Lpad);
    VA_CUDA(cudaGetLastError());
    CUtensorMap tmK, tmV;
    rc = encode_f16_rows_map(&tmK, stK, (long long)p.Hkv * Lpad, C::kBk);
    if (rc) return rc;
    rc = encode_f16_rows_map(&tmV, stV, (long long)p.Hkv * Lpad, C::kBk);
    if (rc) return rc;
    // pairs of 128-token tiles, one CTA per SM
    const dim3 grid((unsigned)((p.Lq + 2 * PpCfg::kBq - 1) / (2 * PpCfg::kBq)), (unsigned)p.Hq);
    prefill_pp_kernel<<<grid, PpCfg::kThreads, PpCfg::kSmemBytes, st>>>(p, tmK, tmV, Lpad);
    VA_CUDA(cudaGetLastError());
    return VA_OK;
}

int launch_prefill_staged_fmt(int fmt, const PrefillParams& p, void* ws, cudaStream_t st) {
    switch (fmt) {
        case VA_BF16P: return launch_prefill_staged<PrefillCfg<Kind::BF16>>(p, ws, st);
        case VA_Q4CP: return launch_prefill_staged<PrefillCfg<Kind::Q4, true>>(p, ws, st);
        case VA_F8P: return launch_prefill_staged<PrefillCfg<Kind::F8>>(p, ws, st);
        case VA_F16:
        case VA_F16P: return launch_prefill_staged<PrefillCfg<Kind::F16>>(p, ws, st);
        case VA_Q8:
        case VA_Q8P: return launch_prefill_staged<PrefillCfg<Kind::Q8>>(p, ws, st);
        case VA_Q4:
        case VA_Q4P: return launch_prefill_staged<PrefillCfg<Kind::Q4>>(p, ws, st);
        case VA_Q3P: return launch_prefill_staged<PrefillCfg<Kind::Q3>>(p, ws, st);
        default: return VA_ERR_INVALID;
    }
}

int launch_prefill_fmt(int fmt, const PrefillParams& p, cudaStream_t st) {
    switch (fmt) {
        case VA_BF16P: return launch_prefill<PrefillCfg<Kind::BF16>>(p, st);
        case VA_Q4CP: return launch_prefill<PrefillCfg<Kind::Q4, true>>(p, st);
        case VA_F8P: return launch_prefill<PrefillCfg<Kind::F8>>(p, st);
        case VA_F16:
        case VA_F16P: return launch_prefill<PrefillCfg<Kind::F16>>(p, st);
        case VA_Q8:
        case VA_Q8P: return launch_prefill<PrefillCfg<Kind::Q8>>(p, st);
        case VA_Q4:
        case VA_Q4P: return launch_prefill<PrefillCfg<Kind::Q4>>(p, st);
        case VA_Q3P: return launch_prefill<PrefillCfg<Kind::Q3>>(p, st);
        default: return VA_ERR_INVALID;
    }
}

}  // namespace host
}  // namespace va

#ifdef PF_TIMELINE
// Development builds only: per-CTA cycle totals of the staged prefill's phases.
extern "C" int va_debug_pf_timeline(void* dst, size_t bytes) {
    if (!dst || bytes < sizeof(va::g_pf_tl)) return VA_ERR_INVALID;
    VA_CUDA(cudaMemcpyFromSymbol(dst, va::g_pf_tl, sizeof(va::g_pf_tl)));
    return VA_OK;
}
#endif
