// Launchers of the batch-1 tensor-core tile kernel (decode_tc.cuh).
#include <algorithm>
#include <mutex>

#include "decode_tc.cuh"
#include "launch.cuh"

namespace va {
#ifdef VA_TC_TIMELINE
__device__ unsigned long long g_tc_timeline[kTlCtas * 16];
#endif
namespace host {

// Per (configuration, device): the dynamic shared-memory attribute is set
// once and the number of resident CTAs per SM cached.
template <class C>
int tc_ctas_per_sm(int dev, int* out) {
    static int occ[kMaxDevices] = {0};
    static std::mutex mu;
    if (occ[dev] == 0) {
        std::lock_guard<std::mutex> lock(mu);
        if (occ[dev] == 0) {
            VA_CUDA(cudaFuncSetAttribute(decode_tc_kernel<C, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            VA_CUDA(cudaFuncSetAttribute(decode_tc_kernel<C, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            int n = 0;
            VA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_tc_kernel<C, false>, C::kThreads,
                                                                  C::kSmemBytes));
            occ[dev] = std::max(1, n);
        }
    }
    *out = occ[dev];
    return VA_OK;
}

template <class C>
int launch_tc(const DecodeParams& p, cudaStream_t st) {
    int dev, occ;
    int rc = current_device(&dev);
    if (rc) return rc;
    rc = tc_ctas_per_sm<C>(dev, &occ);
    if (rc) return rc;
    CUtensorMap tmK, tmV;
    // copy boxes: kBox rows inside a page, kTcBoxC rows of a contiguous cache
    const int box = p.page_rows > 0 ? C::kBox : tc_box_rows<C>();
    rc = encode_rows_map(&tmK, p.K, p.total_rows, C::kRb, box);
    if (rc) return rc;
    rc = encode_rows_map(&tmV, p.V, p.total_rows, C::kRb, box);
    if (rc) return rc;
    const long long units = (long long)p.H * p.S;
    const int grid = (int)std::min<long long>(units, (long long)sm_count(dev) * occ);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(C::kThreads);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // one instantiation per copy path (contiguous rows or a page pool)
    if (p.page_rows > 0) VA_CUDA(cudaLaunchKernelEx(&cfg, decode_tc_kernel<C, true>, p, tmK, tmV));
    else VA_CUDA(cudaLaunchKernelEx(&cfg, decode_tc_kernel<C, false>, p, tmK, tmV));
    return VA_OK;
}

#define VA_TC_INST(...)                                                             \
    template int tc_ctas_per_sm<__VA_ARGS__>(int, int*);                           \
    template int launch_tc<__VA_ARGS__>(const DecodeParams&, cudaStream_t);
VA_TC_INST(TcCfg<Kind::Q4, 128>)
VA_TC_INST(TcCfg<Kind::Q8, 128>)
VA_TC_INST(TcCfg<Kind::Q3, 128>)
VA_TC_INST(TcCfg<Kind::Q4, 128, true>)
#undef VA_TC_INST

}  // namespace host
}  // namespace va

#ifdef VA_TC_TIMELINE
// Development builds only: copies the per-CTA timeline of the last tile-kernel
// launch (kTlCtas x 16 words) to host memory and clears it.
extern "C" int va_debug_tc_timeline(void* dst, size_t bytes) {
    if (!dst || bytes < sizeof(va::g_tc_timeline)) return VA_ERR_INVALID;
    VA_CUDA(cudaMemcpyFromSymbol(dst, va::g_tc_timeline, sizeof(va::g_tc_timeline)));
    static unsigned long long zero[va::kTlCtas * 16];
    VA_CUDA(cudaMemcpyToSymbol(va::g_tc_timeline, zero, sizeof(zero)));
    return VA_OK;
}
#endif
