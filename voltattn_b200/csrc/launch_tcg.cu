// Launchers of the grouped-query tensor-core tile kernel (decode_tcg.cuh).
#include <algorithm>
#include <mutex>

#include "decode_tcg.cuh"
#include "launch.cuh"

namespace va {
namespace host {

template <class C>
static int tcg_ctas_per_sm(int dev, int* out) {
    static int occ[kMaxDevices] = {0};
    static std::mutex mu;
    if (occ[dev] == 0) {
        std::lock_guard<std::mutex> lock(mu);
        if (occ[dev] == 0) {
            VA_CUDA(cudaFuncSetAttribute(decode_tcg_kernel<C, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            VA_CUDA(cudaFuncSetAttribute(decode_tcg_kernel<C, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            int n = 0;
            VA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_tcg_kernel<C, false>, C::kThreads,
                                                                  C::kSmemBytes));
            occ[dev] = std::max(1, n);
        }
    }
    *out = occ[dev];
    return VA_OK;
}

template <class C>
int launch_tcg(const DecodeParams& p, cudaStream_t st) {
    int dev, occ;
    int rc = current_device(&dev);
    if (rc) return rc;
    rc = tcg_ctas_per_sm<C>(dev, &occ);
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
    if (p.page_rows > 0) VA_CUDA(cudaLaunchKernelEx(&cfg, decode_tcg_kernel<C, true>, p, tmK, tmV));
    else VA_CUDA(cudaLaunchKernelEx(&cfg, decode_tcg_kernel<C, false>, p, tmK, tmV));
    return VA_OK;
}

template int launch_tcg<TcgCfg<Kind::Q4, 128, 2>>(const DecodeParams&, cudaStream_t);
template int launch_tcg<TcgCfg<Kind::Q4, 128, 4>>(const DecodeParams&, cudaStream_t);
template int launch_tcg<TcgCfg<Kind::Q4, 128, 8>>(const DecodeParams&, cudaStream_t);

}  // namespace host
}  // namespace va
