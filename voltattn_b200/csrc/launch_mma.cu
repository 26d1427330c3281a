// Launchers of the grouped-query mma.sync kernel (decode_mma.cuh).
#include <algorithm>
#include <mutex>

#include "decode_mma.cuh"
#include "launch.cuh"

namespace va {
namespace host {

template <class C>
static int mma_ctas_per_sm(int dev, int* out) {
    static int occ[kMaxDevices] = {0};
    static std::mutex mu;
    if (occ[dev] == 0) {
        std::lock_guard<std::mutex> lock(mu);
        if (occ[dev] == 0) {
            VA_CUDA(cudaFuncSetAttribute(decode_mma_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            int n = 0;
            VA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_mma_kernel<C>, C::kThreads,
                                                                  C::kSmemBytes));
            occ[dev] = std::max(1, n);
        }
    }
    *out = occ[dev];
    return VA_OK;
}

template <class C>
int launch_mma(const DecodeParams& p, cudaStream_t st) {
    int dev, occ;
    int rc = current_device(&dev);
    if (rc) return rc;
    rc = mma_ctas_per_sm<C>(dev, &occ);
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
    VA_CUDA(cudaLaunchKernelEx(&cfg, decode_mma_kernel<C>, p));
    return VA_OK;
}

#define VA_MMA_INST(K)                                                                 \
    template int launch_mma<MmaCfg<K, 64, 1>>(const DecodeParams&, cudaStream_t);     \
    template int launch_mma<MmaCfg<K, 128, 1>>(const DecodeParams&, cudaStream_t);    \
    template int launch_mma<MmaCfg<K, 64, 2>>(const DecodeParams&, cudaStream_t);     \
    template int launch_mma<MmaCfg<K, 128, 2>>(const DecodeParams&, cudaStream_t);    \
    template int launch_mma<MmaCfg<K, 64, 4>>(const DecodeParams&, cudaStream_t);     \
    template int launch_mma<MmaCfg<K, 128, 4>>(const DecodeParams&, cudaStream_t);    \
    template int launch_mma<MmaCfg<K, 64, 8>>(const DecodeParams&, cudaStream_t);     \
    template int launch_mma<MmaCfg<K, 128, 8>>(const DecodeParams&, cudaStream_t);
VA_MMA_INST(Kind::Q8)
VA_MMA_INST(Kind::Q4)
VA_MMA_INST(Kind::Q3)
#undef VA_MMA_INST

}  // namespace host
}  // namespace va
