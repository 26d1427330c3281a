// Launchers of the tcgen05 prefill kernel (prefill_tc.cuh).
#include <mutex>

#include "launch.cuh"
#include "prefill_tc.cuh"

namespace va {
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
