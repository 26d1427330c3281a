// Launcher of the streaming decode kernel (decode_stream.cuh), shared by the
// launch_stream_g*.cu translation units (one per query-group size G). Where
// a tensor-core kernel serves the shape, it dispatches there instead.
#pragma once

#include <algorithm>
#include <mutex>

#include "decode_stream.cuh"
#include "decode_tc.cuh"
#include "decode_tcg.cuh"
#include "launch.cuh"

namespace va {
namespace host {

template <class C>
int stream_ctas_per_sm(int dev, int* out) {
    static int occ[kMaxDevices] = {0};
    static std::mutex mu;
    if (occ[dev] == 0) {
        std::lock_guard<std::mutex> lock(mu);
        if (occ[dev] == 0) {
            VA_CUDA(cudaFuncSetAttribute(decode_stream_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes));
            int n = 0;
            VA_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_stream_kernel<C>, C::kThreads,
                                                                  C::kSmemBytes));
            occ[dev] = std::max(1, n);
        }
    }
    *out = occ[dev];
    return VA_OK;
}

template <class C>
int launch_stream(const DecodeParams& p, cudaStream_t st) {
    if constexpr (!is_float_kind(C::kKind)) {
        const Consumer c = pick_consumer(C::kKind, C::kD, C::kG);
        // the tile kernels page in 32-row copy boxes
        const bool tc_pages_ok = p.page_rows == 0 || p.page_rows % 32 == 0;
        if constexpr (C::kG == 1 && C::kD == 128 &&
                      (C::kKind == Kind::Q3 || C::kKind == Kind::Q4 || C::kKind == Kind::Q8)) {
            // tensor coordinates are 32-bit and the query is bulk-copied
            if (c == Consumer::kTc && tc_pages_ok && p.total_rows < (1ll << 31) && p.counters &&
                (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0)
                return launch_tc<TcCfg<C::kKind, 128>>(p, st);
        }
        if constexpr ((C::kG == 2 || C::kG == 4 || C::kG == 8) && C::kD == 128 && C::kKind == Kind::Q4) {
            if (c == Consumer::kTc && tc_pages_ok && p.total_rows < (1ll << 31) && p.counters &&
                (reinterpret_cast<uintptr_t>(p.q) & 15u) == 0)
                return launch_tcg<TcgCfg<Kind::Q4, 128, C::kG>>(p, st);
        }
        if (c == Consumer::kMma) return launch_mma<MmaCfg<C::kKind, C::kD, C::kG>>(p, st);
    }
    int dev, occ;
    int rc = current_device(&dev);
    if (rc) return rc;
    rc = stream_ctas_per_sm<C>(dev, &occ);
    if (rc) return rc;
    const long long units = (long long)p.H * p.S;
    const int grid = (int)std::min<long long>(units, (long long)sm_count(dev) * occ);
    // Programmatic stream serialization: the kernel waits for the preceding
    // grid before any global access (griddepcontrol.wait), so only its launch
    // latency and shared-memory prologue overlap the predecessor's tail.
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
    VA_CUDA(cudaLaunchKernelEx(&cfg, decode_stream_kernel<C>, p));
    return VA_OK;
}

template <Kind K, int G>
int launch_stream_dg(const DecodeParams& p, int D, cudaStream_t st) {
    return D == 128 ? launch_stream<StreamCfg<K, 128, G>>(p, st) : launch_stream<StreamCfg<K, 64, G>>(p, st);
}

template <int G>
int launch_stream_fmt_g(int fmt, const DecodeParams& p, int D, cudaStream_t st) {
    switch (fmt) {
        case VA_BF16P: return launch_stream_dg<Kind::BF16, G>(p, D, st);
        case VA_F8P: return launch_stream_dg<Kind::F8, G>(p, D, st);
        case VA_F16P: return launch_stream_dg<Kind::F16, G>(p, D, st);
        case VA_Q8P: return launch_stream_dg<Kind::Q8, G>(p, D, st);
        case VA_Q4P: return launch_stream_dg<Kind::Q4, G>(p, D, st);
        case VA_Q3P: return launch_stream_dg<Kind::Q3, G>(p, D, st);
        default: return VA_ERR_UNSUPPORTED;
    }
}

}  // namespace host
}  // namespace va
