// Streaming-family launchers for one query head per KV head (batch-1
// multi-head decode), and the streaming kernel's tile sizes and occupancy
// for the split heuristic.
#include "launch_stream.cuh"

namespace va {
namespace host {

template int launch_stream_fmt_g<1>(int, const DecodeParams&, int, cudaStream_t);

int stream_cfg_tile_rows(int fmt, int D) {
    switch (fmt) {
        case VA_BF16P: return D == 128 ? StreamCfg<Kind::BF16, 128>::kTr : StreamCfg<Kind::BF16, 64>::kTr;
        case VA_F8P: return D == 128 ? StreamCfg<Kind::F8, 128>::kTr : StreamCfg<Kind::F8, 64>::kTr;
        case VA_F16P: return D == 128 ? StreamCfg<Kind::F16, 128>::kTr : StreamCfg<Kind::F16, 64>::kTr;
        case VA_Q8P: return D == 128 ? StreamCfg<Kind::Q8, 128>::kTr : StreamCfg<Kind::Q8, 64>::kTr;
        case VA_Q4P: return D == 128 ? StreamCfg<Kind::Q4, 128>::kTr : StreamCfg<Kind::Q4, 64>::kTr;
        default: return D == 128 ? StreamCfg<Kind::Q3, 128>::kTr : StreamCfg<Kind::Q3, 64>::kTr;
    }
}

int stream_cfg_occupancy(int fmt, int D, int dev, int* occ) {
    switch (fmt) {
        case VA_BF16P:
            return D == 128 ? stream_ctas_per_sm<StreamCfg<Kind::BF16, 128>>(dev, occ)
                            : stream_ctas_per_sm<StreamCfg<Kind::BF16, 64>>(dev, occ);
        case VA_F8P:
            return D == 128 ? stream_ctas_per_sm<StreamCfg<Kind::F8, 128>>(dev, occ)
                            : stream_ctas_per_sm<StreamCfg<Kind::F8, 64>>(dev, occ);
        case VA_F16P:
            return D == 128 ? stream_ctas_per_sm<StreamCfg<Kind::F16, 128>>(dev, occ)
                            : stream_ctas_per_sm<StreamCfg<Kind::F16, 64>>(dev, occ);
        case VA_Q8P:
            return D == 128 ? stream_ctas_per_sm<StreamCfg<Kind::Q8, 128>>(dev, occ)
                            : stream_ctas_per_sm<StreamCfg<Kind::Q8, 64>>(dev, occ);
        case VA_Q4P:
            return D == 128 ? stream_ctas_per_sm<StreamCfg<Kind::Q4, 128>>(dev, occ)
                            : stream_ctas_per_sm<StreamCfg<Kind::Q4, 64>>(dev, occ);
        default:
            return D == 128 ? stream_ctas_per_sm<StreamCfg<Kind::Q3, 128>>(dev, occ)
                            : stream_ctas_per_sm<StreamCfg<Kind::Q3, 64>>(dev, occ);
    }
}

}  // namespace host
}  // namespace va
