// Streaming-family launchers for 8 query heads per KV head.
#include "launch_stream.cuh"

namespace va {
namespace host {
template int launch_stream_fmt_g<8>(int, const DecodeParams&, int, cudaStream_t);
}  // namespace host
}  // namespace va
