// Streaming-family launchers for 2 query heads per KV head.
#include "launch_stream.cuh"

namespace va {
namespace host {
template int launch_stream_fmt_g<2>(int, const DecodeParams&, int, cudaStream_t);
}  // namespace host
}  // namespace va
