// Streaming-family launchers for 4 query heads per KV head.
#include "launch_stream.cuh"

namespace va {
namespace host {
template int launch_stream_fmt_g<4>(int, const DecodeParams&, int, cudaStream_t);
}  // namespace host
}  // namespace va
