// Host-side launch layer shared by the translation units of the library:
// status helpers, device queries, consumer selection, tensor maps, and the
// launchers of each kernel family. Each family's launchers are defined and
// explicitly instantiated in a translation unit of its own (launch_*.cu),
// so the families compile in parallel; the C ABI (voltattn_api.cu) calls
// them through the declarations below.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/voltattn.h"
#include "decode_stream.cuh"
#include "formats.cuh"

namespace va {

struct PrefillParams;

namespace host {

constexpr int kMaxDevices = 64;

// Records e as this thread's last CUDA error; returns VA_ERR_CUDA.
int cuda_fail(cudaError_t e);
int last_cuda_error();

#define VA_CUDA(call)                                             \
    do {                                                          \
        const cudaError_t e__ = (call);                           \
        if (e__ != cudaSuccess) return ::va::host::cuda_fail(e__); \
    } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_device(int* dev);
int sm_count(int dev);

// Which consumer the quantized "+" formats use (VOLTATTN_CONSUMER=dp|mma|tc
// overrides where the choice applies).
enum class Consumer { kDp, kMma, kTc };
Consumer pick_consumer(Kind k, int D, int G);

// 2-D tensor map of [rows][row_bytes] uint8 codes, boxes of box_rows rows.
int encode_rows_map(CUtensorMap* m, const void* base, long long rows, int row_bytes, int box_rows);

// Kernel families (launch_tc.cu, launch_tcg.cu, launch_mma.cu,
// launch_stream_g*.cu, launch_prefill.cu).
template <class C>
int launch_tc(const DecodeParams& p, cudaStream_t st);
template <class C>
int tc_ctas_per_sm(int dev, int* out);
template <class C>
int launch_tcg(const DecodeParams& p, cudaStream_t st);
template <class C>
int launch_mma(const DecodeParams& p, cudaStream_t st);
// Streaming family for G query heads per KV head; dispatches to the tile or
// mma kernels where those serve the shape.
template <int G>
int launch_stream_fmt_g(int fmt, const DecodeParams& p, int D, cudaStream_t st);
int stream_cfg_tile_rows(int fmt, int D);
int stream_cfg_occupancy(int fmt, int D, int dev, int* occ);
int launch_prefill_fmt(int fmt, const PrefillParams& p, cudaStream_t st);
// Staged prefill: the cache converted once to fp16 rows in ws (prefill_stage_rows
// rows per KV head), then the attention with tensor copies of the tiles.
int prefill_stage_rows(int L);
size_t prefill_stage_bytes(int Hkv, int L, int D);
int launch_prefill_staged_fmt(int fmt, const PrefillParams& p, void* ws, cudaStream_t st);
// fp16 [rows][128] tensor map, 64-element x box_rows boxes, 128-byte swizzle.
int encode_f16_rows_map(CUtensorMap* m, const void* base, long long rows, int box_rows);

}  // namespace host
}  // namespace va
